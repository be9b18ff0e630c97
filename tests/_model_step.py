"""Runs small models built from the reference's own model code for one prefill
step and one decode step, and saves what they produced.

Usage: ``python tests/_model_step.py REF_DIR DEVICE MODE OUT.pt``

* ``REF_DIR``: a NanoInfer checkout or install (the directory holding ``nanovllm``)
* ``DEVICE``: ``cpu`` or ``cuda``
* ``MODE``:
  * ``reference``: the reference's model classes and layers, untouched
  * ``perop``: after ``install(fused=False)``, which swaps in each op's kernel
    while the model code calls the ops one at a time
  * ``fused``: after ``install()``, where the model classes' forwards run the
    fused prologue (q/k norm, rotary and K/V store in one launch) and fold the
    Qwen3-VL residual adds and DeepStack rows into the norms
  * ``truth``: the reference's model in float64 (the same bf16 weights and
    inputs, widened; its norms compute in float32), attention as float64
    SDPA: the yardstick both bf16 runs are measured against. (Not float32:
    there the reference's ``RMSNorm.add_rms_forward`` would update its input
    in place, since ``x.float()`` returns ``x`` itself, and the residual
    would alias the normalised output.)

On ``cpu`` the package's ops are replaced by CPU stand-ins computed with the
oracle in the reference's own rounding order. That makes the fused and per-op
routes comparable bit for bit with the reference's CPU run, and it shows which
ops each route calls. Attention itself (flash-attn, which needs a GPU) is a
CPU SDPA stand-in in every mode. On ``cuda`` everything is real: this
package's kernels, and flash-attn for prefill attention.

Per model (Qwen3, Qwen2.5-VL, Qwen3-VL) the script saves the output of every
decoder layer (the completed ``x + residual``), the final hidden states of
both steps, and the K/V caches after each step. It prints one JSON line with
the op call counts (CPU) or ``{}``.
"""

from __future__ import annotations

import json
import os
import sys
import zlib
from collections import Counter
from pathlib import Path
from types import SimpleNamespace

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

ROOT = Path(__file__).resolve().parents[1]
REF_DIR, DEVICE, MODE, OUT = sys.argv[1], sys.argv[2], sys.argv[3], sys.argv[4]
sys.path[:0] = [str(ROOT), REF_DIR]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

dist.get_rank = lambda *a, **k: 0          # tensor-parallel layers build without a process group
dist.get_world_size = lambda *a, **k: 1

import nanovllm.layers.attention as ref_attention  # noqa: E402
import nanovllm.models.qwen3 as q3  # noqa: E402
import nanovllm.models.qwen3_vl as q3vl  # noqa: E402
import nanovllm.models.qwen25_vl as q25  # noqa: E402
from nanovllm.layers.paged_kv.pytorch_backend import PyTorchPagedKVBackend  # noqa: E402
from nanovllm.utils.context import reset_context, set_context  # noqa: E402

CALLS: Counter = Counter()

if MODE not in ("reference", "truth"):
    from nano_vllm_multimodal_b200.integration import install
    install(fused=(MODE == "fused"))

BF16 = torch.bfloat16
DT = torch.float64 if MODE == "truth" else BF16  # the models' compute dtype
HIDDEN, HEADS, KV_HEADS, HEAD_DIM, INTER, VOCAB = 512, 4, 2, 128, 1024, 128
BLOCKS, BLOCK_SIZE = 4, 256


# ----------------------------------------------------------------------------- CPU stand-ins


def _cpu_stand_ins():
    """Oracle-backed replacements of ``nano_vllm_multimodal_b200.ops`` (order
    "torch": the rounding order of the reference's eager CPU code)."""
    from nano_vllm_multimodal_b200 import ops
    from oracle import ops as o

    def counted(name, fn):
        def wrapper(*a, **k):
            CALLS[name] += 1
            return fn(*a, **k)
        return wrapper

    def add_rms_norm(x, residual, weight, eps, round_sum=False):
        if round_sum:
            return o.add_text_rms_norm(x, residual, weight, eps)
        return o.add_rms_norm(x, residual, weight, eps)

    def deepstack_row_index(rows, tokens):
        index = torch.full((tokens,), -1, dtype=torch.int32)
        index[rows.long()] = torch.arange(rows.numel(), dtype=torch.int32)
        return index

    def add_rms_norm_deepstack(x, residual, weight, eps, vis, row_index):
        rows = torch.nonzero(row_index >= 0).flatten()
        return o.add_text_rms_norm_deepstack(x, residual, weight, eps, rows, vis[row_index[rows].long()])

    def qk_prologue(q, k, *, v=None, positions=None, q_weight=None, k_weight=None, eps=1e-6,
                    rope_mode=0, cos_sin_cache=None, inv_freq=None, sections=(), key_cache=None,
                    value_cache=None, slot_mapping=None, variant=0, emit_k=True):
        CALLS["qk_prologue.store" if key_cache is not None else "qk_prologue.nostore"] += 1
        if not emit_k:
            CALLS["qk_prologue.cache_only_k"] += 1
        if q_weight is not None:
            q, k = o.rms_norm(q, q_weight, eps), o.rms_norm(k, k_weight, eps)
        if rope_mode == ops.ROPE_TABLE:
            q, k = o.apply_rope(positions, q, k, cos_sin_cache)
        elif rope_mode in (ops.ROPE_MROPE_CHUNKED, ops.ROPE_MROPE_INTERLEAVED):
            strategy = "interleaved" if rope_mode == ops.ROPE_MROPE_INTERLEAVED else "chunked"
            q, k = o.mrope_forward(positions, q, k, inv_freq, tuple(sections), strategy)
        if key_cache is not None:
            o.paged_store_(k, v, key_cache, value_cache, slot_mapping)
        return q, (k if emit_k else None)

    def embedding(ids, weight, vocab_start=0, vocab_end=None, mask=False):
        return o.embedding(ids - vocab_start, weight)

    stand_ins = {
        "rms_norm": lambda x, w, eps: o.rms_norm(x, w, eps),
        "add_rms_norm": add_rms_norm,
        "add_rms_norm_deepstack": add_rms_norm_deepstack,
        "deepstack_row_index": deepstack_row_index,
        "deepstack_add": o.add_deepstack_rows,
        "silu_and_mul": o.silu_and_mul,
        "qk_prologue": qk_prologue,
        "paged_store": lambda k, v, kc, vc, s: o.paged_store_(k, v, kc, vc, s),
        "embedding": embedding,
    }
    for name, fn in stand_ins.items():
        setattr(ops, name, counted(name, fn))


def _sdpa_varlen(q, k, v, *, max_seqlen_q, cu_seqlens_q, max_seqlen_k, cu_seqlens_k, softmax_scale,
                 causal, block_table=None):
    """CPU stand-in for flash-attn's varlen prefill (causal, grouped-query)."""
    assert block_table is None and causal
    CALLS["attention.prefill"] += 1
    out = torch.empty_like(q)
    dev = q.device
    group = q.shape[1] // k.shape[1]
    for i in range(cu_seqlens_q.numel() - 1):
        qs, qe = int(cu_seqlens_q[i]), int(cu_seqlens_q[i + 1])
        ks, ke = int(cu_seqlens_k[i]), int(cu_seqlens_k[i + 1])
        qi = q[qs:qe].double().transpose(0, 1)
        ki = k[ks:ke].double().repeat_interleave(group, dim=1).transpose(0, 1)
        vi = v[ks:ke].double().repeat_interleave(group, dim=1).transpose(0, 1)
        s = qi @ ki.transpose(1, 2) * softmax_scale
        mask = torch.ones(qe - qs, ke - ks, dtype=torch.bool, device=dev).tril(diagonal=(ke - ks) - (qe - qs))
        s = s.masked_fill(~mask, float("-inf"))
        out[qs:qe] = (torch.softmax(s, dim=-1) @ vi).transpose(0, 1).to(q.dtype)
    return out


def _decode_attention(q, k_cache, v_cache, *, cache_seqlens, block_table, softmax_scale, causal):
    """CPU stand-in for flash-attn's paged decode (one query token per request)."""
    from oracle import ops as o
    CALLS["attention.decode"] += 1
    return o.paged_decode_attention(q[:, 0], k_cache, v_cache, cache_seqlens, block_table,
                                    softmax_scale).unsqueeze(1)


def _decode_attention_device(q, k_cache, v_cache, *, cache_seqlens, block_table, softmax_scale, causal):
    """Paged decode in float64 with torch ops on q's device (the ``truth`` run)."""
    CALLS["attention.decode"] += 1
    bs = k_cache.shape[1]
    group = q.shape[2] // k_cache.shape[2]
    out = torch.zeros_like(q)
    for b in range(q.shape[0]):
        n = int(cache_seqlens[b])
        t = torch.arange(n, device=q.device)
        slots = block_table[b].long()[t // bs] * bs + t % bs
        k = k_cache.flatten(0, 1)[slots].double().repeat_interleave(group, dim=1)  # [n, heads, D]
        v = v_cache.flatten(0, 1)[slots].double().repeat_interleave(group, dim=1)
        s = torch.einsum("hd,nhd->hn", q[b, 0].double(), k) * softmax_scale
        out[b, 0] = torch.einsum("hn,nhd->hd", torch.softmax(s, dim=-1), v).to(q.dtype)
    return out


if DEVICE == "cpu":
    if MODE not in ("reference", "truth"):
        _cpu_stand_ins()
    ref_attention.flash_attn_varlen_func = _sdpa_varlen
    ref_attention.flash_attn_with_kvcache = _decode_attention
elif MODE == "truth":
    ref_attention.flash_attn_varlen_func = _sdpa_varlen
    ref_attention.flash_attn_with_kvcache = _decode_attention_device


# ----------------------------------------------------------------------------- models


def _configs():
    common = dict(hidden_size=HIDDEN, num_attention_heads=HEADS, num_key_value_heads=KV_HEADS,
                  intermediate_size=INTER, hidden_act="silu", rms_norm_eps=1e-6, vocab_size=VOCAB,
                  max_position_embeddings=4096)
    qwen3 = SimpleNamespace(**common, num_hidden_layers=2, head_dim=HEAD_DIM, attention_bias=False,
                            rope_theta=1e6, rope_scaling=None, tie_word_embeddings=False)
    qwen25 = SimpleNamespace(**common, num_hidden_layers=2, rope_theta=1e6, tie_word_embeddings=False,
                             rope_scaling={"type": "mrope", "mrope_section": [16, 24, 24]})
    qwen3vl = SimpleNamespace(**common, num_hidden_layers=3, head_dim=HEAD_DIM, attention_bias=False,
                              rope_theta=5e6, tie_word_embeddings=True,
                              rope_scaling={"rope_type": "default", "mrope_section": [24, 20, 20],
                                            "mrope_interleaved": True})
    return {
        "qwen3": (lambda: q3.Qwen3ForCausalLM(qwen3), 1),
        "qwen25_vl": (lambda: q25.Qwen25VLForCausalLM(qwen25), 3),
        "qwen3_vl": (lambda: q3vl.Qwen3VLForCausalLM(qwen3vl), 3),
    }


def _seeded(shape, seed, *, mean=0.0, std=1.0, dtype=BF16):
    """bf16 values (widened to ``dtype`` in the float32 run, so every run sees the same numbers)."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std + mean).to(BF16).to(dtype)


def _init_weights(model):
    """Every parameter from a generator seeded by its name: the same weights in
    every mode, since the parameter names do not change."""
    with torch.no_grad():
        for name, p in model.named_parameters():
            seed = zlib.crc32(name.encode())
            if name.endswith("norm.weight"):
                p.copy_(_seeded(p.shape, seed, mean=1.0, std=0.1, dtype=p.dtype))
            elif name.endswith("bias"):
                p.copy_(_seeded(p.shape, seed, std=0.02, dtype=p.dtype))
            elif p.dim() == 2 and "embed" not in name and "lm_head" not in name:
                p.copy_(_seeded(p.shape, seed, std=p.shape[1] ** -0.5, dtype=p.dtype))
            else:
                p.copy_(_seeded(p.shape, seed, dtype=p.dtype))


def _attach_caches(model, device):
    caches = []
    backend = PyTorchPagedKVBackend()
    for module in model.modules():
        if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
            k = torch.full((BLOCKS, BLOCK_SIZE, KV_HEADS, HEAD_DIM), -3.0, dtype=DT, device=device)
            v = torch.full_like(k, -3.0)
            module.k_cache, module.v_cache = k, v
            if hasattr(module, "paged_kv_backend"):
                module.paged_kv_backend = backend
            caches.append((k, v))
    return caches


def _record_layers(model, sink):
    layers = [m for name, m in model.named_modules() if name.endswith(tuple(f"layers.{i}" for i in range(8)))]

    def hook(_module, _inputs, output):
        x, residual = output
        sink.append((x if residual is None else x + residual).detach().clone())

    return [layer.register_forward_hook(hook) for layer in layers]


def _run(name, build, axes, device):
    torch.manual_seed(0)
    torch.set_default_dtype(DT)
    torch.set_default_device(device)
    try:
        model = build()
    finally:
        torch.set_default_device("cpu")
        torch.set_default_dtype(torch.float32)
    model = model.to(device)
    _init_weights(model)
    caches = _attach_caches(model, device)
    seed = zlib.crc32(name.encode())
    out = {}

    # prefill: two sequences (9 and 14 tokens) in blocks 2 and 0; one padding slot (-1)
    lens, blocks = [9, 14], [2, 0]
    tokens = sum(lens)
    ids = torch.randint(0, VOCAB, (tokens,), generator=torch.Generator().manual_seed(seed))
    slots = torch.cat([torch.arange(n) + b * BLOCK_SIZE for n, b in zip(lens, blocks)]).to(torch.int32)
    slots[5] = -1
    pos1 = torch.cat([torch.arange(n) for n in lens])
    if axes == 1:
        positions = pos1
    else:  # seq 1 holds a 2x3 image grid at tokens 4..9 of its span: t fixed, h/w on the grid
        positions = pos1.repeat(3, 1).clone()
        start = lens[0] + 4
        grid = torch.arange(6)
        positions[0, start:start + 6] = 4
        positions[1, start:start + 6] = 4 + grid // 3
        positions[2, start:start + 6] = 4 + grid % 3
    cu = torch.tensor([0, lens[0], tokens], dtype=torch.int32)
    kwargs = {}
    if name == "qwen3_vl":
        rows = torch.arange(lens[0] + 4, lens[0] + 10, dtype=torch.long)
        kwargs = dict(visual_token_rows=rows.to(device),
                      deepstack_visual_embeds=tuple(_seeded((rows.numel(), HIDDEN), seed + 1 + j,
                                                            dtype=DT).to(device) for j in range(3)))
    layer_out = []
    hooks = _record_layers(model, layer_out)
    with torch.inference_mode():
        set_context(True, cu.to(device), cu.to(device), max(lens), max(lens), slots.to(device))
        out["prefill"] = model(ids.to(device), positions.to(device), **kwargs).float().cpu()
        out["prefill_layers"] = [t.float().cpu() for t in layer_out]
        out["prefill_k"] = [k.float().cpu() for k, _ in caches]
        out["prefill_v"] = [v.float().cpu() for _, v in caches]
        layer_out.clear()

        # decode: one new token per sequence
        ids = torch.randint(0, VOCAB, (2,), generator=torch.Generator().manual_seed(seed + 9))
        slots = torch.tensor([b * BLOCK_SIZE + n for n, b in zip(lens, blocks)], dtype=torch.int32)
        pos = torch.tensor(lens)
        positions = pos if axes == 1 else pos.repeat(3, 1)
        context_lens = torch.tensor([n + 1 for n in lens], dtype=torch.int32)
        tables = torch.tensor([[b] for b in blocks], dtype=torch.int32)
        set_context(False, slot_mapping=slots.to(device), context_lens=context_lens.to(device),
                    block_tables=tables.to(device))
        out["decode"] = model(ids.to(device), positions.to(device)).float().cpu()
        out["decode_layers"] = [t.float().cpu() for t in layer_out]
        out["decode_k"] = [k.float().cpu() for k, _ in caches]
        out["decode_v"] = [v.float().cpu() for _, v in caches]
        reset_context()
    for h in hooks:
        h.remove()
    return out


results = {name: _run(name, build, axes, DEVICE) for name, (build, axes) in _configs().items()}
torch.save(results, OUT)
print(json.dumps(dict(CALLS)))
