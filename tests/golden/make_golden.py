"""Generate the golden fixtures by running the reference's OWN modules on the CPU.

Run where the NanoInfer source checkout is available; point
``$NANOINFER_REF`` at the directory that holds its ``nanovllm`` package (no
default: the script refuses to run without it):

    NANOINFER_REF=<checkout> TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py

``TORCHDYNAMO_DISABLE=1`` makes the reference's ``@torch.compile`` methods run
their eager bodies (inductor cannot compile on this CPU image); the numerics
are the eager code's. ``torch.distributed.get_rank/get_world_size`` are patched
to 0/1 so ``VocabParallelEmbedding`` builds without a process group, as the
reference's own tests do.

Inputs come from ``nano_vllm_multimodal_b200.workloads`` (seeded, CPU), cut to
small token counts so the fixture file stays a few MB. Output:
``tests/golden/golden.pt`` (a dict of cases, each ``{"inputs", "outputs",
"meta"}``) and ``tests/golden/MANIFEST.txt`` (sha256 of every reference source
file used). Nothing at test time reads the reference checkout.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path
from unittest.mock import patch

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("NANOINFER_REF"):
    sys.exit("make_golden.py: set NANOINFER_REF to the NanoInfer checkout (the directory holding nanovllm/)")
REF = Path(os.environ["NANOINFER_REF"])
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

from nano_vllm_multimodal_b200 import workloads as W  # noqa: E402

SOURCES = [
    "nanovllm/layers/layernorm.py",
    "nanovllm/layers/activation.py",
    "nanovllm/layers/rotary_embedding.py",
    "nanovllm/layers/multimodal_rotary_embedding.py",
    "nanovllm/layers/embed_head.py",
    "nanovllm/layers/paged_kv/base.py",
    "nanovllm/layers/paged_kv/pytorch_backend.py",
    "nanovllm/models/qwen3_vl.py",
    "nanovllm/models/qwen3.py",
    "nanovllm/models/qwen25_vl.py",
    "nanovllm/engine/model_runner.py",
    "nanovllm/multimodal/runtime.py",
    "nanovllm/layers/attention.py",
    "nanovllm/utils/context.py",
]


def _ref():
    from nanovllm.layers.activation import SiluAndMul
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.multimodal_rotary_embedding import (
        MultimodalRotaryEmbedding, apply_multimodal_rotary_emb)
    from nanovllm.layers.paged_kv.pytorch_backend import PyTorchPagedKVBackend
    from nanovllm.layers.rotary_embedding import RotaryEmbedding
    from nanovllm.engine.model_runner import (
        VisualReplacement, VisualReplacementPlan, build_planned_visual_embeddings)
    from nanovllm.models.qwen3_vl import Qwen3VLLanguageModel, Qwen3VLTextRMSNorm
    from nanovllm.multimodal.runtime import VisionFeatureBundle
    from nanovllm.layers.attention import SDPAAttention
    from nanovllm.utils.context import reset_context, set_context
    with patch("torch.distributed.get_rank", return_value=0), \
            patch("torch.distributed.get_world_size", return_value=1):
        from nanovllm.layers.embed_head import VocabParallelEmbedding
    return dict(RMSNorm=RMSNorm, SiluAndMul=SiluAndMul, RotaryEmbedding=RotaryEmbedding,
                MRoPE=MultimodalRotaryEmbedding, apply_mrope=apply_multimodal_rotary_emb,
                Store=PyTorchPagedKVBackend, TextNorm=Qwen3VLTextRMSNorm,
                add_deepstack=Qwen3VLLanguageModel._add_deepstack_rows,
                Embedding=VocabParallelEmbedding, VisualReplacement=VisualReplacement,
                VisualReplacementPlan=VisualReplacementPlan, Bundle=VisionFeatureBundle,
                build_visual=build_planned_visual_embeddings, SDPA=SDPAAttention,
                set_context=set_context, reset_context=reset_context)


def _rms(R, hidden, weight, eps=1e-6):
    m = R["RMSNorm"](hidden, eps=eps).to(torch.bfloat16)
    with torch.no_grad():
        m.weight.copy_(weight)
    return m


def _text(R, hidden, weight, eps=1e-6):
    m = R["TextNorm"](hidden, eps=eps).to(weight.dtype)
    with torch.no_grad():
        m.weight.copy_(weight)
    return m


def _split(qkv, shape):
    q_size = shape.num_heads * shape.head_dim
    kv_size = shape.num_kv_heads * shape.head_dim
    q, k, v = qkv.split([q_size, kv_size, kv_size], dim=-1)
    return (q.view(-1, shape.num_heads, shape.head_dim),
            k.view(-1, shape.num_kv_heads, shape.head_dim),
            v.view(-1, shape.num_kv_heads, shape.head_dim))


def _small_cache(shape, blocks=4, block_size=16, fill=-3.0):
    c = (blocks, block_size, shape.num_kv_heads, shape.head_dim)
    return torch.full(c, fill, dtype=torch.bfloat16), torch.full(c, fill, dtype=torch.bfloat16)


def _slots(seed, total, n, skip_every=None):
    g = torch.Generator().manual_seed(seed)
    s = torch.randperm(total, generator=g)[:n].to(torch.int32)
    if skip_every:
        s[::skip_every] = -1
    return s


def build():
    R = _ref()
    cases = {}
    no_grad = torch.no_grad()
    no_grad.__enter__()

    # ---- a1/a2: RMSNorm (Qwen3 hidden norms), C1 rows
    d = W.make_layer_inputs(1, tokens=32, cache=False)
    m = _rms(R, 1024, d["w_in"])
    y, res = m(d["hidden"], d["residual"])
    cases["rmsnorm_add_c1"] = dict(inputs=dict(x=d["hidden"], residual=d["residual"], weight=d["w_in"]),
                                   outputs=dict(y=y, residual=res), meta=dict(eps=1e-6))
    cases["rmsnorm_c1"] = dict(inputs=dict(x=d["hidden"], weight=d["w_in"]),
                               outputs=dict(y=m(d["hidden"])), meta=dict(eps=1e-6))
    # a2 on strided per-head views (Qwen3 q/k norm, nanovllm/models/qwen3.py:82-84)
    shp = W.C1
    q, k, v = _split(d["qkv"], shp)
    qn = _rms(R, 128, d["q_weight"])(q)
    kn = _rms(R, 128, d["k_weight"])(k)
    cases["qknorm_c1"] = dict(inputs=dict(qkv=d["qkv"], q_weight=d["q_weight"], k_weight=d["k_weight"]),
                              outputs=dict(q=qn, k=kn), meta=dict(eps=1e-6, heads=(16, 8)))

    # ---- a4: SiluAndMul (eager = two roundings)
    xs = d["gate_up"][:16].contiguous()
    cases["silu_c1"] = dict(inputs=dict(x=xs), outputs=dict(y=R["SiluAndMul"]()(xs)), meta={})

    # ---- a5: 1-D RoPE (C1 positions 0..31 plus large positions of C2)
    rope = R["RotaryEmbedding"](128, 128, 40960, 1e6)
    pos = torch.cat((d["positions"][:16], torch.tensor([8191, 40959, 32767, 12345, 1, 0, 4096, 20000,
                                                        40958, 39999, 7, 1023, 2047, 30000, 5, 9])))
    qr, kr = rope.forward(pos, qn, kn)
    table = rope.cos_sin_cache
    cases["rope_c1"] = dict(
        inputs=dict(positions=pos, q=qn, k=kn),
        outputs=dict(q=qr, k=kr, table_rows=table[pos].clone()),
        meta=dict(base=1e6, max_position=40960,
                  table_sha256=hashlib.sha256(table.contiguous().numpy().tobytes()).hexdigest()))

    # ---- a3: Qwen3VLTextRMSNorm on C3 rows and per-head views
    d3 = W.make_layer_inputs(3, tokens=16, cache=False)
    tn = _text(R, 2048, d3["w_in"])
    h1 = d3["hidden"] + d3["residual"]
    cases["textnorm_c3"] = dict(inputs=dict(x=d3["hidden"], residual=d3["residual"], weight=d3["w_in"]),
                                outputs=dict(y=tn(d3["hidden"]), y_add=tn(h1), sum=h1), meta=dict(eps=1e-6))
    q3, k3, v3 = _split(d3["qkv"], W.C3)
    q3n = _text(R, 128, d3["q_weight"])(q3)
    k3n = _text(R, 128, d3["k_weight"])(k3)

    # ---- a6: interleaved M-RoPE (Qwen3-VL), C3 positions across text/image boundary
    pos3 = W.positions_for(3, W.C3, W._Seeds(3, "cpu"), 2048)[:, 504:520].contiguous()
    mr = R["MRoPE"](head_dim=128, base=5e6, sections=(24, 20, 20), strategy="interleaved")
    q3r, k3r = mr(pos3, q3n, k3n)
    cos3, sin3 = mr.cos_sin(pos3, torch.bfloat16)
    cases["mrope_interleaved_c3"] = dict(
        inputs=dict(positions=pos3, q=q3n, k=k3n),
        outputs=dict(q=q3r, k=k3r, cos=cos3, sin=sin3, inv_freq=mr.inv_freq.clone()),
        meta=dict(base=5e6, sections=(24, 20, 20), strategy="interleaved"))

    # ---- a6: chunked M-RoPE (Qwen2.5-VL), C4 positions incl. decode tokens
    d4 = W.make_layer_inputs(4, cache=False, tokens=8312)
    sel = torch.cat((torch.arange(1016, 1032), torch.arange(8300, 8312)))
    qkv4 = d4["qkv"][sel].contiguous()
    pos4 = d4["positions"][:, sel].contiguous()
    q4, k4, v4 = _split(qkv4, W.C4)
    mc = R["MRoPE"](head_dim=128, base=1e6, sections=(16, 24, 24))
    q4r, k4r = mc(pos4, q4, k4)
    cases["mrope_chunked_c4"] = dict(
        inputs=dict(positions=pos4, q=q4.contiguous(), k=k4.contiguous()),
        outputs=dict(q=q4r, k=k4r, inv_freq=mc.inv_freq.clone()),
        meta=dict(base=1e6, sections=(16, 24, 24), strategy="chunked"))

    # ---- a7/a11: paged store + gather (C2 semantics: 10% slots skipped; small cache)
    d2 = W.make_layer_inputs(2, tokens=40, cache=False)
    q2, k2, v2 = _split(d2["qkv"], W.C2)
    kc, vc = _small_cache(W.C2)
    slots = _slots(2001, kc.shape[0] * kc.shape[1], 40, skip_every=10)
    store = R["Store"]()
    kc_o, vc_o = kc.clone(), vc.clone()
    store.store(k2, v2, kc_o, vc_o, slots)
    table = torch.tensor([2, 0, 3, 1], dtype=torch.int32)
    gathered = store.gather(kc_o, table, 50)
    cases["paged_c2"] = dict(
        inputs=dict(qkv=d2["qkv"], slot_mapping=slots, block_table=table),
        outputs=dict(key_cache=kc_o, value_cache=vc_o, gathered=gathered.contiguous()),
        meta=dict(heads=(16, 8), sequence_length=50, cache_shape=tuple(kc.shape), cache_fill=-3.0))

    # ---- a10: embedding row gather (C2 distribution, vocab cut to 512 rows)
    with patch("torch.distributed.get_rank", return_value=0), \
            patch("torch.distributed.get_world_size", return_value=1):
        emb = R["Embedding"](128, 1024).to(torch.bfloat16)
    g = torch.Generator().manual_seed(2100)
    wemb = (torch.randn(128, 1024, generator=g) * 0.02).to(torch.bfloat16)
    emb.weight.copy_(wemb)
    ids = torch.randint(0, 128, (40,), generator=g)
    cases["embedding_c2"] = dict(inputs=dict(weight=wemb, ids=ids), outputs=dict(y=emb(ids)), meta={})

    # ---- a9: DeepStack add (C3 semantics: sorted image rows)
    g = torch.Generator().manual_seed(3100)
    hs = torch.randn(48, 256, generator=g).to(torch.bfloat16)
    rows = torch.tensor(list(range(8, 24)) + list(range(30, 38)), dtype=torch.int64)
    vis = torch.randn(rows.numel(), 256, generator=g).to(torch.bfloat16)
    cases["deepstack_c3"] = dict(inputs=dict(hidden=hs, rows=rows, vis=vis),
                                 outputs=dict(y=R["add_deepstack"](hs, rows, vis)), meta={})

    # ---- (f) visual-embedding merge of a packed prefill: two feature keys interleaved in
    # the plan, one of them float32 (converted to the bf16 token dtype), 3 DeepStack layers,
    # feature rows offset as after a chunked prefill
    g = torch.Generator().manual_seed(3200)
    tok = torch.randn(40, 64, generator=g).to(torch.bfloat16)
    fa = torch.randn(4, 12, 64, generator=g).to(torch.bfloat16)   # final + 3 layers
    fb = torch.randn(4, 10, 64, generator=g)                      # float32
    keys = ("vision:a", "vision:b")
    plan_rows = ([(3 + i, 0, 2 + i) for i in range(6)] + [(10 + i, 1, i) for i in range(4)]
                 + [(20 + i, 0, 8 + i) for i in range(4)])
    plan = R["VisualReplacementPlan"](
        replacements=tuple(R["VisualReplacement"](output_row=o, feature_key=keys[k], feature_row=f)
                           for o, k, f in plan_rows),
        required_feature_keys=keys, prefix_skipped_features=0)
    bundles = {keys[0]: R["Bundle"](fa[0], tuple(fa[1:])), keys[1]: R["Bundle"](fb[0], tuple(fb[1:]))}
    vm = R["build_visual"](tok, plan, bundles)
    cases["visual_merge_c3"] = dict(
        inputs=dict(tokens=tok, feature_a=fa, feature_b=fb,
                    plan=torch.tensor(plan_rows, dtype=torch.int64)),
        outputs=dict(final_embedding=vm.final_embedding, deepstack=torch.stack(vm.deepstack_embeddings),
                     visual_rows=vm.visual_rows),
        meta=dict(keys=keys))

    # ---- (f) paged decode attention: the reference's SDPA decode branch (the numerical
    # reference of flash_attn_with_kvcache), GQA 16/8, head_dim 128, 16-token blocks,
    # ragged contexts incl. a one-token context, non-sequential block tables
    g = torch.Generator().manual_seed(3300)
    B, NQ_, NKV_, D_, BS_, NB_ = 6, 16, 8, 128, 16, 24
    kc = torch.randn(NB_, BS_, NKV_, D_, generator=g).to(torch.bfloat16)
    vc = torch.randn(NB_, BS_, NKV_, D_, generator=g).to(torch.bfloat16)
    lens = torch.tensor([1, 17, 40, 5, 64, 33], dtype=torch.int32)
    tables = torch.stack([torch.randperm(NB_, generator=g)[:4] for _ in range(B)]).to(torch.int32)
    qd = torch.randn(B, NQ_, D_, generator=g).to(torch.bfloat16)
    attn = R["SDPA"](NQ_, D_, D_ ** -0.5, NKV_)
    attn.k_cache, attn.v_cache = kc, vc
    attn.paged_kv_backend = R["Store"]()
    R["set_context"](False, slot_mapping=torch.full((B,), -1, dtype=torch.int32), context_lens=lens,
                     block_tables=tables)
    od = attn(qd, torch.zeros(B, NKV_, D_, dtype=torch.bfloat16), torch.zeros(B, NKV_, D_, dtype=torch.bfloat16))
    R["reset_context"]()
    cases["decode_attention_c2"] = dict(
        inputs=dict(q=qd, k_cache=kc, v_cache=vc, context_lens=lens, block_tables=tables),
        outputs=dict(out=od), meta=dict(scale=D_ ** -0.5))

    # ---- a8: fused attention prologues, composed from the reference modules
    def fused(dd, shape, norm_mod, rope_fn, slots_seed, skip):
        q_, k_, v_ = _split(dd["qkv"], shape)
        if norm_mod is not None:
            q_ = norm_mod(128, dd["q_weight"])(q_)
            k_ = norm_mod(128, dd["k_weight"])(k_)
        q_, k_ = rope_fn(dd["positions"], q_, k_)
        kc_, vc_ = _small_cache(shape)
        sl = _slots(slots_seed, kc_.shape[0] * kc_.shape[1], q_.shape[0], skip_every=skip)
        kco, vco = kc_.clone(), vc_.clone()
        R["Store"]().store(k_, v_, kco, vco, sl)
        return (dict(qkv=dd["qkv"], positions=dd["positions"], q_weight=dd["q_weight"],
                     k_weight=dd["k_weight"], slot_mapping=sl),
                dict(q=q_, k=k_, key_cache=kco, value_cache=vco))

    d1 = W.make_layer_inputs(1, tokens=16, cache=False)
    i, o = fused(d1, W.C1, lambda h, w: _rms(R, h, w), rope.forward, 1001, 5)
    cases["fused_qwen3_c1"] = dict(inputs=i, outputs=o, meta=dict(heads=(16, 8), norm="rms", rope="table",
                                                                  base=1e6, max_position=40960, eps=1e-6,
                                                                  cache_shape=(4, 16, 8, 128), cache_fill=-3.0))
    d3s = dict(d3)
    d3s["positions"] = pos3
    i, o = fused(d3s, W.C3, lambda h, w: _text(R, h, w), mr, 3001, 7)
    cases["fused_qwen3vl_c3"] = dict(inputs=i, outputs=o, meta=dict(heads=(16, 8), norm="text",
                                                                    rope="interleaved", base=5e6,
                                                                    sections=(24, 20, 20), eps=1e-6,
                                                                    cache_shape=(4, 16, 8, 128), cache_fill=-3.0))
    d4s = dict(qkv=qkv4, positions=pos4, q_weight=d4["q_weight"], k_weight=d4["k_weight"])
    i, o = fused(d4s, W.C4, None, mc, 4001, 9)
    cases["fused_qwen25vl_c4"] = dict(inputs=i, outputs=o, meta=dict(heads=(16, 2), norm=None,
                                                                     rope="chunked", base=1e6,
                                                                     sections=(16, 24, 24), eps=1e-6,
                                                                     cache_shape=(4, 16, 2, 128), cache_fill=-3.0))
    no_grad.__exit__(None, None, None)
    return cases


def main():
    cases = build()
    torch.save(cases, HERE / "golden.pt")
    lines = [f"{hashlib.sha256((REF / s).read_bytes()).hexdigest()}  {s}" for s in SOURCES]
    (HERE / "MANIFEST.txt").write_text(
        "# reference sources that produced golden.pt (sha256, path inside the NanoInfer project)\n"
        + "\n".join(lines) + "\n")
    size = (HERE / "golden.pt").stat().st_size
    print(f"wrote {len(cases)} cases, {size / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
