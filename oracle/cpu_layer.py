"""One fused decoder layer of the reference's CPU path, for the timed CPU baseline.

TEST INFRASTRUCTURE ONLY: ``bench.py``'s ``cpu_baseline`` leg and its
``--impl reference`` arm time this on the host cores; nothing in the product
package imports it.

Two kinds, the same layer:

* ``"reference"``: the reference's own modules, imported from an install of
  NanoInfer (``$NANOINFER_REF`` or the git-ignored ``baseline/_ref``):
  ``nanovllm.layers.layernorm.RMSNorm``, ``nanovllm.models.qwen3_vl.
  Qwen3VLTextRMSNorm``, ``nanovllm.layers.rotary_embedding.get_rope``,
  ``nanovllm.layers.multimodal_rotary_embedding.MultimodalRotaryEmbedding``,
  ``nanovllm.layers.activation.SiluAndMul`` and
  ``nanovllm.layers.paged_kv.pytorch_backend.PyTorchPagedKVBackend`` (store and
  gather; the Triton default refuses CPU tensors). ``@torch.compile`` is
  switched off (``torch._dynamo.config.disable``, the same as
  ``TORCHDYNAMO_DISABLE=1``): inductor cannot compile on these CPU images, and
  the eager bodies are the code being timed.
* ``"port"``: the oracle's restatement of the same ops (``oracle.ops``), where
  no install is present.

The layer is the elementwise part of one decoder layer as the reference's
models call it (``nanovllm/models/qwen3.py:72-88,160-172``,
``qwen3_vl.py:160-180,226-240``, ``qwen25_vl.py:62-78,112-122``): residual
add + input norm, per-head q/k norm (Qwen3, Qwen3-VL), RoPE / M-RoPE, paged
K/V store, residual add + post-attention norm, SiluAndMul. The projections
are inputs.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]


def find_reference() -> Path | None:
    """The directory holding an importable ``nanovllm`` package, if any."""
    for cand in (os.environ.get("NANOINFER_REF"), ROOT / "baseline" / "_ref"):
        if cand and (Path(cand) / "nanovllm" / "__init__.py").is_file():
            return Path(cand)
    return None


_REF = None


def load_reference():
    """Import the reference's layer modules (once); ``None`` if unavailable."""
    global _REF
    if _REF is not None:
        return _REF or None
    ref_dir = find_reference()
    if ref_dir is None:
        _REF = False
        return None
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    import torch._dynamo
    torch._dynamo.config.disable = True
    import torch.distributed as dist
    if not dist.is_initialized():  # tensor-parallel layers build without a process group
        dist.get_rank = lambda *a, **k: 0
        dist.get_world_size = lambda *a, **k: 1
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    try:
        from nanovllm.layers import activation, layernorm, multimodal_rotary_embedding, rotary_embedding
        from nanovllm.layers.paged_kv.pytorch_backend import PyTorchPagedKVBackend
        from nanovllm.models import qwen3_vl
    except Exception:  # an incomplete install: time the port instead
        _REF = False
        return None
    _REF = dict(RMSNorm=layernorm.RMSNorm, TextNorm=qwen3_vl.Qwen3VLTextRMSNorm,
                get_rope=rotary_embedding.get_rope,
                MRoPE=multimodal_rotary_embedding.MultimodalRotaryEmbedding,
                SiluAndMul=activation.SiluAndMul, backend=PyTorchPagedKVBackend(), dir=str(ref_dir))
    return _REF


class CpuLayer:
    """``layer(inputs)`` runs one fused layer on the CPU; ``inputs`` as built by
    ``nano_vllm_multimodal_b200.workloads.make_layer_inputs`` (the caches are
    written in place). ``kind``: ``"reference"``, ``"port"`` or ``"auto"``."""

    def __init__(self, shape, inputs, kind: str = "auto"):
        ref = load_reference() if kind in ("auto", "reference") else None
        if kind == "reference" and ref is None:
            raise RuntimeError("the NanoInfer reference is not importable (NANOINFER_REF / baseline/_ref)")
        self.kind = "reference" if ref is not None else "port"
        self.ref = ref
        self.shape = shape
        s = shape
        self.sizes = (s.num_heads * s.head_dim, s.num_kv_heads * s.head_dim, s.num_kv_heads * s.head_dim)
        if ref is None:
            import oracle.ops as O
            if s.rope == "table":
                self.port_rope = ("table", O.rope_cos_sin_cache(s.head_dim, s.max_position, s.theta))
            else:
                self.port_rope = ("mrope", O.mrope_inv_freq(s.head_dim, s.theta), tuple(s.sections), s.rope)
            return
        text = s.qk_norm == "text"
        norm_cls = ref["TextNorm"] if text else ref["RMSNorm"]
        self.norm_in, self.norm_post = norm_cls(s.hidden, s.eps), norm_cls(s.hidden, s.eps)
        self.norm_in.weight.data = inputs["w_in"].clone()
        self.norm_post.weight.data = inputs["w_post"].clone()
        self.q_norm = self.k_norm = None
        if s.qk_norm is not None:
            self.q_norm, self.k_norm = norm_cls(s.head_dim, s.eps), norm_cls(s.head_dim, s.eps)
            self.q_norm.weight.data = inputs["q_weight"].clone()
            self.k_norm.weight.data = inputs["k_weight"].clone()
        if s.rope == "table":
            self.rope = ref["get_rope"](s.head_dim, s.head_dim, s.max_position, s.theta)
        else:
            self.rope = ref["MRoPE"](head_dim=s.head_dim, base=s.theta, sections=tuple(s.sections),
                                     strategy=s.rope)
        self.act = ref["SiluAndMul"]()

    @torch.inference_mode()
    def __call__(self, d):
        if self.ref is None:
            return self._port(d)
        s = self.shape
        text = s.qk_norm == "text"
        if text:  # Qwen3-VL: a separate activation-dtype add, then the text norm
            h1 = d["hidden"] + d["residual"]
            self.norm_in(h1)
        else:
            _, h1 = self.norm_in(d["hidden"], d["residual"])
        q, k, v = d["qkv"].split(self.sizes, dim=-1)
        q = q.view(-1, s.num_heads, s.head_dim)
        k = k.view(-1, s.num_kv_heads, s.head_dim)
        v = v.view(-1, s.num_kv_heads, s.head_dim)
        if self.q_norm is not None:
            q, k = self.q_norm(q), self.k_norm(k)
        q, k = self.rope(d["positions"], q, k)
        self.ref["backend"].store(k, v, d["key_cache"], d["value_cache"], d["slot_mapping"])
        if text:
            self.norm_post(d["attn_out"] + h1)
        else:
            self.norm_post(d["attn_out"], h1)
        self.act(d["gate_up"])

    def _port(self, d):
        import oracle.ops as O

        s = self.shape
        text = s.qk_norm == "text"
        add_norm = O.add_text_rms_norm if text else O.add_rms_norm
        _, h1 = add_norm(d["hidden"], d["residual"], d["w_in"], s.eps)
        O.qk_norm_rope_store(d["qkv"], s.num_heads, s.num_kv_heads, s.head_dim, positions=d["positions"],
                             rope=self.port_rope, q_weight=d["q_weight"], k_weight=d["k_weight"], eps=s.eps,
                             norm=s.qk_norm, key_cache=d["key_cache"], value_cache=d["value_cache"],
                             slot_mapping=d["slot_mapping"], inplace=True)
        add_norm(d["attn_out"], h1, d["w_post"], s.eps)
        O.silu_and_mul(d["gate_up"])

    def gather(self, cache, block_table, sequence_length):
        """One sequence's paged-KV gather (the reference's PyTorch backend, or the port)."""
        if self.ref is None:
            import oracle.ops as O
            return O.paged_gather(cache, block_table, sequence_length)
        return self.ref["backend"].gather(cache, block_table, sequence_length)
