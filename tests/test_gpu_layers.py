"""Drop-in layer modules on the GPU: reference-shaped calls, CUDA-graph capture,
and the no-fallback contract."""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.activation import SiluAndMul
from nano_vllm_multimodal_b200.layers.attention import attention_prologue
from nano_vllm_multimodal_b200.layers.layernorm import RMSNorm
from nano_vllm_multimodal_b200.layers.qwen3_vl import Qwen3VLTextRMSNorm
from nano_vllm_multimodal_b200.layers.rotary_embedding import get_rope
from tests._util import assert_bitexact, assert_matches_reference, assert_ulp

pytestmark = pytest.mark.gpu


def test_rmsnorm_module_both_forms():
    d = W.make_layer_inputs(1, cache=False)
    m = RMSNorm(1024).to(torch.bfloat16).cuda()
    with torch.no_grad():
        m.weight.copy_(d["w_in"])
    y = m(d["hidden"].cuda())
    assert_matches_reference(y, O.rms_norm(d["hidden"], d["w_in"], 1e-6, order="kernel"),
                             O.rms_norm(d["hidden"], d["w_in"], 1e-6), "RMSNorm")
    y, r = m(d["hidden"].cuda(), d["residual"].cuda())
    ey, er = O.add_rms_norm(d["hidden"], d["residual"], d["w_in"], 1e-6)
    assert_matches_reference(y, O.add_rms_norm(d["hidden"], d["residual"], d["w_in"], 1e-6, order="kernel")[0],
                             ey, "RMSNorm add")
    assert_bitexact(r, er)


def test_text_norm_module_and_dtype_guard():
    d = W.make_layer_inputs(3, tokens=256, cache=False)
    m = Qwen3VLTextRMSNorm(2048).to(torch.bfloat16).cuda()
    with torch.no_grad():
        m.weight.copy_(d["w_in"])
    assert_matches_reference(m(d["hidden"].cuda()), O.text_rms_norm(d["hidden"], d["w_in"], 1e-6, order="kernel"),
                             O.text_rms_norm(d["hidden"], d["w_in"], 1e-6), "text norm")
    y, s = m(d["hidden"].cuda(), d["residual"].cuda())
    ey, es = O.add_text_rms_norm(d["hidden"], d["residual"], d["w_in"], 1e-6)
    assert_matches_reference(y, O.add_text_rms_norm(d["hidden"], d["residual"], d["w_in"], 1e-6,
                                                    order="kernel")[0], ey, "text norm add")
    assert_bitexact(s, es)
    with pytest.raises(TypeError, match="weight dtype"):
        Qwen3VLTextRMSNorm(2048).cuda()(d["hidden"].cuda())


def test_silu_module():
    d = W.make_layer_inputs(4, tokens=128, cache=False)
    assert_ulp(SiluAndMul()(d["gate_up"].cuda()), O.silu_and_mul_fp32(d["gate_up"]), 1)


def test_get_rope_is_cached_and_matches_oracle():
    a = get_rope(128, 128, 40960, 1e6)
    assert get_rope(128, 128, 40960, 1e6) is a
    table = O.rope_cos_sin_cache(128, 40960, 1e6)
    assert torch.equal(a.cos_sin_cache.cpu(), table)


def test_cpu_tensors_raise_no_fallback():
    x = torch.randn(4, 1024, dtype=torch.bfloat16)
    with pytest.raises((NotImplementedError, RuntimeError)):
        ops.rms_norm(x, torch.ones(1024, dtype=torch.bfloat16), 1e-6)
    with pytest.raises((NotImplementedError, RuntimeError)):
        ops.silu_and_mul(torch.randn(4, 64, dtype=torch.bfloat16))
    # a host tensor mixed into a CUDA call is rejected before any launch
    with pytest.raises(RuntimeError, match="must be on"):
        ops.rms_norm(x.cuda(), torch.ones(1024, dtype=torch.bfloat16), 1e-6)


def test_layer_sequence_captures_in_cuda_graph():
    """add+norm -> fused prologue -> add+norm -> SiluAndMul, captured once and
    replayed on new inputs: identical to eager launches."""
    d = W.make_layer_inputs(3, tokens=512)
    shp = d["shape"]
    inv = O.mrope_inv_freq(128, shp.theta).cuda()
    static = {k: d[k].cuda() for k in ("hidden", "residual", "qkv", "attn_out", "gate_up", "positions",
                                       "slot_mapping", "w_in", "w_post", "q_weight", "k_weight")}
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()

    def layer():
        y1, h1 = ops.add_rms_norm(static["hidden"], static["residual"], static["w_in"], 1e-6, True)
        q, k, v = static["qkv"].split([2048, 1024, 1024], -1)
        q, k, v = q.view(-1, 16, 128), k.view(-1, 8, 128), v.view(-1, 8, 128)
        qr, kr = ops.qk_prologue(q, k, v=v, positions=static["positions"], q_weight=static["q_weight"],
                                 k_weight=static["k_weight"], eps=1e-6, rope_mode=ops.ROPE_MROPE_INTERLEAVED,
                                 inv_freq=inv, sections=shp.sections, key_cache=kc, value_cache=vc,
                                 slot_mapping=static["slot_mapping"])
        y2, h2 = ops.add_rms_norm(static["attn_out"], h1, static["w_post"], 1e-6, True)
        act = ops.silu_and_mul(static["gate_up"])
        return y1, qr, kr, y2, h2, act

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            layer()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = layer()
    d2 = W.make_layer_inputs(3, tokens=512)
    for k in ("hidden", "residual", "qkv", "gate_up"):
        static[k].copy_(d2[k].cuda() if k != "hidden" else d2[k].flip(0).cuda())
    graph.replay()
    torch.cuda.synchronize()
    replayed = [o.clone() for o in outs]
    eager = layer()
    for a, b in zip(replayed, eager):
        assert_bitexact(a, b, "graph replay vs eager")
    del graph


def test_attention_prologue_handles_empty_cache_like_reference():
    """Attention.forward stores only when both caches are non-empty (attention.py:87)."""
    d = W.make_layer_inputs(1, tokens=32, cache=False)
    rope = get_rope(128, 128, 40960, 1e6).cuda()
    q, k, v = attention_prologue(d["qkv"].cuda(), num_heads=16, num_kv_heads=8, head_dim=128,
                                 positions=d["positions"].cuda(), rotary_emb=rope,
                                 k_cache=torch.tensor([], device="cuda"), v_cache=torch.tensor([], device="cuda"),
                                 slot_mapping=d["slot_mapping"].cuda())
    eq, ek = O.apply_rope(d["positions"], d["qkv"][:, :2048].reshape(-1, 16, 128),
                          d["qkv"][:, 2048:3072].reshape(-1, 8, 128), O.rope_cos_sin_cache(128, 40960, 1e6))
    assert_bitexact(q, eq)
    assert_bitexact(k, ek)
