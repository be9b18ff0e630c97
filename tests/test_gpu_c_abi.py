"""Parity through the C ABI itself: ctypes, raw device pointers, no torch op.

This is the kind of binding a maintainer adds next to the reference's
extension loader (``nanovllm/layers/paged_kv/loader.py``): each entry point of
``include/nib_b200.h`` is called with plain pointers, element counts and
strides on the current stream, and its output is checked against the CPU
oracle. Bars: bit-exact for the byte/index work (paged store and gather,
embedding, DeepStack rows), for the 1-D RoPE prologue and for the norms
against the kernels' summation order; SiluAndMul within 1 ulp of the fp32
single-rounding result.
"""

import ctypes

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import _lib, workloads as W
from tests._util import assert_bitexact, assert_ulp

pytestmark = pytest.mark.gpu

NIB_BF16 = 2
NIB_ROPE_TABLE = 1
i32, i64, vp, f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float


class QKPrologueArgs(ctypes.Structure):
    """``nib_qk_prologue_args`` field for field."""

    _fields_ = [("struct_size", i32), ("dtype", i32), ("tokens", i64),
                ("num_heads", i32), ("num_kv_heads", i32), ("head_dim", i32),
                ("q", vp), ("q_token_stride", i64), ("q_head_stride", i64),
                ("k", vp), ("k_token_stride", i64), ("k_head_stride", i64),
                ("v", vp), ("v_token_stride", i64), ("v_head_stride", i64),
                ("q_out", vp), ("k_out", vp),
                ("norm", i32), ("weight_dtype", i32), ("q_weight", vp), ("k_weight", vp), ("eps", f32),
                ("rope_mode", i32), ("positions", vp), ("positions_axis_stride", i64),
                ("positions_token_stride", i64), ("cos_sin_table", vp), ("table_rows", i64),
                ("inv_freq", vp), ("sections", i32 * 3),
                ("key_cache", vp), ("value_cache", vp), ("slot_mapping", vp),
                ("num_slots", i64), ("cache_slot_stride", i64), ("status", vp), ("variant", i32)]


SIGNATURES = {
    "nib_rms_norm": [i32, vp, i64, i64, i64, i64, i64, i32, vp, f32, vp, vp],
    "nib_add_rms_norm": [i32, vp, i64, vp, i64, i64, i64, i32, vp, f32, i32, vp, vp, vp],
    "nib_silu_and_mul": [i32, vp, i64, i64, i64, vp, vp],
    "nib_qk_prologue": [ctypes.POINTER(QKPrologueArgs), vp],
    "nib_paged_store": [i32, vp, i64, vp, i64, i64, i64, vp, vp, i64, i64, vp, vp, vp],
    "nib_paged_gather": [i32, vp, i64, i64, i64, i64, i64, vp, i64, vp, vp, vp],
    "nib_embedding": [i32, vp, i64, vp, i64, i64, i64, i64, i64, i32, vp, vp, vp],
    "nib_deepstack_add": [i32, vp, i64, i64, i64, vp, i64, vp, i64, vp, vp],
}


@pytest.fixture(scope="module")
def lib():
    handle = _lib.cdll()
    handle.nib_last_error.restype = ctypes.c_char_p
    for name, argtypes in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    return handle


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ok(lib, rc):
    assert rc == 0, lib.nib_last_error().decode()
    torch.cuda.synchronize()


def test_norms(lib):
    d1 = W.make_layer_inputs(1, tokens=512, cache=False)
    x, res, w = d1["hidden"].cuda(), d1["residual"].cuda(), d1["w_in"].cuda()
    T, H = x.shape
    y = torch.empty_like(x)
    _ok(lib, lib.nib_rms_norm(NIB_BF16, x.data_ptr(), H, 0, T, 1, H, NIB_BF16, w.data_ptr(), 1e-6,
                              y.data_ptr(), _stream()))
    assert_bitexact(y, O.rms_norm(d1["hidden"], d1["w_in"], 1e-6, order="kernel"), "rms_norm")

    r_out = torch.empty_like(x)
    _ok(lib, lib.nib_add_rms_norm(NIB_BF16, x.data_ptr(), H, res.data_ptr(), H, T, H, NIB_BF16,
                                  w.data_ptr(), 1e-6, 0, y.data_ptr(), r_out.data_ptr(), _stream()))
    ey, er = O.add_rms_norm(d1["hidden"], d1["residual"], d1["w_in"], 1e-6, order="kernel")
    assert_bitexact(y, ey, "add_rms_norm")
    assert_bitexact(r_out, er, "add_rms_norm residual")

    # per-head norm of the q heads, read in place from the fused qkv rows
    qkv = d1["qkv"].cuda()
    qo = torch.empty(T, 16, 128, dtype=torch.bfloat16, device="cuda")
    _ok(lib, lib.nib_rms_norm(NIB_BF16, qkv.data_ptr(), qkv.stride(0), 128, T, 16, 128, NIB_BF16,
                              d1["q_weight"].cuda().data_ptr(), 1e-6, qo.data_ptr(), _stream()))
    eq = O.rms_norm(d1["qkv"][:, :2048].reshape(T, 16, 128), d1["q_weight"], 1e-6, order="kernel")
    assert_bitexact(qo, eq, "per-head q norm")

    # Qwen3-VL: the sum is rounded before the text norm
    d3 = W.make_layer_inputs(3, tokens=1024, cache=False)
    x3, r3, w3 = d3["hidden"].cuda(), d3["residual"].cuda(), d3["w_in"].cuda()
    y3, s3 = torch.empty_like(x3), torch.empty_like(x3)
    _ok(lib, lib.nib_add_rms_norm(NIB_BF16, x3.data_ptr(), 2048, r3.data_ptr(), 2048, 1024, 2048,
                                  NIB_BF16, w3.data_ptr(), 1e-6, 1, y3.data_ptr(), s3.data_ptr(), _stream()))
    ey3, es3 = O.add_text_rms_norm(d3["hidden"], d3["residual"], d3["w_in"], 1e-6, order="kernel")
    assert_bitexact(y3, ey3, "text add+norm")
    assert_bitexact(s3, es3, "text add+norm rounded sum")


def test_silu_and_mul(lib):
    d = W.make_layer_inputs(1, tokens=512, cache=False)
    x = d["gate_up"].cuda()
    y = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device="cuda")
    _ok(lib, lib.nib_silu_and_mul(NIB_BF16, x.data_ptr(), x.stride(0), x.shape[0], x.shape[1] // 2,
                                  y.data_ptr(), _stream()))
    assert_ulp(y, O.silu_and_mul_fp32(d["gate_up"]), 1, "silu_and_mul")


def test_qk_prologue_struct_c1(lib):
    """Qwen3 layer: per-head RMSNorm + 1-D RoPE table + paged store, C1 shapes."""
    d = W.make_layer_inputs(1, tokens=512)
    shp = d["shape"]
    T, nq, nkv, D = 512, shp.num_heads, shp.num_kv_heads, shp.head_dim
    table = O.rope_cos_sin_cache(D, shp.max_position, shp.theta)
    qkv, tab = d["qkv"].cuda(), table.cuda()
    pos, slots = d["positions"].cuda(), d["slot_mapping"].cuda()
    qw, kw = d["q_weight"].cuda(), d["k_weight"].cuda()
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
    q_out = torch.empty(T, nq, D, dtype=torch.bfloat16, device="cuda")
    k_out = torch.empty(T, nkv, D, dtype=torch.bfloat16, device="cuda")
    es = qkv.element_size()
    a = QKPrologueArgs(struct_size=ctypes.sizeof(QKPrologueArgs), dtype=NIB_BF16, tokens=T,
                       num_heads=nq, num_kv_heads=nkv, head_dim=D,
                       q=qkv.data_ptr(), q_token_stride=qkv.stride(0), q_head_stride=D,
                       k=qkv.data_ptr() + nq * D * es, k_token_stride=qkv.stride(0), k_head_stride=D,
                       v=qkv.data_ptr() + (nq + nkv) * D * es, v_token_stride=qkv.stride(0), v_head_stride=D,
                       q_out=q_out.data_ptr(), k_out=k_out.data_ptr(),
                       norm=1, weight_dtype=NIB_BF16, q_weight=qw.data_ptr(), k_weight=kw.data_ptr(), eps=1e-6,
                       rope_mode=NIB_ROPE_TABLE, positions=pos.data_ptr(), positions_axis_stride=0,
                       positions_token_stride=1, cos_sin_table=tab.data_ptr(), table_rows=tab.shape[0],
                       key_cache=kc.data_ptr(), value_cache=vc.data_ptr(), slot_mapping=slots.data_ptr(),
                       num_slots=kc.shape[0] * kc.shape[1], cache_slot_stride=nkv * D, variant=0)
    _ok(lib, lib.nib_qk_prologue(ctypes.byref(a), _stream()))
    eq, ek, ekc, evc = O.qk_norm_rope_store(
        d["qkv"], nq, nkv, D, positions=d["positions"], rope=("table", table), q_weight=d["q_weight"],
        k_weight=d["k_weight"], eps=1e-6, norm="rms", key_cache=d["key_cache"],
        value_cache=d["value_cache"], slot_mapping=d["slot_mapping"], order="kernel")
    assert_bitexact(q_out, eq, "q")
    assert_bitexact(k_out, ek, "k")
    assert_bitexact(kc, ekc, "key cache")
    assert_bitexact(vc, evc, "value cache")


def test_paged_store_and_gather(lib):
    """Strided k/v (views of qkv rows), 10% of slots -1, caches prefilled with -3;
    then a gather through a non-sequential block table."""
    g = torch.Generator().manual_seed(77)
    T, nkv, D, blocks, bs = 300, 8, 128, 64, 256
    qkv = torch.randn(T, (16 + 2 * nkv) * D, generator=g).to(torch.bfloat16)
    k = qkv[:, 16 * D:(16 + nkv) * D].reshape(T, nkv, D)
    v = qkv[:, (16 + nkv) * D:].reshape(T, nkv, D)
    slots = torch.randperm(blocks * bs, generator=g)[:T].to(torch.int32)
    slots[torch.randperm(T, generator=g)[:30]] = -1
    kc = torch.full((blocks, bs, nkv, D), -3.0, dtype=torch.bfloat16)
    vc = kc.clone()
    gq, gs = qkv.cuda(), slots.cuda()
    gkc, gvc = kc.cuda(), vc.cuda()
    es = gq.element_size()
    _ok(lib, lib.nib_paged_store(NIB_BF16, gq.data_ptr() + 16 * D * es, gq.stride(0),
                                 gq.data_ptr() + (16 + nkv) * D * es, gq.stride(0), T, nkv * D,
                                 gkc.data_ptr(), gvc.data_ptr(), nkv * D, blocks * bs, gs.data_ptr(),
                                 None, _stream()))
    ekc, evc = O.paged_store(k, v, kc, vc, slots)
    assert_bitexact(gkc, ekc, "key cache")
    assert_bitexact(gvc, evc, "value cache")

    table = torch.randperm(blocks, generator=g)[:16].to(torch.int32)
    n = 16 * bs - 97
    out = torch.empty(n, nkv, D, dtype=torch.bfloat16, device="cuda")
    gt = table.cuda()
    _ok(lib, lib.nib_paged_gather(NIB_BF16, gkc.data_ptr(), bs * nkv * D, nkv * D, blocks, bs, nkv * D,
                                  gt.data_ptr(), n, out.data_ptr(), None, _stream()))
    assert_bitexact(out, O.paged_gather(ekc, table, n), "gather")


def test_embedding_and_deepstack_rows(lib):
    g = torch.Generator().manual_seed(78)
    vocab, H = 5000, 1024
    weight = (torch.randn(vocab, H, generator=g) * 0.02).to(torch.bfloat16)
    ids = torch.randint(0, vocab, (777,), generator=g)
    gw, gi = weight.cuda(), ids.cuda()
    out = torch.empty(777, H, dtype=torch.bfloat16, device="cuda")
    _ok(lib, lib.nib_embedding(NIB_BF16, gi.data_ptr(), 777, gw.data_ptr(), H, vocab, 0, vocab, H, 0,
                               out.data_ptr(), None, _stream()))
    assert_bitexact(out, O.embedding(ids, weight), "embedding")

    T, H2 = 1024, 2048
    hidden = torch.randn(T, H2, generator=g).to(torch.bfloat16)
    rows = torch.sort(torch.randperm(T, generator=g)[:300]).values
    vis = torch.randn(300, H2, generator=g).to(torch.bfloat16)
    gh, gr, gv = hidden.cuda(), rows.cuda(), vis.cuda()
    _ok(lib, lib.nib_deepstack_add(NIB_BF16, gh.data_ptr(), H2, T, H2, gr.data_ptr(), 300, gv.data_ptr(),
                                   H2, None, _stream()))
    assert_bitexact(gh, O.add_deepstack_rows(hidden, rows, vis), "deepstack rows")
