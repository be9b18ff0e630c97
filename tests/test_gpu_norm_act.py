"""RMSNorm / add+RMSNorm / Qwen3-VL text norm / SiluAndMul kernels vs the CPU oracle.

Norms (see ``tests/_util.assert_matches_reference``): bit-exact against the
reference formula with the kernels' fp32 summation order; against PyTorch's
own CPU evaluation within 2 ulp, beyond 1 ulp in at most 1e-5 of the elements
(fp32 outputs: 4 ulp), and every element beyond 1 ulp attributed to a row
whose fp32 statistic differs between the two summation orders. Residual outputs (the rounded sums) are bit-exact.
SiluAndMul: within 1 ulp of the fp32 single-rounding result (what the
reference's compiled GPU kernel computes) and within 2 ulp of the eager
two-rounding CPU result."""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from tests._util import assert_bitexact, assert_matches_reference, assert_ulp

pytestmark = pytest.mark.gpu


def test_golden_rmsnorm(golden):
    c = golden["rmsnorm_add_c1"]
    i = c["inputs"]
    y, r = ops.add_rms_norm(i["x"].cuda(), i["residual"].cuda(), i["weight"].cuda(), 1e-6)
    assert_ulp(y, c["outputs"]["y"], 1, "add_rms y")
    assert_bitexact(r, c["outputs"]["residual"], "add_rms residual")
    c = golden["rmsnorm_c1"]
    assert_ulp(ops.rms_norm(c["inputs"]["x"].cuda(), c["inputs"]["weight"].cuda(), 1e-6),
               c["outputs"]["y"], 1, "rms")


def test_golden_qk_norm_strided(golden):
    c = golden["qknorm_c1"]
    qkv = c["inputs"]["qkv"].cuda()
    q, k, _ = qkv.split([16 * 128, 8 * 128, 8 * 128], dim=-1)
    q, k = q.view(-1, 16, 128), k.view(-1, 8, 128)
    assert_ulp(ops.rms_norm(q, c["inputs"]["q_weight"].cuda(), 1e-6), c["outputs"]["q"], 1, "q norm")
    assert_ulp(ops.rms_norm(k, c["inputs"]["k_weight"].cuda(), 1e-6), c["outputs"]["k"], 1, "k norm")


def test_golden_text_norm(golden):
    c = golden["textnorm_c3"]
    i = c["inputs"]
    assert_ulp(ops.rms_norm(i["x"].cuda(), i["weight"].cuda(), 1e-6), c["outputs"]["y"], 1, "text")
    y, s = ops.add_rms_norm(i["x"].cuda(), i["residual"].cuda(), i["weight"].cuda(), 1e-6, round_sum=True)
    assert_ulp(y, c["outputs"]["y_add"], 1, "text add")
    assert_bitexact(s, c["outputs"]["sum"], "text add sum")


@pytest.mark.parametrize("config", [1, 3, 4])
def test_add_rms_norm_configs(config):
    d = W.make_layer_inputs(config, tokens=2048, cache=False)
    x, r, w = d["hidden"], d["residual"], d["w_in"]
    y, res = ops.add_rms_norm(x.cuda(), r.cuda(), w.cuda(), 1e-6)
    assert_matches_reference(y, O.add_rms_norm(x, r, w, 1e-6, order="kernel")[0],
                             O.add_rms_norm(x, r, w, 1e-6)[0], f"C{config} add+norm",
                             stats=(x.float() + r.float(), 1e-6, True))
    assert_bitexact(res, O.add_rms_norm(x, r, w, 1e-6)[1], "residual")
    y2, s2 = ops.add_rms_norm(x.cuda(), r.cuda(), w.cuda(), 1e-6, round_sum=True)
    ey2, es2 = O.add_text_rms_norm(x, r, w, 1e-6)
    assert_matches_reference(y2, O.add_text_rms_norm(x, r, w, 1e-6, order="kernel")[0], ey2,
                             f"C{config} rounded add+text norm", stats=(es2, 1e-6, True))
    assert_bitexact(s2, es2, "text sum")
    assert torch.equal(x, d["hidden"])  # inputs untouched


@pytest.mark.parametrize("hidden", [64, 128, 256, 896, 1024, 2048, 2560, 3584, 4096, 5120])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_rms_norm_hidden_sizes(hidden, dtype):
    g = torch.Generator().manual_seed(hidden)
    x = torch.randn(67, hidden, generator=g).to(dtype)
    r = torch.randn(67, hidden, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
    tag = f"hidden {hidden} {str(dtype).split('.')[-1]}"
    assert_matches_reference(ops.rms_norm(x.cuda(), w.cuda(), 1e-6), O.rms_norm(x, w, 1e-6, order="kernel"),
                             O.rms_norm(x, w, 1e-6), f"{tag} rms", stats=(x.float(), 1e-6, False))
    y, res = ops.add_rms_norm(x.cuda(), r.cuda(), w.cuda(), 1e-5)
    ey, er = O.add_rms_norm(x, r, w, 1e-5)
    assert_matches_reference(y, O.add_rms_norm(x, r, w, 1e-5, order="kernel")[0], ey, f"{tag} add+norm",
                             max_frac=1e-4, stats=(x.float() + r.float(), 1e-5, True))
    assert_bitexact(res, er, "add residual")


def test_rms_norm_fp32_weight_with_bf16_activations():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(33, 1024, generator=g).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(1024, generator=g)
    assert_matches_reference(ops.rms_norm(x.cuda(), w.cuda(), 1e-6), O.rms_norm(x, w, 1e-6, order="kernel"),
                             O.rms_norm(x, w, 1e-6), "fp32 weight", max_frac=1e-4,
                             stats=(x.float(), 1e-6, False))


def test_rms_norm_per_head_views_and_empty():
    d = W.make_layer_inputs(3, tokens=333, cache=False)
    qkv = d["qkv"].cuda()
    q = qkv[:, : 16 * 128].view(-1, 16, 128)
    k = qkv[:, 16 * 128: 24 * 128].view(-1, 8, 128)
    assert q.stride(0) == 32 * 128
    qc, kc = d["qkv"][:, : 16 * 128].reshape(-1, 16, 128), d["qkv"][:, 16 * 128: 24 * 128].reshape(-1, 8, 128)
    assert_matches_reference(ops.rms_norm(q, d["q_weight"].cuda(), 1e-6),
                             O.text_rms_norm(qc, d["q_weight"], 1e-6, order="kernel"),
                             O.text_rms_norm(qc, d["q_weight"], 1e-6), "C3 q heads", max_frac=1e-4,
                             stats=(qc.float(), 1e-6, False))
    assert_matches_reference(ops.rms_norm(k, d["k_weight"].cuda(), 1e-6),
                             O.rms_norm(kc, d["k_weight"], 1e-6, order="kernel"),
                             O.rms_norm(kc, d["k_weight"], 1e-6), "C3 k heads", max_frac=1e-4,
                             stats=(kc.float(), 1e-6, False))
    empty = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    assert ops.rms_norm(empty, torch.ones(1024, dtype=torch.bfloat16, device="cuda"), 1e-6).shape == (0, 1024)


def test_golden_silu(golden):
    c = golden["silu_c1"]
    y = ops.silu_and_mul(c["inputs"]["x"].cuda())
    assert_ulp(y, c["outputs"]["y"], 1, "silu vs eager reference")


@pytest.mark.parametrize("config", [1, 3, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_configs(config, dtype):
    d = W.make_layer_inputs(config, tokens=1024, cache=False)
    x = d["gate_up"].to(dtype)
    y = ops.silu_and_mul(x.cuda())
    assert_ulp(y, O.silu_and_mul_fp32(x), 1, "vs fp32 single rounding")
    d2 = assert_ulp(y, O.silu_and_mul(x), 2, "vs eager two roundings")
    assert int((d2 > 1).sum()) <= max(3, int(1e-5 * d2.numel()))


@pytest.mark.parametrize("rows,inter", [(1023, 512), (13, 136), (5, 16384), (7, 2056), (1, 8), (3, 1000)])
def test_silu_row_shapes(rows, inter):
    """CTA shapes: several rows per CTA with a ragged last CTA (short rows), up to 8
    vectors per thread (long rows), partial last vector group."""
    g = torch.Generator().manual_seed(rows * 7 + inter)
    x = torch.randn(rows, 2 * inter, generator=g).to(torch.bfloat16)
    y = ops.silu_and_mul(x.cuda())
    assert_ulp(y, O.silu_and_mul_fp32(x), 1, f"silu rows={rows} inter={inter}")


def test_silu_rejects_rows_longer_than_supported():
    x = torch.zeros(2, 2 * 16392, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="larger than this build supports"):
        ops.silu_and_mul(x)


def test_silu_extreme_values_and_fp32():
    vals = torch.tensor([-200.0, -100.0, -88.9, -88.5, -87.5, -80.5, -80.0, -20.0, -1e-3, 0.0, -0.0,
                         1e-30, 3.0, 80.0, 80.5, 100.0, 3e38, float("inf"), float("-inf"), -5.0,
                         -2.5, 0.5, 7.0, -1e-38])
    x = torch.cat((vals.view(1, -1), torch.full((1, vals.numel()), 1.5)), dim=1)
    # a row whose vectors all take the fast (approximate ex2/rcp) form: edges of its range,
    # tiny and subnormal gates
    edge = torch.tensor([-79.9, 79.9, -1e-30, 1e-38, -3e-39, 0.0, -0.0, 1e-3,
                         -40.0, 40.0, -1e-20, 2e-38, -7e-39, 0.25, -0.25, 60.0,
                         -79.5, 79.5, 5e-39, -5e-39, 1.0, -1.0, 12.0, -12.0])
    edge_row = torch.cat((edge.view(1, -1), torch.full((1, edge.numel()), -3.0)), dim=1)
    x = torch.cat((x, edge_row), dim=0)
    for dt in (torch.bfloat16, torch.float32):
        xx = x.to(dt)
        y = ops.silu_and_mul(xx.cuda())
        assert_ulp(y, O.silu_and_mul_fp32(xx), 1 if dt != torch.float32 else 2, f"extremes {dt}")


def test_silu_strided_rows():
    g = torch.Generator().manual_seed(9)
    big = torch.randn(50, 7000, generator=g).to(torch.bfloat16)
    x = big[:, 8:8 + 6144]
    y = ops.silu_and_mul(big.cuda()[:, 8:8 + 6144])
    assert_ulp(y, O.silu_and_mul_fp32(x.contiguous()), 1, "strided")
