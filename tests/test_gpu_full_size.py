"""Parity at the full C5 size (262,144 tokens, a 16,384 x 256-slot K/V cache pair),
through properties that do not depend on size, checked on the device:

* the two prologue kernels (bulk-copy pipelined and register-staged) give
  bit-identical q, k and caches at full size;
* every written slot holds exactly the token's rotated k and raw v, and every
  other slot keeps its sentinel (-3);
* a random sample of tokens / rows matches the CPU oracle bit for bit (norms in
  the kernels' summation order, M-RoPE given the kernel's own cos/sin), and
  against the oracle's own cos/sin within 1 ulp except where a cos/sin value
  differs from the host's, there within that difference's propagated bound;
  SiluAndMul within 1 ulp of the fp32 single-rounding result;
* the many-sequence paged gather over the full cache equals direct indexing.

Inputs are generated on the device (seeded) and need about 45 GB of HBM.
"""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from tests._util import assert_bitexact, assert_trig_bounded, assert_ulp

pytestmark = pytest.mark.gpu

SHP = W.C5
T = SHP.tokens
NQ, NKV, D = SHP.num_heads, SHP.num_kv_heads, SHP.head_dim


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _normal(shape, seed, mean=0.0, std=1.0):
    t = torch.randn(shape, generator=_gen(seed), device="cuda", dtype=torch.float32)
    return (t * std + mean).to(torch.bfloat16)


@pytest.fixture(scope="module")
def c5():
    d = {
        "qkv": _normal((T, (NQ + 2 * NKV) * D), 50001),
        "positions": torch.randint(0, 32768, (3, T), generator=_gen(50002), device="cuda"),
        "slots": torch.randperm(SHP.num_blocks * SHP.block_size, generator=_gen(50003),
                                device="cuda")[:T].to(torch.int32),
        "q_weight": _normal((D,), 50004, 1.0, 0.1),
        "k_weight": _normal((D,), 50005, 1.0, 0.1),
        "inv_freq": O.mrope_inv_freq(D, SHP.theta).cuda(),
    }
    yield d
    d.clear()
    torch.cuda.empty_cache()


def _prologue(d, variant):
    qkv = d["qkv"]
    q, k, v = qkv.split([NQ * D, NKV * D, NKV * D], -1)
    q, k, v = q.view(-1, NQ, D), k.view(-1, NKV, D), v.view(-1, NKV, D)
    shape = (SHP.num_blocks, SHP.block_size, NKV, D)
    kc = torch.full(shape, -3.0, dtype=torch.bfloat16, device="cuda")
    vc = torch.full(shape, -3.0, dtype=torch.bfloat16, device="cuda")
    qr, kr = ops.qk_prologue(q, k, v=v, positions=d["positions"], q_weight=d["q_weight"],
                             k_weight=d["k_weight"], eps=SHP.eps, rope_mode=ops.ROPE_MROPE_INTERLEAVED,
                             inv_freq=d["inv_freq"], sections=SHP.sections, key_cache=kc, value_cache=vc,
                             slot_mapping=d["slots"], variant=variant)
    return qr, kr, kc, vc


def test_c5_full_prologue_variants_placement_and_sample(c5):
    q1, k1, kc1, vc1 = _prologue(c5, 2)
    q2, k2, kc2, vc2 = _prologue(c5, 1)
    assert torch.equal(q1, q2) and torch.equal(k1, k2), "pipelined vs register-staged q/k"
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2), "pipelined vs register-staged caches"
    del q2, k2, kc2, vc2
    torch.cuda.empty_cache()

    slots = c5["slots"].long()
    v = c5["qkv"][:, (NQ + NKV) * D:].view(T, NKV, D)
    fk, fv = kc1.view(-1, NKV, D), vc1.view(-1, NKV, D)
    assert torch.equal(fk[slots], k1), "key cache rows at the written slots"
    assert torch.equal(fv[slots], v), "value cache rows at the written slots"
    untouched = torch.ones(fk.shape[0], dtype=torch.bool, device="cuda")
    untouched[slots] = False
    n_untouched = int(untouched.sum())
    assert n_untouched == fk.shape[0] - T
    for start in range(0, fk.shape[0], 1 << 20):  # chunks keep the temporaries small
        sl = slice(start, start + (1 << 20))
        keep = untouched[sl]
        assert bool((fk[sl][keep] == -3).all()) and bool((fv[sl][keep] == -3).all()), "untouched slots"

    # 2,048 random tokens against the oracle composition
    idx = torch.randperm(T, generator=_gen(50006), device="cuda")[:2048]
    rows = c5["qkv"][idx].cpu()
    qs = O.text_rms_norm(rows[:, :NQ * D].reshape(-1, NQ, D), c5["q_weight"].cpu(), SHP.eps, order="kernel")
    ks = O.text_rms_norm(rows[:, NQ * D:(NQ + NKV) * D].reshape(-1, NKV, D), c5["k_weight"].cpu(), SHP.eps,
                         order="kernel")
    cos, sin = ops.mrope_cos_sin(c5["positions"][:, idx].contiguous(), c5["inv_freq"], torch.bfloat16)
    eq, ek = O.apply_mrope(qs, ks, cos.cpu(), sin.cpu(), SHP.sections, "interleaved")
    assert_bitexact(q1[idx], eq, "q sample")
    assert_bitexact(k1[idx], ek, "k sample")
    # the same sample end to end against the oracle's own cos/sin (host libm):
    # cos/sin within 1 ulp, rarely different, and the rotation within the
    # propagated bound of such a difference
    cc, cs = O.mrope_cos_sin(c5["positions"][:, idx].cpu(), c5["inv_freq"].cpu(), torch.bfloat16)
    dc = assert_ulp(cos, cc, 1, "C5 sample cos vs CPU")
    ds = assert_ulp(sin, cs, 1, "C5 sample sin vs CPU")
    assert float(((dc > 0) | (ds > 0)).float().mean()) < 1e-3, "C5 sample: too many cos/sin differ from the CPU"
    trig_differs = ((dc > 0) | (ds > 0)).any(dim=0).any(dim=-1)
    oq, ok = O.apply_mrope(qs, ks, cc, cs, SHP.sections, "interleaved")
    assert_trig_bounded(q1[idx], oq, qs, trig_differs, "C5 full-size prologue q, oracle cos/sin")
    assert_trig_bounded(k1[idx], ok, ks, trig_differs, "C5 full-size prologue k, oracle cos/sin")

    # the many-sequence gather over the full cache: 8 sequences x 16,384 tokens
    seqs, n = 8, SHP.extra["gather_len"]
    tables = W.make_gather_inputs(5, sequences=seqs, seq_len=n, num_blocks=SHP.num_blocks).cuda()
    lens = torch.full((seqs,), n, dtype=torch.int32, device="cuda")
    cu = torch.arange(seqs + 1, dtype=torch.int64, device="cuda") * n
    out = ops.paged_gather_varlen(kc1, tables, lens, cu, seqs * n, n)
    assert torch.equal(out, kc1[tables.long()].reshape(seqs * n, NKV, D)), "gather vs direct index"


def test_c5_full_norm_and_silu_samples():
    x = _normal((T, SHP.hidden), 50011)
    res = _normal((T, SHP.hidden), 50012)
    w = _normal((SHP.hidden,), 50013, 1.0, 0.1)
    y, s = ops.add_rms_norm(x, res, w, SHP.eps, True)
    idx = torch.randperm(T, generator=_gen(50014), device="cuda")[:1024]
    ey, es = O.add_text_rms_norm(x[idx].cpu(), res[idx].cpu(), w.cpu(), SHP.eps, order="kernel")
    assert_bitexact(y[idx], ey, "text add+norm sample")
    assert_bitexact(s[idx], es, "rounded residual sample")
    del x, res, y, s
    gu = _normal((T, 2 * SHP.intermediate), 50015)
    act = ops.silu_and_mul(gu)
    assert_ulp(act[idx], O.silu_and_mul_fp32(gu[idx].cpu()), 1, "silu sample")
    del gu, act
    torch.cuda.empty_cache()
