"""1-D RoPE and M-RoPE kernels vs the CPU oracle and the reference's golden outputs.

Tolerances:
* 1-D RoPE reads the same fp32 table as the reference and does the same
  uncontracted fp32 products and sums: bit-exact.
* M-RoPE rounds cos/sin of ``fp32(pos) * inv_freq`` to the activation dtype.
  The kernel calls CUDA's ``sincosf``; the CPU oracle uses the host libm. The
  two may differ in the last fp32 bit, which flips the bf16 rounding of a
  cos/sin value once in ~10^4-10^5. Hence: (1) given the kernel's own cos/sin,
  the rotation is bit-exact against the oracle; (2) the kernel's cos/sin equal
  torch's CUDA ``cos``/``sin`` bit-for-bit and are within 1 ulp of the CPU
  oracle's; (3) end to end, every element is within 1 ulp of the oracle except
  at tokens whose cos/sin differ from the CPU's.
"""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import (
    MultimodalRotaryEmbedding, apply_multimodal_rotary_emb)
from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding, apply_rotary_emb
from tests._util import assert_bitexact, assert_trig_bounded, assert_ulp

pytestmark = pytest.mark.gpu


def test_golden_rope_table(golden):
    c = golden["rope_c1"]
    rope = RotaryEmbedding(128, 128, 40960, 1e6).cuda()
    q, k = rope(c["inputs"]["positions"].cuda(), c["inputs"]["q"].cuda(), c["inputs"]["k"].cuda())
    assert_bitexact(q, c["outputs"]["q"], "rope q")
    assert_bitexact(k, c["outputs"]["k"], "rope k")


@pytest.mark.parametrize("config", [1, 2])
def test_rope_table_configs_strided(config):
    d = W.make_layer_inputs(config, cache=False)
    table = O.rope_cos_sin_cache(128, 40960, 1e6)
    qkv = d["qkv"]
    q, k = qkv[:, :2048].view(-1, 16, 128), qkv[:, 2048:3072].view(-1, 8, 128)
    gq, gk = qkv.cuda()[:, :2048].view(-1, 16, 128), qkv.cuda()[:, 2048:3072].view(-1, 8, 128)
    aq, ak = ops.rope(d["positions"].cuda(), gq, gk, table.cuda())
    eq, ek = O.apply_rope(d["positions"], q, k, table)
    assert_bitexact(aq, eq, "q")
    assert_bitexact(ak, ek, "k")


def test_apply_rotary_emb_generic_matches_table_path():
    d = W.make_layer_inputs(1, tokens=64, cache=False)
    table = O.rope_cos_sin_cache(128, 1024, 1e6)
    q = d["qkv"][:, :2048].reshape(-1, 16, 128)
    cs = table[d["positions"]]
    cos, sin = cs.chunk(2, dim=-1)
    out = apply_rotary_emb(q.cuda(), cos.cuda(), sin.cuda())
    eq, _ = O.apply_rope(d["positions"], q, q[:, :1], table)
    assert_bitexact(out, eq, "generic 1-D rotation")


def _check_mrope(positions, q, k, base, sections, strategy, what):
    inv = O.mrope_inv_freq(128, base)
    gpos, gq, gk, ginv = positions.cuda(), q.cuda(), k.cuda(), inv.cuda()
    aq, ak = ops.mrope(gpos, gq, gk, ginv, sections, strategy)
    # (2) cos/sin: kernel vs torch CUDA (bit-exact) and vs CPU (<= 1 ulp)
    gc, gs = ops.mrope_cos_sin(gpos, ginv, q.dtype)
    f = gpos.float().unsqueeze(-1) * ginv.view(1, 1, -1)
    emb = torch.cat((f, f), -1)
    assert_bitexact(gc, emb.cos().to(q.dtype), f"{what}: cos vs torch CUDA")
    assert_bitexact(gs, emb.sin().to(q.dtype), f"{what}: sin vs torch CUDA")
    cc, cs = O.mrope_cos_sin(positions, inv, q.dtype)
    dc = assert_ulp(gc, cc, 1, f"{what}: cos vs CPU")
    ds = assert_ulp(gs, cs, 1, f"{what}: sin vs CPU")
    frac = float(((dc > 0) | (ds > 0)).float().mean())
    assert frac < 1e-3, f"{what}: {frac:.2e} of cos/sin values differ from the CPU"
    # (1) rotation given the kernel's own cos/sin: bit-exact
    eq, ek = O.apply_mrope(q, k, gc.cpu(), gs.cpu(), sections, strategy)
    assert_bitexact(aq, eq, f"{what}: q given kernel cos/sin")
    assert_bitexact(ak, ek, f"{what}: k given kernel cos/sin")
    # (3) end to end vs the CPU oracle: <= 1 ulp where cos/sin agree; where one
    # differs, within the propagated bound of that 1-ulp difference
    oq, ok = O.mrope_forward(positions, q, k, inv, sections, strategy)
    trig_differs = ((dc > 0) | (ds > 0)).any(dim=0).any(dim=-1)  # [T]
    for name, a, o, x in (("q", aq, oq, q), ("k", ak, ok, k)):
        assert_trig_bounded(a, o, x, trig_differs, f"{what} {name}")


def test_golden_mrope_interleaved(golden):
    c = golden["mrope_interleaved_c3"]
    q, k = ops.mrope(c["inputs"]["positions"].cuda(), c["inputs"]["q"].cuda(), c["inputs"]["k"].cuda(),
                     c["outputs"]["inv_freq"].cuda(), (24, 20, 20), "interleaved")
    assert_ulp(q, c["outputs"]["q"], 1, "golden interleaved q")
    assert_ulp(k, c["outputs"]["k"], 1, "golden interleaved k")


def test_golden_mrope_chunked(golden):
    c = golden["mrope_chunked_c4"]
    q, k = ops.mrope(c["inputs"]["positions"].cuda(), c["inputs"]["q"].cuda(), c["inputs"]["k"].cuda(),
                     c["outputs"]["inv_freq"].cuda(), (16, 24, 24), "chunked")
    assert_ulp(q, c["outputs"]["q"], 1, "golden chunked q")
    assert_ulp(k, c["outputs"]["k"], 1, "golden chunked k")


def test_mrope_interleaved_c3_full():
    d = W.make_layer_inputs(3, tokens=4096, cache=False)
    qkv = d["qkv"]
    q = qkv[:, :2048].reshape(-1, 16, 128)
    k = qkv[:, 2048:3072].reshape(-1, 8, 128)
    _check_mrope(d["positions"], q, k, 5e6, (24, 20, 20), "interleaved", "C3")


def test_mrope_chunked_c4_full():
    d = W.make_layer_inputs(4, cache=False)
    qkv = d["qkv"]
    q = qkv[:, :2048].reshape(-1, 16, 128)
    k = qkv[:, 2048:2304].reshape(-1, 2, 128)
    _check_mrope(d["positions"], q, k, 1e6, (16, 24, 24), "chunked", "C4")


def test_mrope_large_positions_c5():
    d = W.make_layer_inputs(5, tokens=2048, cache=False)
    qkv = d["qkv"]
    q = qkv[:, :2048].reshape(-1, 16, 128)
    k = qkv[:, 2048:3072].reshape(-1, 8, 128)
    _check_mrope(d["positions"], q, k, 5e6, (24, 20, 20), "interleaved", "C5 positions")


def test_interleaved_fixed_golden_output_generic_kernel():
    """The reference's fixed KAT (``tests/test_qwen3_vl_runtime.py:178-217``), D = 8, fp32."""
    q = torch.tensor([[[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]]])
    k = torch.tensor([[[8.0, 7.0, 6.0, 5.0, 4.0, 3.0, 2.0, 1.0]]])
    cos = torch.tensor([[[1.0, 101.0, 102.0, 4.0, 1.0, 101.0, 102.0, 4.0]],
                        [[201.0, 2.0, 203.0, 204.0, 201.0, 2.0, 203.0, 204.0]],
                        [[301.0, 302.0, 3.0, 304.0, 301.0, 302.0, 3.0, 304.0]]])
    sin = torch.tensor([[[10.0, 1001.0, 1002.0, 40.0, 10.0, 1001.0, 1002.0, 40.0]],
                        [[2001.0, 20.0, 2003.0, 2004.0, 2001.0, 20.0, 2003.0, 2004.0]],
                        [[3001.0, 3002.0, 30.0, 3004.0, 3001.0, 3002.0, 30.0, 3004.0]]])
    before = [t.clone() for t in (q, k, cos, sin)]
    aq, ak = apply_multimodal_rotary_emb(q.cuda(), k.cuda(), cos.cuda(), sin.cuda(), (2, 1, 1),
                                         strategy="interleaved")
    torch.testing.assert_close(aq.cpu(), torch.tensor([[[-49.0, -116.0, -201.0, -304.0, 15.0, 52.0, 111.0, 192.0]]]))
    torch.testing.assert_close(ak.cpu(), torch.tensor([[[-32.0, -46.0, -42.0, -20.0, 84.0, 146.0, 186.0, 204.0]]]))
    for a, b in zip((q, k, cos, sin), before):
        assert torch.equal(a, b)


@pytest.mark.parametrize("strategy", ["chunked", "interleaved"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_generic_apply_matches_oracle(strategy, dtype):
    """``apply_multimodal_rotary_emb`` on random cos/sin, incl. a non-fused head dim (80)."""
    g = torch.Generator().manual_seed(29)
    for D, sections in ((128, (24, 20, 20)), (80, (16, 12, 12))):
        q = torch.randn(5, 2, D, generator=g).to(dtype)
        k = torch.randn(5, 1, D, generator=g).to(dtype)
        cos = torch.randn(3, 5, D, generator=g).to(dtype)
        sin = torch.randn(3, 5, D, generator=g).to(dtype)
        aq, ak = apply_multimodal_rotary_emb(q.cuda(), k.cuda(), cos.cuda(), sin.cuda(), sections, strategy)
        eq, ek = O.apply_mrope(q, k, cos, sin, sections, strategy)
        assert_bitexact(aq, eq, f"q {D} {dtype}")
        assert_bitexact(ak, ek, f"k {D} {dtype}")


@pytest.mark.parametrize("strategy", ["chunked", "interleaved"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_vector_apply_head_counts_strides_alignment(strategy, dtype):
    """The vectorised apply kernel over head counts that leave partial head groups
    and several load chunks (1..40 heads), head dims 64/128/256, a strided view of
    a wider row, and cos/sin whose base is not 16-byte aligned (the kernel must
    then take the per-element path): bit-exact against the oracle every time."""
    g = torch.Generator().manual_seed(31)
    T = 37
    for D, sections in ((64, (12, 10, 10)), (128, (24, 20, 20)), (256, (48, 40, 40))):
        for heads in (1, 3, 16, 20, 40):
            wide = torch.randn(T, heads + 3, D, generator=g).to(dtype)
            x = wide[:, 2:2 + heads]
            cos = torch.randn(3, T, D, generator=g).to(dtype)
            sin = torch.randn(3, T, D, generator=g).to(dtype)
            ex, _ = O.apply_mrope(x.contiguous(), x[:, :1].contiguous(), cos, sin, sections, strategy)
            got = ops.mrope_apply(x.cuda(), cos.cuda(), sin.cuda(), sections, strategy == "interleaved")
            assert_bitexact(got, ex, f"D={D} heads={heads} {dtype}")
            if heads == 3:
                n = cos.numel()
                cbuf = torch.empty(2 * n + 1, dtype=dtype, device="cuda")
                cm = cbuf[1:1 + n].view(3, T, D)
                sm = cbuf[1 + n:].view(3, T, D)
                cm.copy_(cos.cuda())
                sm.copy_(sin.cuda())
                got = ops.mrope_apply(x.cuda(), cm, sm, sections, strategy == "interleaved")
                assert_bitexact(got, ex, f"misaligned cos/sin D={D} {dtype}")


@pytest.mark.parametrize("D", [64, 128, 256, 12, 6, 2])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_mrope_cos_sin_head_dims_and_dtypes(D, dtype):
    """Paired-frequency kernel (even D/2; compile-time pairs for 64/128/256) and the
    per-element kernel (odd D/2) against torch's CUDA cos/sin, bit-exact; positions
    read through a token stride of 2 and a token count that leaves partial CTAs."""
    g = torch.Generator().manual_seed(D)
    T = 1001  # not a multiple of the 4 tokens per thread
    pos = torch.randint(0, 40000, (3, 2 * T), generator=g).cuda()[:, ::2]
    inv = (1.0 / (5e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))).cuda()
    c, s = ops.mrope_cos_sin(pos, inv, dtype)
    f = pos.float().unsqueeze(-1) * inv.view(1, 1, -1)
    emb = torch.cat((f, f), -1)
    assert_bitexact(c, emb.cos().to(dtype), f"cos D={D} {dtype}")
    assert_bitexact(s, emb.sin().to(dtype), f"sin D={D} {dtype}")


def test_module_forward_and_cos_sin():
    d = W.make_layer_inputs(3, tokens=512, cache=False)
    mod = MultimodalRotaryEmbedding(head_dim=128, base=5e6, sections=(24, 20, 20),
                                    strategy="interleaved").cuda()
    q = d["qkv"][:, :2048].reshape(-1, 16, 128)
    k = d["qkv"][:, 2048:3072].reshape(-1, 8, 128)
    aq, ak = mod(d["positions"].cuda(), q.cuda(), k.cuda())
    c, s = mod.cos_sin(d["positions"].cuda(), torch.bfloat16)
    eq, ek = O.apply_mrope(q, k, c.cpu(), s.cpu(), (24, 20, 20), "interleaved")
    assert_bitexact(aq, eq, "module q")
    assert_bitexact(ak, ek, "module k")
    # the module's own validation messages (multimodal_rotary_embedding.py:20-31,95-96)
    with pytest.raises(ValueError, match=r"positions must have shape \[3, num_tokens\]"):
        mod(d["positions"][:2].cuda(), q.cuda(), k.cuda())
    with pytest.raises(ValueError, match="rotary positions must match"):
        mod(d["positions"][:, :5].cuda(), q.cuda(), k.cuda())


@pytest.mark.parametrize("rope_kind,nq,nkv,dim,tokens,dtype", [
    ("table", 16, 8, 128, 4099, torch.bfloat16), ("interleaved", 16, 8, 128, 3000, torch.bfloat16),
    ("chunked", 16, 2, 128, 8312, torch.bfloat16), ("table", 14, 2, 64, 777, torch.bfloat16),
    ("interleaved", 8, 8, 256, 300, torch.bfloat16), ("chunked", 28, 4, 128, 1, torch.bfloat16),
    ("table", 16, 8, 128, 513, torch.float16), ("interleaved", 16, 8, 128, 700, torch.float16),
    ("chunked", 16, 2, 64, 257, torch.float16)])
def test_rotary_only_kernels_agree(rope_kind, nq, nkv, dim, tokens, dtype):
    """Rotary alone (the rotary modules' forward): the automatic choice (the
    warp-per-token rotary kernel) is bit-identical to the pipelined and the
    register-staged prologue kernels on strided q/k views of a qkv row, and to
    the oracle given the kernel's cos/sin."""
    g = torch.Generator().manual_seed(tokens + dim)
    qkv = torch.randn(tokens, (nq + 2 * nkv) * dim, generator=g).to(dtype)
    q = qkv[:, :nq * dim].view(tokens, nq, dim)
    k = qkv[:, nq * dim:(nq + nkv) * dim].view(tokens, nkv, dim)
    half = dim // 2
    if rope_kind == "table":
        table = O.rope_cos_sin_cache(dim, 40960, 1e6)
        pos = torch.randint(0, 40960, (tokens,), generator=g)
        kw = dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=table.cuda())
        eq, ek = O.apply_rope(pos, q, k, table)
    else:
        sections = (half - 2 * (half // 3), half // 3, half // 3) if rope_kind == "interleaved" else \
            (half // 4, half // 4, half - 2 * (half // 4))
        inv = O.mrope_inv_freq(dim, 5e6)
        pos = torch.randint(0, 32768, (3, tokens), generator=g)
        mode = ops.ROPE_MROPE_INTERLEAVED if rope_kind == "interleaved" else ops.ROPE_MROPE_CHUNKED
        kw = dict(rope_mode=mode, inv_freq=inv.cuda(), sections=sections)
        c, s = ops.mrope_cos_sin(pos.cuda(), inv.cuda(), dtype)
        eq, ek = O.apply_mrope(q, k, c.cpu(), s.cpu(), sections, rope_kind)
    # one device row: q and k are consecutive head ranges of it, with the row's token stride
    # even for a single token (view() picks its own stride for a size-1 dimension)
    gqkv = qkv.cuda()
    row = gqkv.stride(0)
    gq = gqkv.as_strided((tokens, nq, dim), (row, dim, 1), 0)
    gk = gqkv.as_strided((tokens, nkv, dim), (row, dim, 1), nq * dim)
    outs = [ops.qk_prologue(gq, gk, positions=pos.cuda(), variant=v, **kw) for v in (0, 1, 2)]
    for v, (aq, ak) in zip((1, 2), outs[1:]):
        assert_bitexact(outs[0][0], aq.cpu(), f"q auto vs variant {v}")
        assert_bitexact(outs[0][1], ak.cpu(), f"k auto vs variant {v}")
    assert_bitexact(outs[0][0], eq, "q vs oracle")
    assert_bitexact(outs[0][1], ek, "k vs oracle")
