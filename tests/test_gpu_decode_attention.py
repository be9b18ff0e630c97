"""Paged decode attention (``nib_decode_attention``) against the oracle and the reference,
both kernels: the tensor-core one (the default where it applies) and the CUDA-core one.

Tolerances (attention is floating point; both kernels accumulate in fp32):
* CUDA-core kernel against the float64 oracle: |out - oracle| <= 2^-7 * |oracle| + 1e-4,
  i.e. one bf16 ulp (the fp32 result rounded once; near a rounding midpoint its
  last-bit fp32 error can pick the other neighbour) plus a floor for outputs that
  nearly cancel;
* tensor-core kernel: the probabilities enter P.V as bf16/fp16 (as in flash-attn's
  decode kernel, the reference's), which adds at most 2^-8 x the softmax-weighted
  mean of |v| (``oracle.paged_decode_attention_abs``) to that bound; and its error
  against the oracle is no larger than flash-attn's own on the same inputs;
* against the reference's own SDPA decode output (golden fixture, CPU bf16):
  |out - reference| <= 2^-6 * max(1, |reference|), the bound the oracle meets.
"""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200.layers.attention import flash_attn_with_kvcache, paged_decode_attention

pytestmark = pytest.mark.gpu


def _close_to_oracle(out, expect, what, vabs=None):
    """``vabs`` (the softmax-weighted mean of |v|): the tensor-core kernel's bound."""
    o, e = out.detach().cpu().double(), expect.double()
    bound = 2.0 ** -7 * e.abs() + 1e-4
    if vabs is not None:
        bound = bound + 2.0 ** -8 * vabs
    bad = (o - e).abs() > bound
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} elements off, max {float((o - e).abs().max()):.3g}"


def _oracle(q, kc, vc, cl, tb, scale, variant=ops.DECODE_TENSOR_CORES):
    """Expected output and, for the tensor-core kernel, its P-rounding term."""
    expect = O.paged_decode_attention(q, kc, vc, cl, tb, scale)
    vabs = O.paged_decode_attention_abs(q, kc, vc, cl, tb, scale) if variant != ops.DECODE_CUDA_CORES else None
    return expect, vabs


def test_golden_reference_case(golden):
    c = golden["decode_attention_c2"]
    i = c["inputs"]
    args = (i["q"], i["k_cache"], i["v_cache"], i["context_lens"], i["block_tables"], c["meta"]["scale"])
    ref = c["outputs"]["out"].double()
    for variant in (ops.DECODE_AUTO, ops.DECODE_CUDA_CORES):
        out = ops.decode_attention(*(t.cuda() for t in args[:5]), args[5], variant=variant)
        assert bool(((out.cpu().double() - ref).abs() <= 2.0 ** -6 * ref.abs().clamp(min=1.0)).all())
        expect, vabs = _oracle(*args, variant=variant)
        _close_to_oracle(out, expect, f"golden, variant {variant}", vabs)


@pytest.mark.parametrize("nq,nkv", [(16, 8), (16, 2)])
def test_tensor_cores_as_accurate_as_flash_attn(nq, nkv):
    """Against the float64 oracle, the tensor-core kernel's error (largest and mean
    absolute) is no larger than that of flash-attn's flash_attn_with_kvcache, the
    reference's decode kernel, on the same inputs."""
    fa = pytest.importorskip("flash_attn").flash_attn_with_kvcache
    q, kc, vc, cl, tb = _case(nq + 7 * nkv, 8, nq, nkv, 128, 256, [1, 100, 256, 700, 2049, 4000, 3, 8000])
    scale = 128 ** -0.5
    g = [t.cuda() for t in (q, kc, vc, cl, tb)]
    mine = ops.decode_attention(*g, scale).cpu().double()
    theirs = fa(g[0].unsqueeze(1), g[1], g[2], cache_seqlens=g[3], block_table=g[4], softmax_scale=scale,
                causal=True)[:, 0].cpu().double()
    expect = O.paged_decode_attention(q, kc, vc, cl, tb, scale).double()
    e_mine, e_fa = (mine - expect).abs(), (theirs - expect).abs()
    assert float(e_mine.max()) <= float(e_fa.max()) * 1.05 + 1e-6, (float(e_mine.max()), float(e_fa.max()))
    assert float(e_mine.mean()) <= float(e_fa.mean()) * 1.05 + 1e-7, (float(e_mine.mean()), float(e_fa.mean()))


def _case(seed, batch, nq, nkv, dim, bs, lens, nblocks=None, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    need = [max(1, -(-n // bs)) for n in lens]
    nblocks = nblocks or sum(need) + 3
    kc = torch.randn(nblocks, bs, nkv, dim, generator=g).to(dtype)
    vc = torch.randn(nblocks, bs, nkv, dim, generator=g).to(dtype)
    width = max(need)
    perm = torch.randperm(nblocks, generator=g)
    tables = torch.full((batch, width), -1, dtype=torch.int32)
    at = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[at:at + n].to(torch.int32)
        at += n
    q = torch.randn(batch, nq, dim, generator=g).to(dtype)
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32), tables


@pytest.mark.parametrize("nq,nkv,dim,bs,lens", [
    (16, 8, 128, 256, [1, 255, 256, 257, 1000, 3]),       # Qwen3 GQA, 256-token blocks
    (16, 2, 128, 16, [7, 64, 300, 33]),                   # Qwen2.5-VL GQA 8, small blocks
    (14, 2, 64, 24, [50, 1, 97]),                         # 7 heads per kv head, non-power-of-2 blocks
    (8, 8, 256, 32, [0, 40, 129]),                        # MHA, head_dim 256, an empty context
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("variant", [ops.DECODE_CUDA_CORES, ops.DECODE_TENSOR_CORES])
def test_matches_oracle(nq, nkv, dim, bs, lens, dtype, variant):
    q, kc, vc, cl, tb = _case(nq * 1000 + dim + bs, len(lens), nq, nkv, dim, bs, lens, dtype=dtype)
    scale = dim ** -0.5
    args = (q.cuda(), kc.cuda(), vc.cuda(), cl.cuda(), tb.cuda(), scale)
    if variant == ops.DECODE_TENSOR_CORES and not _mma_shape(nq, nkv, dim, bs):
        with pytest.raises(RuntimeError, match="tensor-core kernel needs"):
            ops.decode_attention(*args, variant=variant)
        return
    out = ops.decode_attention(*args, variant=variant)
    expect, vabs = _oracle(q, kc, vc, cl, tb, scale, variant)
    _close_to_oracle(out, expect, f"{nq}/{nkv} D{dim} bs{bs} variant {variant}", vabs)
    if 0 in lens:
        assert not out[lens.index(0)].any()


def _mma_shape(nq, nkv, dim, bs):
    """The tensor-core kernel's shapes: head_dim 64/128, <= 16 q heads per kv head,
    block size a multiple of 16."""
    return dim in (64, 128) and nq // nkv <= 16 and bs % 16 == 0


@pytest.mark.parametrize("nq,nkv", [(16, 8), (16, 2), (12, 1), (16, 16)])
def test_tensor_cores_match_cuda_cores_and_ignore_stale_slots(nq, nkv):
    """The tensor-core kernel against the CUDA-core kernel and the oracle, with
    NaN in every cache slot past each context (a block's unwritten tail), a split
    context whose split boundaries fall inside 16-token tiles, and a context of
    one token. Stale slots must not reach the output (0 x NaN is NaN)."""
    lens = [1, 17, 255, 4000, 16]
    q, kc, vc, cl, tb = _case(nq * 31 + nkv, len(lens), nq, nkv, 128, 256, lens)
    for b, n in enumerate(lens):  # poison the unwritten tail of each sequence's last block
        last = int(tb[b, (n - 1) // 256])
        kc[last, n % 256 or 256:] = float("nan")
        vc[last, n % 256 or 256:] = float("nan")
    args = (q.cuda(), kc.cuda(), vc.cuda(), cl.cuda(), tb.cuda(), 128 ** -0.5)
    mma = ops.decode_attention(*args, variant=ops.DECODE_TENSOR_CORES)
    fma = ops.decode_attention(*args, variant=ops.DECODE_CUDA_CORES)
    assert not torch.isnan(mma).any() and not torch.isnan(fma).any()
    expect, vabs = _oracle(q, kc, vc, cl, tb, 128 ** -0.5)
    _close_to_oracle(mma, expect, f"tensor cores {nq}/{nkv}", vabs)
    _close_to_oracle(fma, expect, f"CUDA cores {nq}/{nkv}")
    assert torch.equal(ops.decode_attention(*args), mma), "the default is the tensor-core kernel"


def test_long_contexts_split_across_ctas_and_strided_q():
    """Few requests with long contexts take several CTAs per (request, kv head) and a
    combine pass; q is a strided view (a slice of a fused qkv row)."""
    q, kc, vc, cl, tb = _case(77, 2, 16, 8, 128, 256, [20000, 9000])
    qkv = torch.randn(2, (16 + 16) * 128).to(torch.bfloat16)
    qkv[:, :2048] = q.reshape(2, -1)
    qv = qkv.cuda()[:, :2048].view(2, 16, 128)
    assert qv.stride(0) == 32 * 128
    for variant in (ops.DECODE_CUDA_CORES, ops.DECODE_TENSOR_CORES):
        out = ops.decode_attention(qv, kc.cuda(), vc.cuda(), cl.cuda(), tb.cuda(), 128 ** -0.5, variant=variant)
        expect, vabs = _oracle(q, kc, vc, cl, tb, 128 ** -0.5, variant)
        _close_to_oracle(out, expect, f"split contexts, variant {variant}", vabs)


@pytest.mark.parametrize("nq,nkv,dim,bs", [(16, 2, 128, 64), (16, 8, 128, 256), (8, 1, 64, 32)])
def test_many_ragged_requests(nq, nkv, dim, bs):
    """160 requests of ragged lengths: many one-tile contexts, two empty ones, long
    ones split over CTAs, NaN in every stale slot past a context. The default
    (tensor-core) kernel and the CUDA-core kernel against the oracle; empty
    contexts give zeros; two calls give the same bits."""
    g = torch.Generator().manual_seed(nq * 100 + nkv * 10 + dim)
    lens = torch.randint(1, 1200, (160,), generator=g)
    lens[::7] = torch.randint(1, 17, (lens[::7].numel(),), generator=g)
    lens[[5, 99]] = 0
    lens[[50, 51]] = torch.tensor([9000, 4097])
    lens = lens.tolist()
    q, kc, vc, cl, tb = _case(nq + nkv + dim, len(lens), nq, nkv, dim, bs, lens)
    for b, n in enumerate(lens):
        last = int(tb[b, max(n - 1, 0) // bs])
        kc[last, n % bs or (bs if n else 0):] = float("nan")
        vc[last, n % bs or (bs if n else 0):] = float("nan")
    scale = dim ** -0.5
    args = (q.cuda(), kc.cuda(), vc.cuda(), cl.cuda(), tb.cuda(), scale)
    out = ops.decode_attention(*args)
    assert not torch.isnan(out).any()
    expect, vabs = _oracle(q, kc, vc, cl, tb, scale)
    _close_to_oracle(out, expect, f"ragged {nq}/{nkv} D{dim}", vabs)
    for b in (5, 99):
        assert not out[b].any(), "an empty context gives zeros"
    fma = ops.decode_attention(*args, variant=ops.DECODE_CUDA_CORES)
    _close_to_oracle(fma, expect, f"CUDA cores, ragged {nq}/{nkv} D{dim}")
    assert torch.equal(ops.decode_attention(*args), out), "deterministic"


def test_flash_attn_shaped_drop_in():
    q, kc, vc, cl, tb = _case(5, 4, 16, 8, 128, 256, [3, 700, 256, 1])
    qg, kg, vg, cg, tg = q.cuda(), kc.cuda(), vc.cuda(), cl.cuda(), tb.cuda()
    o = flash_attn_with_kvcache(qg.unsqueeze(1), kg, vg, cache_seqlens=cg, block_table=tg,
                                softmax_scale=128 ** -0.5, causal=True)
    assert o.shape == (4, 1, 16, 128)
    assert torch.equal(o[:, 0], paged_decode_attention(qg, kg, vg, cg, tg, 128 ** -0.5))
    with pytest.raises(NotImplementedError, match="one query token"):
        flash_attn_with_kvcache(torch.cat((qg.unsqueeze(1), qg.unsqueeze(1)), 1), kg, vg,
                                cache_seqlens=cg, block_table=tg)
    with pytest.raises(NotImplementedError, match="unsupported arguments"):
        flash_attn_with_kvcache(qg.unsqueeze(1), kg, vg, cache_seqlens=cg, block_table=tg, softcap=30.0)


@pytest.mark.parametrize("variant", [ops.DECODE_CUDA_CORES, ops.DECODE_TENSOR_CORES])
def test_bad_block_and_length_reported(monkeypatch, variant):
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    q, kc, vc, cl, tb = _case(9, 2, 16, 8, 128, 16, [20, 5])
    bad = tb.clone()
    bad[0, 1] = 999
    with pytest.raises(ValueError, match="block"):
        ops.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), cl.cuda(), bad.cuda(), 0.1, variant=variant)
    long = cl.clone()
    long[1] = 10_000
    with pytest.raises(ValueError, match="out of range"):
        ops.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), long.cuda(), tb.cuda(), 0.1, variant=variant)


@pytest.mark.parametrize("batch", [4, 128])
def test_drop_in_captures_in_a_cuda_graph(batch):
    """ModelRunner captures its decode steps in CUDA graphs, attention included. The
    drop-in reads no device value on the host, so it captures; replays with new
    queries, context lengths and block tables written in place equal eager calls.
    4 requests split their contexts over many CTAs, 128 over two (partials in the
    workspace, merged by a second launch inside the graph)."""
    nq, nkv, D, bs, width = 16, 8, 128, 256, 8
    g = torch.Generator().manual_seed(batch)
    nblocks = batch * width
    kc = torch.randn(nblocks, bs, nkv, D, generator=g).to(torch.bfloat16).cuda()
    vc = torch.randn(nblocks, bs, nkv, D, generator=g).to(torch.bfloat16).cuda()
    q = torch.empty(batch, 1, nq, D, dtype=torch.bfloat16, device="cuda")
    lens = torch.empty(batch, dtype=torch.int32, device="cuda")
    tables = torch.empty(batch, width, dtype=torch.int32, device="cuda")

    def fill(seed):
        gg = torch.Generator().manual_seed(seed)
        q.copy_(torch.randn(batch, 1, nq, D, generator=gg).to(torch.bfloat16))
        lens.copy_(torch.randint(1, width * bs + 1, (batch,), generator=gg).to(torch.int32))
        tables.copy_(torch.randperm(nblocks, generator=gg).view(batch, width).to(torch.int32))

    def call():
        return flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens, block_table=tables,
                                       softmax_scale=D ** -0.5, causal=True)

    fill(1)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = call()
    for seed in (2, 3):
        fill(seed)
        graph.replay()
        eager = call()
        torch.cuda.synchronize()
        assert torch.equal(out, eager), f"replay {seed}"
    del graph
