"""Embedding row gather and DeepStack add vs the oracle (bit-exact)."""

from unittest.mock import patch

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.qwen3_vl import add_deepstack_rows, add_deepstack_rows_
from tests._util import assert_bitexact, ulp_diff

pytestmark = pytest.mark.gpu


def test_golden_embedding(golden):
    c = golden["embedding_c2"]
    with patch("torch.distributed.get_rank", return_value=0), \
            patch("torch.distributed.get_world_size", return_value=1):
        from nano_vllm_multimodal_b200.layers.embed_head import VocabParallelEmbedding
        emb = VocabParallelEmbedding(128, 1024).to(torch.bfloat16).cuda()
    with torch.no_grad():
        emb.weight.copy_(c["inputs"]["weight"])
    assert_bitexact(emb(c["inputs"]["ids"].cuda()), c["outputs"]["y"], "embedding")


def test_embedding_c2_full_vocab():
    d = W.make_layer_inputs(2, cache=False)
    w, ids = d["embedding"], d["token_ids"]
    assert w.shape == (151936, 1024)
    assert_bitexact(ops.embedding(ids.cuda(), w.cuda()), O.embedding(ids, w), "C2 embedding")


def test_embedding_tensor_parallel_mask_matches_reference_semantics():
    """tp=2 shard of rank 1: ids outside the shard give zero rows (the reference
    multiplies by the mask before its all-reduce, embed_head.py:35-41)."""
    g = torch.Generator().manual_seed(3)
    full = torch.randn(64, 256, generator=g).to(torch.bfloat16)
    shard = full[32:].contiguous()
    ids = torch.randint(0, 64, (50,), generator=g)
    out = ops.embedding(ids.cuda(), shard.cuda(), 32, 64, mask=True)
    mask = (ids >= 32) & (ids < 64)
    exp = torch.zeros(50, 256, dtype=torch.bfloat16)
    exp[mask] = full[ids[mask]]
    assert_bitexact(out, exp, "masked shard")


def test_embedding_bad_id_reported(monkeypatch):
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    w = torch.randn(16, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="out of range"):
        ops.embedding(torch.tensor([1, 16], device="cuda"), w)


def test_golden_deepstack(golden):
    c = golden["deepstack_c3"]
    i = c["inputs"]
    h = i["hidden"].cuda()
    before = h.clone()
    out = add_deepstack_rows(h, i["rows"].cuda(), i["vis"].cuda())
    assert_bitexact(out, c["outputs"]["y"], "deepstack out of place")
    assert torch.equal(h, before)  # input not mutated (tests/test_qwen3_vl_model.py:474-493)
    add_deepstack_rows_(h, i["rows"].cuda(), i["vis"].cuda())
    assert_bitexact(h, c["outputs"]["y"], "deepstack in place")


def test_deepstack_c3_three_layers():
    d = W.make_layer_inputs(3, tokens=4096, cache=False)
    rows, vis = d["deepstack_rows"], d["deepstack"]
    h = d["hidden"]
    g = h.cuda()
    for layer in range(3):
        h = O.add_deepstack_rows(h, rows, vis[layer])
        g = add_deepstack_rows(g, rows.cuda(), vis[layer].cuda())
    assert_bitexact(g, h, "three DeepStack adds")


def test_deepstack_empty_rows_return_same_object():
    h = torch.randn(3, 16, device="cuda", dtype=torch.bfloat16)
    out = add_deepstack_rows(h, torch.empty(0, dtype=torch.long, device="cuda"),
                             torch.empty(0, 16, device="cuda", dtype=torch.bfloat16))
    assert out is h


# ------------------------------------------------------- DeepStack folded into add + norm


def _deepstack_case(seed, tokens, hidden, n_vis, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, hidden, generator=g).to(dtype)
    r = torch.randn(tokens, hidden, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
    rows = torch.randperm(tokens, generator=g)[:n_vis].sort().values
    vis = torch.randn(n_vis, hidden, generator=g).to(dtype)
    return x, r, w, rows, vis


def test_deepstack_row_index():
    rows = torch.tensor([0, 3, 4, 9, 299])
    idx = ops.deepstack_row_index(rows.cuda(), 300).cpu()
    expect = torch.full((300,), -1, dtype=torch.int32)
    expect[rows] = torch.arange(5, dtype=torch.int32)
    assert torch.equal(idx, expect)
    assert torch.equal(ops.deepstack_row_index(rows[:0].cuda(), 7).cpu(), torch.full((7,), -1, dtype=torch.int32))
    assert ops.deepstack_row_index(rows[:0].cuda(), 0).numel() == 0


@pytest.mark.parametrize("hidden", [64, 1024, 2048, 4096])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_add_rms_norm_deepstack_matches_composition(hidden, dtype):
    """One pass = rounded layer-output add, _add_deepstack_rows, next input norm:
    bit-exact against the oracle composition (kernel statistics order). Covers the
    warp-per-row kernel (1..8 vectors per lane) and the CTA-per-row kernel (4096)."""
    x, r, w, rows, vis = _deepstack_case(hidden, 301, hidden, 120, dtype)
    idx = ops.deepstack_row_index(rows.cuda(), 301)
    y, s = ops.add_rms_norm_deepstack(x.cuda(), r.cuda(), w.cuda(), 1e-6, vis.cuda(), idx)
    ey, es = O.add_text_rms_norm_deepstack(x, r, w, 1e-6, rows, vis, order="kernel")
    assert_bitexact(s, es, "updated residual")
    assert_bitexact(y, ey, "normed")
    # and within the usual bound of the reference's own operation order
    ty, ts = O.add_text_rms_norm_deepstack(x, r, w, 1e-6, rows, vis)
    assert_bitexact(s, ts, "updated residual vs torch order")
    d = ulp_diff(y, ty)
    assert int(d.max()) <= 2 and int((d > 1).sum()) <= max(3, int(1e-4 * d.numel()))


def test_add_rms_norm_deepstack_fp32_weight_and_no_visual_rows():
    x, r, w, rows, vis = _deepstack_case(7, 64, 2048, 16, torch.bfloat16)
    w32 = w.float()
    idx = ops.deepstack_row_index(rows.cuda(), 64)
    y, s = ops.add_rms_norm_deepstack(x.cuda(), r.cuda(), w32.cuda(), 1e-6, vis.cuda(), idx)
    ey, es = O.add_text_rms_norm_deepstack(x, r, w32, 1e-6, rows, vis, order="kernel")
    assert_bitexact(s, es, "fp32 weight residual")
    # the reference promotes to fp32 here; the op keeps the activation dtype, i.e.
    # the fp32 product rounded once (the layer class rejects fp32 weights)
    assert_bitexact(y, ey.to(torch.bfloat16), "fp32 weight normed")
    # no visual rows at all: the plain rounded-sum add + norm
    none = ops.deepstack_row_index(rows[:0].cuda(), 64)
    y0, s0 = ops.add_rms_norm_deepstack(x.cuda(), r.cuda(), w.cuda(), 1e-6, vis[:0].cuda(), none)
    y1, s1 = ops.add_rms_norm(x.cuda(), r.cuda(), w.cuda(), 1e-6, round_sum=True)
    assert_bitexact(y0, y1, "no visual rows")
    assert_bitexact(s0, s1, "no visual rows residual")


def test_add_rms_norm_deepstack_layer_api():
    from nano_vllm_multimodal_b200.layers.qwen3_vl import Qwen3VLTextRMSNorm, deepstack_row_index
    x, r, w, rows, vis = _deepstack_case(9, 256, 2048, 64, torch.bfloat16)
    norm = Qwen3VLTextRMSNorm(2048, eps=1e-6).to(torch.bfloat16).cuda()
    with torch.no_grad():
        norm.weight.copy_(w)
    idx = deepstack_row_index(rows.cuda(), 256)
    y, s = norm(x.cuda(), r.cuda(), deepstack=(vis.cuda(), idx))
    ey, es = O.add_text_rms_norm_deepstack(x, r, w, 1e-6, rows, vis, order="kernel")
    assert_bitexact(y, ey, "layer API")
    assert_bitexact(s, es, "layer API residual")
    with pytest.raises(ValueError, match="needs the residual"):
        norm(x.cuda(), deepstack=(vis.cuda(), idx))


def test_add_rms_norm_deepstack_bad_index_reported(monkeypatch):
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    x, r, w, rows, vis = _deepstack_case(11, 32, 1024, 4, torch.bfloat16)
    idx = ops.deepstack_row_index(rows.cuda(), 32)
    idx[5] = 4  # one past the visual rows
    with pytest.raises(ValueError, match="out of range"):
        ops.add_rms_norm_deepstack(x.cuda(), r.cuda(), w.cuda(), 1e-6, vis.cuda(), idx)
    with pytest.raises(ValueError, match="out of range"):
        ops.deepstack_row_index(torch.tensor([3, 40]).cuda(), 32)
