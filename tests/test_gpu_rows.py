"""Embedding row gather and DeepStack add vs the oracle (bit-exact)."""

from unittest.mock import patch

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.qwen3_vl import add_deepstack_rows, add_deepstack_rows_
from tests._util import assert_bitexact

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
