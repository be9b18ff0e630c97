"""Boundary indices and a head shape the config tests do not use.

* Qwen2.5-VL-7B-like attention (28 q / 4 kv heads of 128, chunked M-RoPE
  [16,24,24], no q/k norm): seven q head groups and one k group, through both
  prologue kernels, with the first and the last cache slot written and -1 slots
  skipped; bit-exact against the oracle given the kernel's own cos/sin.
* 1-D RoPE at position 0 and at the last row of the cos/sin table.
* A paged gather through block 0 and the last block, of a length that ends
  exactly on a block boundary and of one that ends inside a block.
* Embedding ids 0 and vocab - 1.
"""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops
from tests._util import assert_bitexact

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


@pytest.mark.parametrize("T,variant", [(777, 1), (2500, 2)])
def test_qwen25_vl_7b_heads_first_and_last_slot(T, variant):
    nq, nkv, D, sections = 28, 4, 128, (16, 24, 24)
    g = torch.Generator().manual_seed(T)
    qkv = torch.randn(T, (nq + 2 * nkv) * D, generator=g).to(BF)
    blocks, bs = 32, 128
    slots = torch.randperm(blocks * bs - 2, generator=g)[:T].to(torch.int32) + 1
    slots[0], slots[T // 2], slots[-1] = 0, blocks * bs - 1, -1
    slots[1::13] = -1
    pos = torch.randint(0, 16384, (3, T), generator=g)
    pos[:, 0] = 0
    inv = O.mrope_inv_freq(D, 1e6)
    kc = torch.full((blocks, bs, nkv, D), -3.0, dtype=BF)
    vc = kc.clone()
    gq = qkv.cuda()
    q, k, v = gq.split([nq * D, nkv * D, nkv * D], -1)
    gkc, gvc = kc.cuda(), vc.cuda()
    aq, ak = ops.qk_prologue(q.view(T, nq, D), k.view(T, nkv, D), v=v.view(T, nkv, D), positions=pos.cuda(),
                             rope_mode=ops.ROPE_MROPE_CHUNKED, inv_freq=inv.cuda(), sections=sections,
                             key_cache=gkc, value_cache=gvc, slot_mapping=slots.cuda(), variant=variant)
    cos, sin = ops.mrope_cos_sin(pos.cuda(), inv.cuda(), BF)
    cq, ck, cv = qkv.split([nq * D, nkv * D, nkv * D], -1)
    eq, ek = O.apply_mrope(cq.reshape(T, nq, D), ck.reshape(T, nkv, D), cos.cpu(), sin.cpu(), sections, "chunked")
    assert_bitexact(aq, eq, "q")
    assert_bitexact(ak, ek, "k")
    ekc, evc = O.paged_store(ek, cv.reshape(T, nkv, D), kc, vc, slots)
    assert_bitexact(gkc, ekc, "key cache (slots 0 and last written, -1 skipped)")
    assert_bitexact(gvc, evc, "value cache")


def test_rope_table_first_and_last_row():
    D, rows, T = 128, 4096, 64
    g = torch.Generator().manual_seed(11)
    table = O.rope_cos_sin_cache(D, rows, 1e6)
    pos = torch.randint(0, rows, (T,), generator=g)
    pos[0], pos[1], pos[-1] = 0, rows - 1, rows - 1
    q = torch.randn(T, 16, D, generator=g).to(BF)
    k = torch.randn(T, 8, D, generator=g).to(BF)
    aq, ak = ops.rope(pos.cuda(), q.cuda(), k.cuda(), table.cuda())
    eq, ek = O.apply_rope(pos, q, k, table)
    assert_bitexact(aq, eq, "q")
    assert_bitexact(ak, ek, "k")


def test_gather_first_and_last_block_and_embedding_ends():
    g = torch.Generator().manual_seed(12)
    blocks, bs = 16, 64
    cache = torch.randn(blocks, bs, 2, 128, generator=g).to(BF)
    table = torch.tensor([blocks - 1, 0, 7, blocks - 1], dtype=torch.int32)
    gc, gt = cache.cuda(), table.cuda()
    for n in (4 * bs, 3 * bs + 1, 1):
        assert_bitexact(ops.paged_gather(gc, gt, n), O.paged_gather(cache, table, n), f"gather {n}")
    vocab, H = 1000, 256
    w = torch.randn(vocab, H, generator=g).to(BF)
    ids = torch.tensor([0, vocab - 1, 5, vocab - 1, 0], dtype=torch.int64)
    assert_bitexact(ops.embedding(ids.cuda(), w.cuda()), O.embedding(ids, w), "embedding ends")
