"""Paged-KV store / gather kernels and the PagedKVCache owner (bit-exact).

Restates the reference's CUDA parity matrix
(``tests/test_paged_kv_cuda.py:80-153``: dtype x heads x head_dim x tokens x
mapping, caches prefilled with -3), its strided fused-qkv case (``:51-78``)
and its runtime-owner tests (``:155-273``), with the numpy oracle as the
expected result."""

import gc

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.attention import store_kvcache
from nano_vllm_multimodal_b200.layers.paged_kv import create_paged_kv_backend
from tests._util import assert_bitexact

pytestmark = pytest.mark.gpu


def test_golden_store_gather(golden):
    c = golden["paged_c2"]
    qkv = c["inputs"]["qkv"].cuda()
    k = qkv[:, 2048:3072].view(-1, 8, 128)
    v = qkv[:, 3072:].view(-1, 8, 128)
    kc = torch.full(c["meta"]["cache_shape"], c["meta"]["cache_fill"], dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    backend = create_paged_kv_backend("cuda")
    backend.store(k, v, kc, vc, c["inputs"]["slot_mapping"].cuda())
    assert_bitexact(kc, c["outputs"]["key_cache"], "key cache")
    assert_bitexact(vc, c["outputs"]["value_cache"], "value cache")
    g = backend.gather(kc, c["inputs"]["block_table"].cuda(), c["meta"]["sequence_length"])
    assert_bitexact(g, c["outputs"]["gathered"], "gather")


def test_store_gather_full_parity_matrix():
    torch.manual_seed(23)
    backend = create_paged_kv_backend("cuda")
    num_blocks, block_size = 41, 16
    num_slots = num_blocks * block_size
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for heads in (1, 2, 8):
            for head_dim in (64, 80, 128, 256):
                for tokens in (1, 8, 257):
                    for mapping in ("contiguous", "random_with_skips"):
                        key = torch.randn(tokens, heads, head_dim).to(dtype)
                        value = torch.randn_like(key)
                        if mapping == "contiguous":
                            slots = torch.arange(tokens, dtype=torch.int32)
                        else:
                            slots = torch.randperm(num_slots, dtype=torch.int32)[:tokens]
                            slots[::11] = -1
                        kc = torch.full((num_blocks, block_size, heads, head_dim), -3.0).to(dtype)
                        ekc, evc = O.paged_store(key, value, kc, kc.clone(), slots)
                        gkc, gvc = kc.cuda(), kc.clone().cuda()
                        stream = torch.cuda.Stream()
                        stream.wait_stream(torch.cuda.current_stream())
                        with torch.cuda.stream(stream):
                            backend.store(key.cuda(), value.cuda(), gkc, gvc, slots.cuda())
                        stream.synchronize()
                        what = f"{dtype} h{heads} d{head_dim} t{tokens} {mapping}"
                        assert_bitexact(gkc, ekc, what + " key")
                        assert_bitexact(gvc, evc, what + " value")
                        table = torch.randperm(num_blocks, dtype=torch.int32)
                        n = min(tokens, num_slots)
                        assert_bitexact(backend.gather(gkc, table.cuda(), n), O.paged_gather(ekc, table, n),
                                        what + " gather")


def test_store_accepts_fused_qkv_noncontiguous_token_stride():
    torch.manual_seed(29)
    packed = torch.randn(9, 8, 64, dtype=torch.float16)
    key, value = packed[:, 4:6], packed[:, 6:8]
    slots = torch.tensor([0, 17, 4, 31, 8, 23, 2, 15, 9], dtype=torch.int32)
    kc = torch.full((4, 8, 2, 64), -3.0, dtype=torch.float16)
    ekc, evc = O.paged_store(key, value, kc, kc.clone(), slots)
    gp = packed.cuda()
    gkc, gvc = kc.cuda(), kc.clone().cuda()
    assert gp[:, 4:6].stride(0) > 2 * 64
    store_kvcache(gp[:, 4:6], gp[:, 6:8], gkc, gvc, slots.cuda())
    assert_bitexact(gkc, ekc, "key")
    assert_bitexact(gvc, evc, "value")


def test_store_c2_full_size_skips_and_untouched():
    d = W.make_layer_inputs(2)
    qkv = d["qkv"]
    k, v = qkv[:, 2048:3072].reshape(-1, 8, 128), qkv[:, 3072:].reshape(-1, 8, 128)
    assert int((d["slot_mapping"] == -1).sum()) == 26
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
    ops.paged_store(qkv.cuda()[:, 2048:3072].view(-1, 8, 128), qkv.cuda()[:, 3072:].view(-1, 8, 128),
                    kc, vc, d["slot_mapping"].cuda())
    valid = d["slot_mapping"] >= 0
    flat_k = kc.view(-1, 8, 128)
    written = d["slot_mapping"][valid].long().cuda()
    assert_bitexact(flat_k[written], k[valid], "written rows")
    assert_bitexact(vc.view(-1, 8, 128)[written], v[valid], "written v rows")
    mask = torch.ones(flat_k.shape[0], dtype=torch.bool, device="cuda")
    mask[written] = False
    assert bool((flat_k[mask] == -3).all())  # 4096*256 - 230 slots untouched


def test_gather_varlen_matches_per_sequence_gather():
    g = torch.Generator().manual_seed(5)
    nb, bs = 64, 16
    cache = torch.randn(nb, bs, 2, 128, generator=g).to(torch.bfloat16)
    lens = [1, 16, 17, 100, 0, 255]
    tables = torch.stack([torch.randperm(nb, generator=g)[:16] for _ in lens]).to(torch.int32)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int64)
    out = ops.paged_gather_varlen(cache.cuda(), tables.cuda(), torch.tensor(lens, dtype=torch.int32).cuda(),
                                  cu.cuda(), int(cu[-1]), max(lens))
    exp = torch.cat([O.paged_gather(cache, tables[i], n) for i, n in enumerate(lens)])
    assert_bitexact(out, exp, "varlen gather")


def test_gather_c5_shape_property():
    """C5 gather at its real per-sequence length (16384 tokens through 64 random
    blocks of a 16384-block cache), checked against a direct index on the GPU
    and the CPU oracle on a slice."""
    shp = W.C5
    nb = 1024  # a 1024-block slice of the C5 cache keeps the test to 0.5 GiB
    cache = torch.randn(nb, shp.block_size, shp.num_kv_heads, shp.head_dim, device="cuda",
                        dtype=torch.bfloat16)
    tables = W.make_gather_inputs(5, sequences=4, seq_len=16384, num_blocks=nb).cuda()
    lens = torch.full((4,), 16384, dtype=torch.int32, device="cuda")
    cu = torch.arange(5, dtype=torch.int64, device="cuda") * 16384
    out = ops.paged_gather_varlen(cache, tables, lens, cu, 4 * 16384, 16384)
    direct = cache[tables.long()].reshape(4 * 16384, shp.num_kv_heads, shp.head_dim)
    assert_bitexact(out, direct, "varlen vs index")
    small = O.paged_gather(cache[:, :, :1].cpu().contiguous(), tables[0].cpu(), 1000)
    assert_bitexact(out[:1000, :1], small, "vs oracle")


def test_invalid_block_flagged_and_zero_rows(monkeypatch):
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    cache = torch.randn(4, 8, 1, 64, device="cuda", dtype=torch.float16)
    tables = torch.tensor([[0, 9]], dtype=torch.int32, device="cuda")  # 9 is out of range
    with pytest.raises(ValueError, match="invalid physical block"):
        ops.paged_gather_varlen(cache, tables, torch.tensor([16], dtype=torch.int32, device="cuda"),
                                torch.tensor([0, 16], dtype=torch.int64, device="cuda"), 16, 16)


def test_empty_inputs():
    backend = create_paged_kv_backend("cuda")
    kc = torch.full((2, 4, 1, 64), -3.0, dtype=torch.float16, device="cuda")
    empty = torch.empty(0, 1, 64, dtype=torch.float16, device="cuda")
    backend.store(empty, empty, kc, kc, torch.empty(0, dtype=torch.int32, device="cuda"))
    assert bool((kc == -3).all())
    assert backend.gather(kc, torch.tensor([1, 0], dtype=torch.int32, device="cuda"), 0).shape == (0, 1, 64)


# ---- runtime owner (torch.classes.nanovllm_paged_kv.PagedKVCache) -------------------


def test_runtime_allocation_store_and_gather():
    torch.manual_seed(11)
    backend = create_paged_kv_backend("cuda")
    alloc = backend.allocate((2, 5, 8, 2, 128), dtype=torch.bfloat16, device="cuda")
    assert alloc.owner is not None and alloc.tensor.shape == (2, 5, 8, 2, 128)
    alloc.tensor.fill_(-5)
    kc, vc = alloc.tensor[0], alloc.tensor[1]
    key = torch.randn(10, 2, 128, dtype=torch.bfloat16)
    value = torch.randn_like(key)
    slots = torch.tensor([0, 9, 17, -1, 31, 2, 7, 20, 39, 12], dtype=torch.int32)
    ekc, evc = O.paged_store(key, value, kc.cpu(), vc.cpu(), slots)
    backend.store(key.cuda(), value.cuda(), kc, vc, slots.cuda())
    assert_bitexact(kc, ekc, "key")
    assert_bitexact(vc, evc, "value")
    table = torch.tensor([4, 1, 3], dtype=torch.int32)
    assert_bitexact(backend.gather(kc, table.cuda(), 19), O.paged_gather(ekc, table, 19), "gather")


def test_runtime_owner_async_copies_pinned_slot_mapping():
    backend = create_paged_kv_backend("cuda")
    alloc = backend.allocate((2, 1, 8, 1, 64), dtype=torch.float16, device="cuda")
    host = torch.tensor([0, 3, 7], dtype=torch.int32).pin_memory()
    with torch.cuda.stream(torch.cuda.Stream()):
        dev = backend.copy_slots_async(alloc, host)
        torch.cuda.current_stream().synchronize()
    assert dev.device.type == "cuda" and torch.equal(dev.cpu(), host)


def test_runtime_owner_empty_and_reuse():
    backend = create_paged_kv_backend("cuda")
    alloc = backend.allocate((2, 1, 8, 1, 64), dtype=torch.float16, device="cuda")
    e = backend.copy_slots_async(alloc, torch.empty(0, dtype=torch.int32, pin_memory=True))
    assert e.device.type == "cuda" and e.dtype == torch.int32 and e.numel() == 0
    first = backend.copy_slots_async(alloc, torch.tensor([0, 3, 7, 2], dtype=torch.int32).pin_memory())
    torch.cuda.current_stream().synchronize()
    second_host = torch.tensor([6, 1], dtype=torch.int32).pin_memory()
    second = backend.copy_slots_async(alloc, second_host)
    torch.cuda.current_stream().synchronize()
    assert first.data_ptr() == second.data_ptr()
    assert torch.equal(second.cpu(), second_host)
    with pytest.raises(RuntimeError, match="pinned"):
        backend.copy_slots_async(alloc, torch.tensor([1], dtype=torch.int32))


def test_async_copy_retains_ephemeral_pinned_host_tensor():
    backend = create_paged_kv_backend("cuda")
    alloc = backend.allocate((2, 1, 8, 1, 64), dtype=torch.float16, device="cuda")
    host = torch.tensor([0, 3, 7], dtype=torch.int32).pin_memory()
    dev = backend.copy_slots_async(alloc, host)
    assert alloc.owner.pending_host_copy_count() == 1
    del host
    gc.collect()
    torch.cuda.current_stream().synchronize()
    assert dev.tolist() == [0, 3, 7]


def test_repeated_async_slot_copy_and_store_matches_decode_sequence():
    backend = create_paged_kv_backend("cuda")
    alloc = backend.allocate((2, 1, 16, 1, 64), dtype=torch.float16, device="cuda")
    alloc.tensor.fill_(-1)
    kc, vc = alloc.tensor[0], alloc.tensor[1]
    for step in range(64):
        key = torch.full((1, 1, 64), step, dtype=torch.float16, device="cuda")
        host = torch.tensor([step % 16], dtype=torch.int32, pin_memory=True)
        dev = backend.copy_slots_async(alloc, host)
        del host
        backend.store(key, -key, kc, vc, dev)
    torch.cuda.synchronize()
    expected = torch.arange(48, 64, dtype=torch.float16, device="cuda")
    assert torch.equal(kc[0, :, 0, 0], expected)
    assert torch.equal(vc[0, :, 0, 0], -expected)
