"""The allocation-free paged gather, called through the C ABI.

Some callers cannot allocate device memory: hosts whose memory planner
reserves the whole GPU up front and hands a library only the buffers it asked
for, and runtimes that forbid cudaMalloc/cudaFree on the serving path (both
synchronise the device). ``nib_paged_gather_varlen_noalloc`` serves them:
the caller passes the cache, block tables, sequence lengths and the output
buffer, and the per-sequence output offsets (which ``nib_paged_gather_varlen``
takes from its caller) are built in a fixed device array of the library.

The tests check its output against the existing entry point on two calls in a
row (the second with fewer sequences, so stale offsets from the first would
show), bit-exact as every gather test here; against the CPU oracle at 1, 1001
and 4096 sequences (the table's capacity: the last scan thread writes the
final offset) with lengths that include 0 and -1 (a negative length gathers
nothing); a call captured in a CUDA graph and replayed after the lengths were
changed in place; and that batches above the table's capacity are refused.
This file is named to be collected last.
"""

import ctypes

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import _lib, ops

pytestmark = pytest.mark.gpu

NIB_BF16 = 2
MAX_SEQS = 4096  # NIB_NOALLOC_MAX_SEQS in include/nib_b200.h


def _bind():
    lib = _lib.cdll()
    f = lib.nib_paged_gather_varlen_noalloc
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    f.argtypes = [ctypes.c_int, vp, i64, i64, i64, i64, i64, vp, i64, vp, i64, i64, vp, vp, vp]
    f.restype = ctypes.c_int
    lib.nib_last_error.restype = ctypes.c_char_p
    return lib, f


def _noalloc_gather(f, cache, tables, lens, total, max_len):
    out = torch.empty(total, cache.shape[2], cache.shape[3], dtype=cache.dtype, device=cache.device)
    rc = f(NIB_BF16, cache.data_ptr(), cache.stride(0), cache.stride(1), cache.shape[0], cache.shape[1],
           cache.shape[2] * cache.shape[3], tables.data_ptr(), tables.stride(0), lens.data_ptr(),
           lens.numel(), max_len, out.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    return rc, out


def _case(seed, lens, nb=96, bs=16):
    g = torch.Generator().manual_seed(seed)
    cache = torch.randn(nb, bs, 2, 128, generator=g).to(torch.bfloat16).cuda()
    need = max(1, -(-max(lens) // bs))
    tables = torch.stack([torch.randperm(nb, generator=g)[:need] for _ in lens]).to(torch.int32).cuda()
    lens_t = torch.tensor(lens, dtype=torch.int32).cuda()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int64).cuda()
    return cache, tables, lens_t, cu, int(sum(lens)), max(lens)


def test_noalloc_gather_matches_existing_entry_point_twice():
    lib, f = _bind()
    for seed, lens in ((1, [5, 300, 0, 17, 256, 1, 129]), (2, [40, 3, 250])):
        cache, tables, lens_t, cu, total, max_len = _case(seed, lens)
        rc, out = _noalloc_gather(f, cache, tables, lens_t, total, max_len)
        assert rc == 0, lib.nib_last_error().decode()
        ref = ops.paged_gather_varlen(cache, tables, lens_t, cu, total, max_len)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"seed {seed}: outputs differ"


def test_noalloc_gather_refuses_batches_above_the_table():
    lib, f = _bind()
    cache, tables, lens_t, _, total, max_len = _case(3, [4])
    big = lens_t.repeat(MAX_SEQS + 1)
    rc = f(NIB_BF16, cache.data_ptr(), cache.stride(0), cache.stride(1), cache.shape[0], cache.shape[1],
           cache.shape[2] * cache.shape[3], tables.data_ptr(), 0, big.data_ptr(), big.numel(), max_len,
           cache.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"exceed the fixed offset table" in lib.nib_last_error()


def _oracle_gather(cache, tables, lens):
    """Sequence after sequence, max(len, 0) rows each, from the CPU oracle."""
    cache_c, tables_c = cache.cpu(), tables.cpu()
    parts = [O.paged_gather(cache_c, tables_c[i], max(int(n), 0)) for i, n in enumerate(lens.tolist())]
    return torch.cat(parts) if parts else cache_c.new_empty((0, *cache_c.shape[2:]))


@pytest.mark.parametrize("num_seqs", [1, 1001, MAX_SEQS])
def test_noalloc_gather_matches_the_oracle_across_the_offset_table(num_seqs):
    """Random lengths in [-1, 9] (0 and -1 included): the scan crosses warps and,
    at 4096 sequences, every one of the 1024 threads' four entries is used."""
    lib, f = _bind()
    g = torch.Generator().manual_seed(num_seqs)
    nb, bs = 64, 4
    cache = torch.randn(nb, bs, 2, 128, generator=g).to(torch.bfloat16).cuda()
    lens = torch.randint(-1, 10, (num_seqs,), generator=g, dtype=torch.int32)
    lens[0] = 9
    if num_seqs > 2:
        lens[1], lens[2] = 0, -1
    tables = torch.randint(0, nb, (num_seqs, 3), generator=g, dtype=torch.int32).cuda()
    total = int(lens.clamp(min=0).sum())
    rc, out = _noalloc_gather(f, cache, tables, lens.cuda(), total, 9)
    assert rc == 0, lib.nib_last_error().decode()
    torch.cuda.synchronize()
    ref = _oracle_gather(cache, tables, lens)
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))
    cu = torch.cat([torch.zeros(1, dtype=torch.int64), lens.clamp(min=0).cumsum(0)]).cuda()
    other = ops.paged_gather_varlen(cache, tables, lens.cuda(), cu, total, 9)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), other.view(torch.int16))


def test_noalloc_gather_in_a_cuda_graph_reads_lengths_at_replay():
    """Warm-up call first (it looks up the table's address), then a captured
    call; the lengths are changed in place and the graph replayed."""
    lib, f = _bind()
    g = torch.Generator().manual_seed(11)
    nb, bs = 32, 16
    cache = torch.randn(nb, bs, 2, 128, generator=g).to(torch.bfloat16).cuda()
    tables = torch.stack([torch.randperm(nb, generator=g)[:4] for _ in range(5)]).to(torch.int32).cuda()
    lens = torch.tensor([30, 64, 1, 17, 40], dtype=torch.int32).cuda()
    total, max_len = int(lens.sum()), 64
    out = torch.zeros(total, 2, 128, dtype=torch.bfloat16, device="cuda")
    args = lambda st: (NIB_BF16, cache.data_ptr(), cache.stride(0), cache.stride(1), nb, bs, 256,
                       tables.data_ptr(), tables.stride(0), lens.data_ptr(), 5, max_len, out.data_ptr(),
                       None, st)
    assert f(*args(torch.cuda.current_stream().cuda_stream)) == 0, lib.nib_last_error().decode()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rc = f(*args(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.nib_last_error().decode()
    for new in ([5, 0, 64, 2, 33], [-1, 10, 3, 50, 1]):
        lens.copy_(torch.tensor(new, dtype=torch.int32))
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        ref = _oracle_gather(cache, tables, lens.cpu())
        n = ref.shape[0]
        assert torch.equal(out[:n].cpu().view(torch.int16), ref.view(torch.int16)), new
        assert not out[n:].any(), "rows past the new total were written"
