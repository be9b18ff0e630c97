"""Seeded paged-KV store / gather inputs shared by a test and its child process
(plain torch: the child must not load this repo's binding)."""

import torch

DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def parity_cases():
    """The reference's CUDA/PyTorch parity matrix (its tests/test_paged_kv_cuda.py:80-153):
    dtype x kv heads x head_dim x tokens x slot pattern, caches prefilled with -3."""
    cases = []
    seed = 0
    for dtype in DTYPES:
        for heads in (1, 2, 8):
            for dim in (64, 80, 128, 256):
                for tokens in (1, 8, 257):
                    for pattern in ("contiguous", "random"):
                        seed += 1
                        cases.append((seed, dtype, heads, dim, tokens, pattern))
    return cases


def parity_inputs(seed, dtype, heads, dim, tokens, pattern, block_size=16):
    g = torch.Generator().manual_seed(seed)
    blocks = (tokens + block_size - 1) // block_size + 2
    key = torch.randn(tokens, heads, dim, generator=g).to(dtype)
    value = torch.randn(tokens, heads, dim, generator=g).to(dtype)
    if pattern == "contiguous":
        slots = torch.arange(tokens, dtype=torch.int32)
    else:
        slots = torch.randperm(blocks * block_size, generator=g)[:tokens].to(torch.int32)
        slots[::11] = -1
    cache_shape = (blocks, block_size, heads, dim)
    table = torch.randperm(blocks, generator=g).to(torch.int32)
    return key, value, slots, cache_shape, table


def timing_inputs(device):
    """C5 head shapes: store of 65,536 tokens (k/v strided views of qkv rows) into a
    1,024-block cache pair; gather of 16 sequences x 16,384 tokens from it."""
    g = torch.Generator().manual_seed(4242)
    tokens, nq, nkv, dim = 65536, 16, 8, 128
    qkv = torch.randn(tokens, (nq + 2 * nkv) * dim, generator=g).to(torch.bfloat16).to(device)
    k = qkv[:, nq * dim:(nq + nkv) * dim].view(tokens, nkv, dim)
    v = qkv[:, (nq + nkv) * dim:].view(tokens, nkv, dim)
    slots = torch.randperm(1024 * 256, generator=g)[:tokens].to(torch.int32).to(device)
    tables = torch.stack([torch.randperm(1024, generator=g)[:64] for _ in range(16)]).to(torch.int32).to(device)
    return k, v, slots, tables


def time_ms(fn, flush, reps=10, warmup=3):
    """Median of one call at a time, each after writing a 512 MB buffer and reading it
    back (the L2 flushed and left clean, so no call pays for the flush's write-back)."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        flush.zero_()
        flush.view(torch.int64).sum()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return sorted(times)[len(times) // 2]


def digest(*tensors):
    """sha256 of the tensors' bytes, in order (large results compared without a host copy kept)."""
    import hashlib
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().contiguous().view(torch.uint8).cpu().numpy().tobytes())
    return h.hexdigest()
