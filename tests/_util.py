"""Shared helpers for the parity tests."""

import torch

BF16 = torch.bfloat16


def ordered_bits(t: torch.Tensor) -> torch.Tensor:
    """Map a float tensor's bit patterns to integers whose difference counts
    ulps (+0 and -0 both map to 0)."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        b = t.view(torch.int16).to(torch.int64) & 0xFFFF
        sign = (b & 0x8000) != 0
        mag = b & 0x7FFF
    elif t.dtype == torch.float32:
        b = t.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        sign = (b & 0x80000000) != 0
        mag = b & 0x7FFFFFFF
    else:
        raise TypeError(t.dtype)
    return torch.where(sign, -mag, mag)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.shape == b.shape, (a.shape, b.shape)
    assert a.dtype == b.dtype, (a.dtype, b.dtype)
    return (ordered_bits(a) - ordered_bits(b)).abs()


def assert_ulp(actual, expected, max_ulp=1, what=""):
    """Every element within ``max_ulp`` units in the last place (NaNs must match)."""
    a, e = actual.detach().cpu(), expected.detach().cpu()
    assert a.shape == e.shape, (what, a.shape, e.shape)
    assert a.dtype == e.dtype, (what, a.dtype, e.dtype)
    na, ne = torch.isnan(a.float()), torch.isnan(e.float())
    assert torch.equal(na, ne), f"{what}: NaN positions differ"
    d = ulp_diff(torch.where(na, torch.zeros_like(a), a), torch.where(ne, torch.zeros_like(e), e))
    worst = int(d.max()) if d.numel() else 0
    assert worst <= max_ulp, (f"{what}: max ulp diff {worst} > {max_ulp} "
                              f"({int((d > max_ulp).sum())} of {d.numel()} elements)")
    return d


def assert_bitexact(actual, expected, what=""):
    a, e = actual.detach().cpu(), expected.detach().cpu()
    assert a.shape == e.shape and a.dtype == e.dtype, (what, a.shape, e.shape, a.dtype, e.dtype)
    ai = a.contiguous().view(torch.uint8) if a.numel() else a
    ei = e.contiguous().view(torch.uint8) if e.numel() else e
    assert torch.equal(ai, ei), f"{what}: not bit-exact"


def cuda(*ts):
    return tuple(t.cuda() if torch.is_tensor(t) else t for t in ts)
