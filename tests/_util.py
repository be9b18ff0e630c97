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


def assert_matches_reference(actual, kernel_order, torch_order, what="", max_ulp=None, max_frac=None):
    """Two-level parity for ops downstream of fp32 statistics (norms):

    * bit-exact against the reference formula evaluated with the kernels'
      fp32 summation order (``order="kernel"`` in the oracle);
    * against the reference as PyTorch runs it on this CPU: within ``max_ulp``
      (16-bit: 2, float32: 4), and for 16-bit outputs at most
      ``max(3, max_frac * n)`` elements (``max_frac`` default 1e-5) beyond
      1 ulp. A last-bit difference in the
      fp32 statistics can move a value across a rounding boundary of the
      first (normalised) rounding; the weight multiply then rounds again.
    """
    assert_bitexact(actual, kernel_order, f"{what} (kernel statistics order)")
    sixteen = actual.dtype in (torch.bfloat16, torch.float16)
    if max_ulp is None:
        max_ulp = 2 if sixteen else 4
    d = assert_ulp(actual, torch_order, max_ulp, f"{what} (torch order)")
    if sixteen:
        beyond = int((d > 1).sum())
        limit = max(3, int((1e-5 if max_frac is None else max_frac) * d.numel()))
        assert beyond <= limit, f"{what}: {beyond} of {d.numel()} elements beyond 1 ulp of the torch-order result"
    return d
