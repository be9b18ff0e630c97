"""Shared helpers for the parity tests."""

import os
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]


def report_dir() -> Path:
    """Where GPU tests write their measurement reports (JSON): ``$NIB_TEST_REPORT_DIR``,
    else ``test_reports/`` at the repository root (git-ignored). Created on demand."""
    d = Path(os.environ.get("NIB_TEST_REPORT_DIR") or (ROOT / "test_reports"))
    d.mkdir(parents=True, exist_ok=True)
    return d

BF16 = torch.bfloat16

# Measured parity exceptions (elements beyond 1 ulp of the reference's own
# CPU evaluation, and what they are attributed to), filled by the helpers
# below; tests/conftest.py writes it out at the end of a GPU session.
PARITY_REPORT: dict = {}


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


def _norm_statistics(s32, eps, dtype, add):
    """Per-row fp32 statistic 1/sqrt(mean(s^2) + eps) in the two orders: PyTorch's
    CPU evaluation (the reference's) and the kernels' fixed summation order."""
    from oracle import ops as o
    n = s32.shape[-1]
    rows = s32.reshape(-1, n)
    return (o._inv_rms(rows, eps, "torch", dtype, add).flatten(),
            o._inv_rms(rows, eps, "kernel", dtype, add).flatten())


def assert_matches_reference(actual, kernel_order, torch_order, what="", max_ulp=None, max_frac=None,
                             stats=None):
    """Two-level parity for ops downstream of fp32 statistics (norms):

    * bit-exact against the reference formula evaluated with the kernels'
      fp32 summation order (``order="kernel"`` in the oracle);
    * against the reference as PyTorch runs it on this CPU: within ``max_ulp``
      (16-bit: 2, float32: 4), and for 16-bit outputs at most
      ``max(3, max_frac * n)`` elements (``max_frac`` default 1e-5) beyond
      1 ulp. A last-bit difference in the
      fp32 statistics can move a value across a rounding boundary of the
      first (normalised) rounding; the weight multiply then rounds again.

    ``stats=(s32, eps, add)`` (the fp32 rows the statistic is taken over)
    attributes every exception: each element beyond 1 ulp of the torch-order
    result must sit in a row whose fp32 statistic differs between the two
    orders, and rows whose statistics agree must match the torch order bit for
    bit. The counts and the largest statistic difference (fp32 ulps) go to
    ``PARITY_REPORT``.
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
    if stats is not None:
        s32, eps, add = stats
        st_torch, st_kernel = _norm_statistics(s32.float(), eps, actual.dtype, add)
        differs = st_torch != st_kernel                       # [rows]
        dr = d.reshape(differs.numel(), -1)
        assert not bool((dr > 1)[~differs].any()), \
            f"{what}: an element beyond 1 ulp in a row whose fp32 statistic agrees"
        assert not bool((dr > 0)[~differs].any()), \
            f"{what}: a row with the same fp32 statistic is not bit-exact against the torch order"
        stat_ulps = ulp_diff(st_torch, st_kernel)
        PARITY_REPORT.setdefault("norms", {})[what] = {
            "rows": int(differs.numel()), "rows_with_different_statistic": int(differs.sum()),
            "max_statistic_diff_fp32_ulp": int(stat_ulps.max()) if stat_ulps.numel() else 0,
            "elements": int(d.numel()), "elements_beyond_1ulp": int((d > 1).sum()),
            "max_ulp": int(d.max()) if d.numel() else 0}
    return d


def rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def assert_trig_bounded(actual, expected, x, trig_differs, what=""):
    """M-RoPE against the CPU oracle when cos/sin may differ in the last bit.

    Tokens whose cos/sin all agree with the CPU's: every element within 1 ulp.
    Tokens where some cos or sin differs (by 1 bf16 ulp, checked by the caller):
    every element within the effect of that difference, propagated through the
    rotation ``o = x*cos + rot(x)*sin`` with its roundings:
    ``|a - o| <= 2**-6 * (|x| + |rot(x)|) + 2 ulp(o)``. The counts and the largest
    share of that bound go to ``PARITY_REPORT``.
    ``actual``/``expected``/``x``: [tokens, heads, D]; ``trig_differs``: [tokens].
    """
    a, e, xx = actual.detach().cpu(), expected.detach().cpu(), x.detach().cpu()
    d = ulp_diff(a, e)
    tok_bad = (d > 1).any(dim=-1).any(dim=-1)
    assert not bool((tok_bad & ~trig_differs).any()), f"{what}: > 1 ulp at a token whose cos/sin agree"
    ef = e.float()
    spacing = torch.exp2(torch.floor(torch.log2(ef.abs().clamp_min(2.0 ** -126))) - 7)
    bound = 2.0 ** -6 * (xx.float().abs() + rotate_half(xx.float()).abs()) + 2 * spacing
    err = (a.float() - ef).abs()
    sel = trig_differs
    ratio = float((err[sel] / bound[sel]).max()) if bool(sel.any()) else 0.0
    assert ratio <= 1.0, f"{what}: error {ratio:.3f} x the propagated bound of a 1-ulp cos/sin difference"
    PARITY_REPORT.setdefault("mrope", {})[what] = {
        "tokens": int(trig_differs.numel()), "tokens_with_trig_difference": int(trig_differs.sum()),
        "elements_beyond_1ulp": int((d > 1).sum()), "max_ulp": int(d.max()) if d.numel() else 0,
        "max_share_of_bound": round(ratio, 4)}
    return d
