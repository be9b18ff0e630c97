"""Host-side pieces of bench.py that need no GPU: the command line, the clock
summary that decides whether a run is kept, and the even token split."""

import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_defaults_finish_within_the_contract():
    a = bench.parse_args([])
    assert (a.gpus, a.steps, a.warmup, a.impl) == (1, 10, 3, "ours")
    assert a.tokens == 262144 and a.layers == 28
    assert a.warmup >= 3


@pytest.mark.parametrize("name", ["decode_attention", "step_inputs", "mrope", "rows", "visual_merge", "paged_store",
                                  "head_norm"])
def test_every_standalone_component_is_accepted(name):
    assert bench.parse_args(["--component", name]).component == name


def test_unknown_component_is_rejected():
    with pytest.raises(SystemExit):
        bench.parse_args(["--component", "nothing"])


def _line(sm, reasons=()):
    flags = ["Active" if r in reasons else "Not Active"
             for r in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")]
    return ", ".join(["0", str(sm), "1965", "900.0", "0x0"] + flags)


def test_clock_summary_takes_the_median_under_load_and_collects_reasons():
    lines = [_line(345), _line(1650, ["sw_power_cap"]), _line(1700), _line(1680), "garbage", ""]
    c = bench.summarize_clocks(lines)
    # the idle sample (below half of the top clock) is left out of the median
    assert c["sm_mhz"] == 1680 and c["sm_max_mhz"] == 1965
    assert c["reasons"] == ["sw_power_cap"] and c["samples"] == 4


def test_clock_summary_reports_thermal_slowdown_and_nothing_without_samples():
    c = bench.summarize_clocks([_line(1500, ["hw_thermal_slowdown"]), _line(1520)])
    assert c["reasons"] == ["hw_thermal_slowdown"]
    assert bench.summarize_clocks([]) is None
    assert bench.summarize_clocks(["clocks.sm [MHz], ..."]) is None


@pytest.mark.parametrize("n,world", [(262144, 1), (262144, 8), (64, 3), (5, 8), (0, 2)])
def test_shards_cover_every_unit_once(n, world):
    parts = [bench.shard(n, r, world) for r in range(world)]
    at = 0
    for start, count in parts:
        assert start == at and count >= 0
        at += count
    assert at == n
    assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
