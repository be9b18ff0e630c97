"""Programmatic dependent launch (``NIB_B200_PDL=1``, off by default) changes
only when a kernel's CTAs are scheduled: every kernel waits for its
predecessor's completion before it touches global memory. So a fixed chain of
the library's kernels must give the same bits with it off and on, eagerly and
replayed from a CUDA graph (``tests/_pdl_child.py``; the switch is read once
per process, hence one child process per mode)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _run(pdl: bool) -> dict:
    env = dict(os.environ)
    env.pop("NIB_B200_PDL", None)
    if pdl:
        env["NIB_B200_PDL"] = "1"
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "_pdl_child.py")], env=env, cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_programmatic_dependent_launch_gives_the_same_bits():
    off, on = _run(False), _run(True)
    assert off["eager"] == off["graph"], "graph replay differs from the eager chain (launch off)"
    assert on["eager"] == on["graph"], "graph replay differs from the eager chain (launch on)"
    assert off["eager"] == on["eager"], "programmatic dependent launch changed the results"
