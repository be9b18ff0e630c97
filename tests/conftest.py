import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "golden.pt", weights_only=True)


def pytest_sessionfinish(session, exitstatus):
    """Write the measured parity exceptions (tests/_util.PARITY_REPORT) to
    parity_report.json in the report directory (tests/_util.report_dir) when a
    GPU session produced any."""
    try:
        from tests._util import PARITY_REPORT, report_dir
    except ImportError:
        return
    if PARITY_REPORT:
        import json
        (report_dir() / "parity_report.json").write_text(json.dumps(PARITY_REPORT, indent=1, sort_keys=True))
