"""Shared fixtures. GPU tests carry ``@pytest.mark.gpu`` and run on a B200 (``pytest -m gpu``);
everything else runs on the CPU (``pytest -m "not gpu"``)."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
