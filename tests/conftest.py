"""Shared pytest configuration.

GPU tests carry ``@pytest.mark.gpu``; ``-m "not gpu"`` runs the CPU suite
(oracle against the golden vectors, host logic, the C-ABI export check).
"""
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.json"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def golden():
    return json.loads(GOLDEN.read_text())


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle
