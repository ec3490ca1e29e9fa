"""pytest configuration: the `gpu` marker and import paths for the product package and the oracle."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "marlin-mlx_b200", ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built libmarlin_q4.so")


@pytest.fixture(scope="session")
def oracle():
    import q4_oracle
    return q4_oracle.COracle()
