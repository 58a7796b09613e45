"""Shared pytest setup: import paths and the ``gpu`` marker."""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO / "mlir-cim22_b200", REPO / "oracle", REPO / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    return oracle
