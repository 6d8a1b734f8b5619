"""Shared pytest configuration: the `gpu` marker and import paths."""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for sub in (REPO, REPO / "oracle"):
    if str(sub) not in sys.path:
        sys.path.insert(0, str(sub))


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return REPO / "tests" / "golden"
