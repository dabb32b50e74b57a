"""Shared pytest configuration: the `gpu` marker and import paths."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def built_library():
    """Builds (or reuses) libsandmuon_b200.so in-tree."""
    from sandmuon_b200.csrc.build import build
    return build()
