"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a machine without a GPU (oracle pins, golden fixtures, host logic, ABI
exports); `-m gpu` runs the CUDA parity tests through the C ABI on a B200."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ffnerf-experimental_b200"
for p in (PKG, ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libffnerf.so")


def pytest_collection_modifyitems(config, items):
    # tests/test_zz_* run last: a run that stops at the first failure has run everything else
    items.sort(key=lambda it: Path(str(it.fspath)).name.startswith("test_zz_"))


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()
