import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the vlb200 C ABI on cuda:0)")


@pytest.fixture(scope="session")
def grids():
    from vastloom_b200 import GRIDS_PATH, read_codebooks

    if not GRIDS_PATH.exists():
        from vastloom_b200.build import build_codebooks

        if not build_codebooks():
            pytest.skip("codebook data file is not built")
    return read_codebooks()


@pytest.fixture(scope="session")
def oracle(grids):
    from oracle.oracle import Oracle

    return Oracle(grids)


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference

    if not Reference.available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built")
    return Reference()


@pytest.fixture(scope="session")
def device(grids):
    import vastloom_b200 as vb

    if vb.device_count() == 0:
        pytest.fail("no CUDA device: GPU tests must run on a B200")
    dev = vb.Device(0)
    yield dev
    dev.close()


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """Norm-wise relative error max|a-b| / max|b| (element-wise relative error is meaningless
    near zero)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / (den if den > 0 else 1.0))
