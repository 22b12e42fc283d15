import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))



def _reference_dir():
    """qw6's source tree, for the tests that read or compile it: $QW6_REF, else
    BASELINE.json's `reference_path`.  None when neither names an existing
    tree (those tests then skip)."""
    p = os.environ.get("QW6_REF")
    if not p:
        try:
            import json
            p = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            p = None
    return Path(p) if p and Path(p).is_dir() else None


REF_DIR = _reference_dir() or ROOT / "_no_reference_tree"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libqw6cuda on cuda:0)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref/libqw6ref.so not built (reference tree absent when building)")
    return Reference()


@pytest.fixture
def rng():
    return np.random.Generator(np.random.PCG64(1234))


def rel_err(y, ref):
    """max|y - ref| / max|ref| (the north-star tolerance metric)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / (den if den > 0 else 1.0))


def same_bits(a, b):
    """Bit-identical fp32 arrays; NaN positions must agree (payloads may not:
    the CPU and the GPU produce different default NaNs for inf*0)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a.view(np.uint32)[~na], b.view(np.uint32)[~nb])


@pytest.fixture(scope="session")
def cuda():
    """The in-tree CUDA library and a context on cuda:0 (gpu tests only)."""
    from qw6_b200 import lib
    lib.load()
    ctx = lib.Context(0)
    yield ctx
    ctx.close()
