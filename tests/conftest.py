import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import ctypes
        lib = ctypes.CDLL("libcuda.so.1")
        n = ctypes.c_int(0)
        return lib.cuInit(0) == 0 and lib.cuDeviceGetCount(ctypes.byref(n)) == 0 and n.value > 0
    except OSError:
        return False


@pytest.fixture(scope="session")
def gpu_lib():
    """The product library on a GPU machine; GPU tests fail (not skip) without it."""
    from nebula_b200 import lib
    if not lib.LIB_PATH.exists():
        raise RuntimeError("libqwen_gpu.so is not built")
    return lib.load()


@pytest.fixture(scope="session")
def ref2048():
    from oracle import oracle
    return oracle.RefCPU(2048, 512)


@pytest.fixture(scope="session")
def ref2560():
    from oracle import oracle
    return oracle.RefCPU(2560, 640)


@pytest.fixture(scope="session")
def restate():
    from oracle import oracle
    return oracle.Restate()


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# The float parity bar stated for the path: rel-L2 <= 1e-5 and
# max-abs <= 1e-4 * max|ref| against the reference CPU MoE.
REL_L2 = 1e-5
MAX_ABS = 1e-4


def assert_parity(out, ref, what=""):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    r = rel_l2(out, ref)
    m = float(np.max(np.abs(out - ref))) if out.size else 0.0
    bound = MAX_ABS * float(np.max(np.abs(ref))) if ref.size else 0.0
    assert r <= REL_L2, f"{what}: rel-L2 {r:.3e} > {REL_L2}"
    assert m <= bound, f"{what}: max-abs {m:.3e} > {bound:.3e}"
    return r, m
