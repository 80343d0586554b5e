import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(GOLDEN / "ref_small.npz")


@pytest.fixture(scope="session")
def oracle_c():
    """The plain-C oracle library (built by oracle/Makefile)."""
    import ctypes
    import subprocess
    so = REPO / "oracle" / "liboracle_c.so"
    if not so.exists():
        subprocess.run(["make", "-C", str(REPO / "oracle"), str(so)], check=True,
                       capture_output=True)
    lib = ctypes.CDLL(str(so))
    c = ctypes
    lib.oracle_dequant_tensor.argtypes = [c.c_void_p, c.c_int, c.c_int64, c.c_float, c.c_float, c.c_void_p]
    lib.oracle_dequant_grouped.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p, c.c_int, c.c_int64,
                                           c.c_int64, c.c_int64, c.c_void_p]
    lib.oracle_rope_table.argtypes = [c.c_int, c.c_int, c.c_float, c.c_void_p, c.c_void_p]
    lib.oracle_half_to_float.argtypes = [c.c_uint16]
    lib.oracle_half_to_float.restype = c.c_float
    return lib
