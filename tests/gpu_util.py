"""Helpers for GPU tests: device buffers through torch, calls through the C ABI."""
import ctypes as C

import numpy as np

from n730_b200 import _lib


def torch():
    import torch as t
    return t


def dev(a, dtype=None):
    t = torch()
    x = t.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        x = x.to(dtype)
    return x.cuda()


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def qweight_from_oracle(prec, w_rows, w_cols, codes, scale=1.0, zp=0.0, s16=None, z16=None, group=0):
    """Register packed codes from host numpy arrays; returns the handle."""
    lib = _lib.cuda()
    out = C.c_void_p()
    codes = np.ascontiguousarray(np.frombuffer(bytes(codes), np.uint8) if isinstance(codes, (bytes, bytearray)) else codes)
    sp = s16.ctypes.data_as(C.c_void_p) if s16 is not None else None
    zpp = z16.ctypes.data_as(C.c_void_p) if z16 is not None else None
    rc = lib.n730_qweight_create(prec, w_rows, w_cols, group, scale, zp, codes.ctypes.data_as(C.c_void_p),
                                 sp, zpp, 0, None, C.byref(out))
    _lib.check(rc, "qweight_create")
    return out


def rel_err(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))
