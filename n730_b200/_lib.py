"""ctypes bindings of the two native libraries.

``cuda()`` loads ``lib/n730_cuda.so`` and declares every symbol of
``include/n730_cuda.h``; ``core()`` loads ``lib/n730core.so``
(``include/n730core.h``).  The first block of ``_CUDA_SIGS`` is the
reference's own table (``src-code/inference.py:46-138``); the reference's
Python host code can bind the same library with its own table unchanged.
There is no fallback: a missing library raises ``FileNotFoundError``.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"

vp, fp, bp, pp = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.POINTER(C.c_void_p)
i32, i64, f32, u64 = C.c_int32, C.c_int64, C.c_float, C.c_uint64
i64p = C.POINTER(C.c_int64)

_CUDA_SIGS = {
    # --- reference ABI (inference.py:54-138) ---
    "n730_cuda_init": ([i32, i32, i32, i32, i32, i32, pp], i32),
    "n730_cuda_destroy": ([vp], None),
    "n730_load_activations": ([vp, fp, i32, i32], i32),
    "n730_get_activations": ([vp, fp, i32, i32], i32),
    "n730_upload_weight": ([vp, bp, i32, i32, f32, f32], i32),
    "n730_upload_norm_weight": ([fp, i32, pp], i32),
    "n730_free_device_buf": ([vp], None),
    "n730_rmsnorm": ([vp, vp, i32, f32], i32),
    "n730_linear": ([vp, vp, i32, i32, i32], i32),
    "n730_linear_from_buf": ([vp, fp, fp, i32, i32, i32], i32),
    "n730_residual_add": ([vp, vp, i32], i32),
    "n730_add_bias": ([vp, fp, fp, i32, i32], i32),
    "n730_swiglu": ([vp, vp, i32, i32], i32),
    "n730_apply_rope": ([vp, vp, vp, i32, i32, i32, i32], i32),
    "n730_rope_precompute": ([i32, i32, f32, pp, pp], i32),
    "n730_softmax_scores": ([vp, i32, i32, i32, i32], i32),
    "n730_attention_forward": ([vp, fp, fp, fp, fp, i32, i32, i32, i32, i32, i32], i32),
    "n730_attention_qk_only": ([vp, fp, fp, i32, i32, i32, i32, i32], i32),
    "n730_get_scores": ([vp, fp, i32, i32, i32], i32),
    "n730_device_alloc": ([i32, pp], i32),
    "n730_device_free": ([vp], None),
    "n730_memcpy_d2d": ([vp, vp, i32], i32),
    "n730_memcpy_h2d": ([vp, fp, i32], i32),
    "n730_memcpy_d2h": ([fp, vp, i32], i32),
    "n730_sync": ([], i32),
    "n730_cuda_version": ([], C.c_char_p),
    # --- fast path ---
    "n730_last_error": ([], C.c_char_p),
    "n730_qweight_create": ([i32, i32, i32, i32, f32, f32, vp, vp, vp, i32, vp, pp], i32),
    "n730_qweight_destroy": ([vp], None),
    "n730_qweight_info": ([vp, i64p], i32),
    "n730_qweight_set_layout": ([vp, i32, vp], i32),
    "n730_dequant_to_f32": ([vp, vp, vp], i32),
    "n730_embed": ([vp, vp, i32, vp, vp], i32),
    "n730_qlinear": ([vp, vp, i32, i32, vp, i32, vp, vp, i32, vp, f32, i32, vp], i32),
    "n730_quantize_grouped": ([vp, i32, i32, i32, i32, vp, vp, vp, vp], i32),
    "n730_qgemm": ([vp, vp, i32, i32, vp, i32, vp, vp, i32, vp, f32, i32, vp, vp], i32),
    "n730_sample": ([vp, i32, i32, i32, f32, f32, u64, u64, vp, vp, vp], i32),
    "n730_qweight_load_blocks": ([C.c_char_p, i32, vp, vp, vp, vp], i32),
    "n730_tp_wait_check": ([i64, i32, vp], i32),
    "n730_attention_forward_noalloc": ([vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp], i32),
}

_CORE_SIGS = {
    # scheduler.py:56-84
    "n730_open": ([C.c_char_p], i64),
    "n730_close": ([i64], None),
    "n730_read_layer": ([i64, i64, fp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)], i32),
    "n730_layer_elements": ([i64, i64], i32),
    "n730_probe_layer_size": ([i64, i64], i32),
    "n730_version": ([], C.c_char_p),
    "n730_read_block": ([i64, i64, i64p, vp, i64], i32),
}

CUDA_ERRORS = {-10: "CUDA error", -11: "out of device memory", -12: "null pointer",
               -13: "bad argument", -14: "unsupported", -15: "device wait timed out",
               -16: "wrong state", -17: "collective error"}
CORE_ERRORS = {-1: "BAD_MAGIC — not a valid .n730 file", -2: "FILE — I/O error",
               -3: "ALLOC — out of memory", -4: "BAD_LAYER — corrupt layer block",
               -5: "BAD_PREC — unknown precision id", -6: "NULL — null pointer"}

_cuda = None
_core = None


def _load(name: str, sigs: dict):
    path = Path(os.environ.get("N730_LIB_DIR", LIB_DIR)) / name
    if not path.exists():
        raise FileNotFoundError(
            f"{path} not found: build the native libraries with `python -m n730_b200.build` "
            f"(there is no CPU fallback)")
    lib = C.CDLL(str(path))
    for fn, (args, res) in sigs.items():
        f = getattr(lib, fn)
        f.argtypes = args
        f.restype = res
    return lib


def cuda():
    global _cuda
    if _cuda is None:
        _cuda = _load("n730_cuda.so", _CUDA_SIGS)
    return _cuda


def core():
    global _core
    if _core is None:
        _core = _load("n730core.so", _CORE_SIGS)
    return _core


class N730Error(RuntimeError):
    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        msg = CUDA_ERRORS.get(code, CORE_ERRORS.get(code, f"error {code}"))
        super().__init__(f"{where}: {msg} ({code}){': ' + detail if detail else ''}")


def check(rc: int, where: str = ""):
    """Raise on a negative return code (the reference's check(), inference.py:141-143)."""
    if rc is not None and rc < 0:
        detail = ""
        if _cuda is not None and rc <= -10:
            d = _cuda.n730_last_error()
            detail = d.decode() if d else ""
        raise N730Error(rc, where, detail)
    return rc
