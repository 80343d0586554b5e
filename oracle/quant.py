"""Oracle: quantisers and dequantisers of the N730 packed-weight format.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Per-tensor formats restate ``src-code/converter.py:41-115`` (quantise) and
``src-code/converter.py:344-371`` / ``src-code/cpp/n730core.cpp:57-142``
(dequantise).  The arithmetic is kept exactly:

* INT8: symmetric, ``scale = absmax/127``, ``q = clip(round(w/scale),-127,127)+128``,
  ``zero_point = 128`` (converter.py:41-51).
* INT4 / INT2: asymmetric, ``scale = (max-min)/qmax`` in float64,
  ``zp = clip(round(-min/scale), 0, qmax)``,
  ``q = clip(round(w/scale)+zp, 0, qmax)`` with the division done in float32
  (NumPy 2 keeps a Python-float scalar "weak", so ``flat / scale`` is an fp32
  division by ``float32(scale)``) (converter.py:54-109).
* Degenerate range (< 1e-9): all-zero codes, scale 1.0, zero point 0.0.
* Packing: INT4 low nibble = element 2j; INT2 bits [2i, 2i+1] = element 4j+i
  (converter.py:73-75,103-108), flattened row-major [rows, cols].
* Dequant: ``w = (float(q) - zp) * scale`` in float32 (n730core.cpp:65,80-82,98-101).

Group-wise extension (absent from the reference): the same formulas applied
to each group of ``g`` consecutive elements of a row, with the scale rounded
to fp16 (stored) and the codes computed against that fp16 scale, so the
stored scale is the one the dequantiser uses.  INT8 grouped keeps the
reference's symmetric form with zero point 128.  Dequant per group is the
reference per-element formula with ``float(scale16)`` and ``float(zero16)``.
"""
from __future__ import annotations

import math

import numpy as np

PREC_INT2, PREC_INT4, PREC_INT8, PREC_FP16 = 2, 4, 8, 16
# group-wise precision ids (extension): 0x40 | bits
PREC_INT2_G, PREC_INT4_G, PREC_INT8_G = 0x42, 0x44, 0x48
BITS = {PREC_INT2: 2, PREC_INT4: 4, PREC_INT8: 8, PREC_FP16: 16,
        PREC_INT2_G: 2, PREC_INT4_G: 4, PREC_INT8_G: 8}
QMAX = {2: 3, 4: 15}


# ----------------------------------------------------------------------------
# per-tensor quantisers: converter.py:41-115
# ----------------------------------------------------------------------------
def quantize_int8(weights: np.ndarray):
    flat = weights.flatten().astype(np.float32)
    abs_max = float(np.max(np.abs(flat)))
    if abs_max < 1e-9:
        return bytes(flat.size), 1.0, 0.0
    scale = abs_max / 127.0
    q = np.clip(np.round(flat / scale), -127, 127).astype(np.int8)
    return (q.astype(np.int16) + 128).astype(np.uint8).tobytes(), scale, 128.0


def _quantize_asym(weights: np.ndarray, bits: int):
    qmax = QMAX[bits]
    per_byte = 8 // bits
    flat = weights.flatten().astype(np.float32)
    w_min = float(np.min(flat))
    w_max = float(np.max(flat))
    if abs(w_max - w_min) < 1e-9:
        return bytes(math.ceil(flat.size / per_byte)), 1.0, 0.0
    scale = (w_max - w_min) / float(qmax)
    zp = int(np.clip(round(-w_min / scale), 0, qmax))
    q = np.clip(np.round(flat / scale) + zp, 0, qmax).astype(np.uint8)
    return pack_codes(q, bits).tobytes(), scale, float(zp)


def quantize_int4(weights: np.ndarray):
    return _quantize_asym(weights, 4)


def quantize_int2(weights: np.ndarray):
    return _quantize_asym(weights, 2)


def quantize_fp16(weights: np.ndarray):
    return weights.flatten().astype(np.float16).tobytes(), 1.0, 0.0


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    """Pack a flat uint8 code vector, element 0 in the least-significant bits."""
    q = np.asarray(q, dtype=np.uint8).ravel()
    if bits == 8:
        return q.copy()
    per_byte = 8 // bits
    pad = (-q.size) % per_byte
    if pad:
        q = np.concatenate([q, np.zeros(pad, np.uint8)])
    q = q.reshape(-1, per_byte)
    mask = (1 << bits) - 1
    out = np.zeros(q.shape[0], np.uint8)
    for i in range(per_byte):
        out |= (q[:, i] & mask) << (bits * i)
    return out


def unpack_codes(raw: np.ndarray, bits: int, n: int) -> np.ndarray:
    raw = np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw
    if bits == 8:
        return raw[:n].copy()
    per_byte = 8 // bits
    mask = (1 << bits) - 1
    out = np.empty(raw.size * per_byte, np.uint8)
    for i in range(per_byte):
        out[i::per_byte] = (raw >> (bits * i)) & mask
    return out[:n]


# ----------------------------------------------------------------------------
# per-tensor dequant: converter.py:344-371 == n730core.cpp:57-142
# ----------------------------------------------------------------------------
def dequant_tensor(raw: bytes, prec: int, n: int, scale: float, zp: float) -> np.ndarray:
    raw = np.frombuffer(bytes(raw), np.uint8)
    if prec == PREC_FP16:
        return raw[: 2 * n].view(np.float16).astype(np.float32)
    q = unpack_codes(raw, BITS[prec], n).astype(np.float32)
    return (q - np.float32(zp)) * np.float32(scale)


# ----------------------------------------------------------------------------
# group-wise extension
# ----------------------------------------------------------------------------
def check_group(prec: int, rows: int, cols: int, group: int):
    bits = BITS[prec]
    per16 = 128 // bits            # elements per 16 bytes of codes
    if group <= 0 or cols % group or group % per16:
        raise ValueError(f"group size {group} invalid for {bits}-bit cols={cols} "
                         f"(need cols % group == 0 and group % {per16} == 0)")


def quantize_grouped(weights: np.ndarray, bits: int, group: int):
    """Return (codes uint8 [rows, cols*bits/8], scale16 [rows, G], zero16 [rows, G])."""
    w = np.ascontiguousarray(weights, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("grouped quantisation needs a 2-D tensor")
    rows, cols = w.shape
    prec = {2: PREC_INT2_G, 4: PREC_INT4_G, 8: PREC_INT8_G}[bits]
    check_group(prec, rows, cols, group)
    G = cols // group
    wg = w.reshape(rows, G, group)
    if bits == 8:
        amax = np.abs(wg).max(axis=-1).astype(np.float64)
        degen = amax < 1e-9
        scale64 = amax / 127.0
    else:
        wmin = wg.min(axis=-1).astype(np.float64)
        wmax = wg.max(axis=-1).astype(np.float64)
        degen = np.abs(wmax - wmin) < 1e-9
        scale64 = (wmax - wmin) / float(QMAX[bits])
    with np.errstate(over="ignore"):
        s16 = scale64.astype(np.float16)
    if np.any(~np.isfinite(s16) & ~degen):
        raise ValueError("group scale overflows fp16")
    degen = degen | (s16 == 0)
    s16 = np.where(degen, np.float16(1.0), s16)
    s32 = s16.astype(np.float32)
    if bits == 8:
        q = np.clip(np.round(wg / s32[..., None]), -127, 127) + np.float32(128)
        z16 = np.full((rows, G), 128.0, np.float16)
    else:
        qmax = QMAX[bits]
        zp = np.clip(np.round(-wmin / s32.astype(np.float64)), 0, qmax).astype(np.float32)
        q = np.clip(np.round(wg / s32[..., None]) + zp[..., None], 0, qmax)
        z16 = zp.astype(np.float16)
    q = q.astype(np.uint8)
    q[degen] = 0
    z16 = np.where(degen, np.float16(0.0), z16)
    codes = pack_codes(q.reshape(-1), bits).reshape(rows, cols * bits // 8)
    return codes, s16.astype(np.float16), z16.astype(np.float16)


def dequant_grouped(codes: np.ndarray, scale16: np.ndarray, zero16: np.ndarray,
                    bits: int, rows: int, cols: int) -> np.ndarray:
    """w = (float(q) - float(z16)) * float(s16), fp32, per group along cols."""
    q = unpack_codes(np.asarray(codes, np.uint8).reshape(-1), bits, rows * cols)
    q = q.reshape(rows, cols).astype(np.float32)
    G = scale16.shape[1]
    g = cols // G
    s = np.repeat(scale16.astype(np.float32), g, axis=1)
    z = np.repeat(zero16.astype(np.float32), g, axis=1)
    return (q - z) * s


def gemv(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y = x @ W.T in fp32 (the reference's CPU matmul form, inference.py:668)."""
    return np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
