"""Converter to the ``.n730`` packed-weight format (reference API, plus group-wise blocks).

Mirrors ``src-code/converter.py``: the same module-level names
(``quantize_int8/int4/int2/fp16``, ``QUANTIZERS``, ``pad_to_page``,
``serialize_layer``, ``convert``, ``inspect_n730``, ``read_layer``,
``generate_synthetic_weights``) with the same arguments and outputs.  For
per-tensor precisions the written file is byte-identical to the reference's.

Extension (absent from the reference): a sensitivity-map profile may assign a
group-wise precision, either ``{"assigned_precision": "INT4G", "group_size": 128}``
or the shorthands ``"INT4G128"``, ``"INT2G64"``, ``"INT8G32"`` and ``"INT8PC"``
(INT8 per output channel, i.e. one group per row).  Grouped blocks carry fp16
scale and zero per group (layout in ``n730_b200.formats``); the quantiser
applies the reference's per-tensor formula to each group with the fp16 scale.

Unlike the reference, ``convert`` spools blocks to a temporary file instead of
holding them all in RAM (a 72B INT4 model is ~36 GB of blocks); the output
bytes are unchanged.  ``N730Writer`` writes very large files in one streaming
pass with a reserved header area.
"""
from __future__ import annotations

import argparse
import json
import math
import re
import shutil
import struct
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

from .formats import (BLOCK_HEADER, FORMAT_VERSION, GROUPED, LAYER_MAGIC, MAGIC, PAGE_SIZE,
                      PRECISION_BITS, PRECISION_ID, PREC_INT2_G, PREC_INT4_G, PREC_INT8_G,
                      min_group_multiple, pad_to_page, read_block, read_header)

__all__ = ["MAGIC", "LAYER_MAGIC", "FORMAT_VERSION", "PAGE_SIZE", "PRECISION_BITS",
           "PRECISION_ID", "quantize_int8", "quantize_int4", "quantize_int2", "quantize_fp16",
           "quantize_grouped", "QUANTIZERS", "pad_to_page", "serialize_layer", "convert",
           "inspect_n730", "read_layer", "generate_synthetic_weights", "N730Writer",
           "parse_precision"]


# ---------------------------------------------------------------------------
# per-tensor quantisers (converter.py:41-115)
# ---------------------------------------------------------------------------
def quantize_int8(weights: np.ndarray):
    """Symmetric INT8 stored as uint8 with offset 128 (converter.py:41-51)."""
    flat = weights.flatten().astype(np.float32)
    abs_max = float(np.max(np.abs(flat)))
    if abs_max < 1e-9:
        return bytes(flat.size), 1.0, 0.0
    scale = abs_max / 127.0
    q = np.clip(np.round(flat / scale), -127, 127).astype(np.int8)
    return (q.astype(np.int16) + 128).astype(np.uint8).tobytes(), scale, 128.0


def _pack(q: np.ndarray, bits: int) -> bytes:
    per = 8 // bits
    pad = (-q.size) % per
    if pad:
        q = np.append(q, np.zeros(pad, np.uint8))
    q = q.reshape(-1, per)
    out = np.zeros(q.shape[0], np.uint8)
    for i in range(per):
        out |= (q[:, i] & ((1 << bits) - 1)) << (bits * i)
    return out.tobytes()


def _quantize_asym(weights: np.ndarray, bits: int):
    qmax = (1 << bits) - 1
    flat = weights.flatten().astype(np.float32)
    w_min, w_max = float(np.min(flat)), float(np.max(flat))
    if abs(w_max - w_min) < 1e-9:
        return bytes(math.ceil(flat.size / (8 // bits))), 1.0, 0.0
    scale = (w_max - w_min) / float(qmax)
    zp = int(np.clip(round(-w_min / scale), 0, qmax))
    q = np.clip(np.round(flat / scale) + zp, 0, qmax).astype(np.uint8)
    return _pack(q, bits), scale, float(zp)


def quantize_int4(weights: np.ndarray):
    """Asymmetric INT4, two codes per byte, low nibble first (converter.py:54-76)."""
    return _quantize_asym(weights, 4)


def quantize_int2(weights: np.ndarray):
    """Asymmetric INT2, four codes per byte, LSB first (converter.py:79-109)."""
    return _quantize_asym(weights, 2)


def quantize_fp16(weights: np.ndarray):
    return weights.flatten().astype(np.float16).tobytes(), 1.0, 0.0


QUANTIZERS = {"INT2": quantize_int2, "INT4": quantize_int4,
              "INT8": quantize_int8, "FP16": quantize_fp16}


# ---------------------------------------------------------------------------
# group-wise quantiser (extension)
# ---------------------------------------------------------------------------
def quantize_grouped(weights: np.ndarray, bits: int, group: int):
    """Quantise [rows, cols] per group of ``group`` elements along cols.

    INT4/INT2: ``scale = (max-min)/qmax`` (float64) rounded to fp16 ``s``;
    ``zp = clip(round(-min/s), 0, qmax)``; ``q = clip(round(w/s) + zp, 0, qmax)``
    with an fp32 division.  INT8: ``s = fp16(absmax/127)``,
    ``q = clip(round(w/s), -127, 127) + 128``, zero 128.  Groups with range
    (or absmax) below 1e-9, or whose fp16 scale underflows to 0, get codes 0,
    scale 1, zero 0 (the reference's degenerate rule).
    Returns ``(codes uint8 [rows*cols*bits/8], scale fp16 [rows, G], zero fp16 [rows, G])``.
    """
    w = np.ascontiguousarray(weights, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("grouped precision needs a 2-D tensor")
    rows, cols = w.shape
    if group <= 0 or cols % group or group % min_group_multiple(bits):
        raise ValueError(f"group size {group} invalid for INT{bits} with cols={cols}")
    G = cols // group
    wg = w.reshape(rows, G, group)
    if bits == 8:
        amax = np.abs(wg).max(axis=-1).astype(np.float64)
        degen = amax < 1e-9
        scale = amax / 127.0
    else:
        wmin = wg.min(axis=-1).astype(np.float64)
        wmax = wg.max(axis=-1).astype(np.float64)
        degen = np.abs(wmax - wmin) < 1e-9
        scale = (wmax - wmin) / float((1 << bits) - 1)
    with np.errstate(over="ignore"):
        s16 = scale.astype(np.float16)
    if np.any(~np.isfinite(s16) & ~degen):
        raise ValueError("group scale overflows fp16")
    degen |= s16 == 0
    s16 = np.where(degen, np.float16(1.0), s16).astype(np.float16)
    s32 = s16.astype(np.float32)[..., None]
    if bits == 8:
        q = np.clip(np.round(wg / s32), -127, 127) + np.float32(128)
        z16 = np.full((rows, G), 128.0, np.float16)
    else:
        qmax = (1 << bits) - 1
        zp = np.clip(np.round(-wmin / s32[..., 0].astype(np.float64)), 0, qmax).astype(np.float32)
        q = np.clip(np.round(wg / s32) + zp[..., None], 0, qmax)
        z16 = zp.astype(np.float16)
    q = q.astype(np.uint8)
    q[degen] = 0
    z16 = np.where(degen, np.float16(0.0), z16).astype(np.float16)
    codes = np.frombuffer(_pack(q.reshape(-1), bits), np.uint8) if bits != 8 else q.reshape(-1)
    return codes, s16, z16


_SHORT = re.compile(r"^(INT[248])(?:G(\d+)|(PC))$")


def parse_precision(name: str, profile: dict | None = None, cols: int | None = None):
    """Return ``(precision_name, group_size)``; group 0 for per-tensor precisions."""
    profile = profile or {}
    if name in ("INT2", "INT4", "INT8", "FP16"):
        return name, 0
    if name in ("INT2G", "INT4G", "INT8G"):
        g = int(profile.get("group_size", 0))
        if g <= 0:
            raise ValueError(f"{name} needs a group_size")
        return name, g
    m = _SHORT.match(name)
    if not m:
        raise ValueError(f"Unknown precision: {name}")
    base = m.group(1) + "G"
    if m.group(3):
        if cols is None:
            raise ValueError("INT8PC needs the tensor's column count")
        return base, int(cols)
    return base, int(m.group(2))


# ---------------------------------------------------------------------------
# blocks and files
# ---------------------------------------------------------------------------
def serialize_layer(layer_idx: int, precision: str, weights: np.ndarray, layer_name: str,
                    group_size: int = 0):
    """One padded block plus its seek-table metadata (converter.py:133-177)."""
    shape = weights.shape
    rows = shape[0]
    cols = shape[1] if len(shape) > 1 else 1
    if precision in ("INT2G", "INT4G", "INT8G"):
        bits = PRECISION_BITS[precision]
        codes, s16, z16 = quantize_grouped(weights.reshape(rows, cols), bits, group_size)
        payload = codes.tobytes() + s16.astype("<f2").tobytes() + z16.astype("<f2").tobytes()
        scale, zero_point = 1.0, 0.0
    else:
        payload, scale, zero_point = QUANTIZERS[precision](weights)
    header = struct.pack(BLOCK_HEADER, LAYER_MAGIC, layer_idx, PRECISION_ID[precision],
                         rows, cols, scale, zero_point, len(payload))
    block = pad_to_page(header + payload)
    meta = {"layer_idx": layer_idx, "layer_name": layer_name, "precision": precision,
            "rows": rows, "cols": cols, "scale": scale, "zero_point": zero_point,
            "original_bytes": weights.size * 4, "stored_bytes": len(payload),
            "block_bytes": len(block)}
    if group_size:
        meta["group_size"] = group_size
    return block, meta


def _choose(name, weights, lookup):
    if weights.ndim == 1:
        return "FP16", 0
    prof = lookup.get(name)
    if prof is None:
        return "INT4", 0
    cols = weights.shape[1] if weights.ndim > 1 else 1
    return parse_precision(prof["assigned_precision"], prof, cols)


def convert(weight_layers, sensitivity_map: dict, output_path: Path, verbose: bool = True):
    """Write a ``.n730`` file (converter.py:179-281); same bytes as the reference.

    ``weight_layers`` is any iterable of ``(name, np.ndarray)``; blocks are
    spooled to a temporary file so only one tensor is in memory at a time.
    """
    output_path = Path(output_path)
    lookup = {p["layer_name"]: p for p in sensitivity_map["profiles"]}
    seek_table = []
    total_orig = total_stored = 0
    t0 = time.time()
    offset = 0
    with tempfile.TemporaryFile(dir=output_path.parent if output_path.parent.exists() else None) as spool:
        for idx, (name, weights) in enumerate(weight_layers):
            precision, group = _choose(name, np.asarray(weights), lookup)
            block, meta = serialize_layer(idx, precision, np.asarray(weights), name, group)
            meta["file_offset"] = offset
            offset += len(block)
            spool.write(block)
            seek_table.append(meta)
            total_orig += meta["original_bytes"]
            total_stored += meta["stored_bytes"]
            if verbose:
                print(f"  {idx + 1:>4}  [{precision:<5}]  {name[:60]}")
        total = len(seek_table)
        file_header = {
            "format": "N730", "version": FORMAT_VERSION, "project": "N730",
            "model_id": sensitivity_map["model_id"], "total_layers": total,
            "total_params": sensitivity_map["total_params"],
            "original_mb": round(total_orig / (1024 ** 2), 2),
            "stored_mb": round(total_stored / (1024 ** 2), 2),
            "compression": round(total_orig / max(total_stored, 1), 2),
            "page_size": PAGE_SIZE, "seek_table": seek_table,
        }
        # two-pass header exactly as converter.py:246-256
        hj = json.dumps(file_header, indent=2).encode("utf-8")
        data_start = len(pad_to_page(MAGIC + struct.pack(">II", FORMAT_VERSION, len(hj)) + hj))
        for e in seek_table:
            e["file_offset"] += data_start
        hj = json.dumps(file_header, indent=2).encode("utf-8")
        pre = pad_to_page(MAGIC + struct.pack(">II", FORMAT_VERSION, len(hj)) + hj)
        if len(pre) != data_start:
            raise RuntimeError("header grew across a page boundary; offsets would be wrong")
        spool.seek(0)
        with open(output_path, "wb") as f:
            f.write(pre)
            shutil.copyfileobj(spool, f, 16 << 20)
    if verbose:
        print(f"  converted {total} tensors in {time.time() - t0:.1f}s -> {output_path}")
    return file_header


class N730Writer:
    """Single-pass streaming writer for very large models.

    The caller declares the number of tensors up front; a header area of
    ``reserve_bytes`` (page-rounded) is reserved, blocks are written as they
    are added, and the JSON header is written into the reserved area on
    ``close()``.  Offsets are absolute, so the reference readers accept the
    file (they read ``header_size`` bytes of JSON and seek by offset).
    """

    def __init__(self, path, model_id: str, total_params: int, n_tensors: int,
                 reserve_bytes: int | None = None):
        self.path = Path(path)
        self.model_id, self.total_params = model_id, total_params
        reserve = reserve_bytes or (16 + 4096 + 512 * n_tensors)
        self.data_start = ((reserve + PAGE_SIZE - 1) // PAGE_SIZE) * PAGE_SIZE
        self.f = open(self.path, "wb")
        self.f.write(bytes(self.data_start))
        self.offset = self.data_start
        self.seek_table = []
        self.total_orig = self.total_stored = 0

    def add(self, name: str, weights: np.ndarray, precision: str, group_size: int = 0):
        block, meta = serialize_layer(len(self.seek_table), precision, weights, name, group_size)
        meta["file_offset"] = self.offset
        self.f.write(block)
        self.offset += len(block)
        self.seek_table.append(meta)
        self.total_orig += meta["original_bytes"]
        self.total_stored += meta["stored_bytes"]
        return meta

    def close(self):
        hdr = {"format": "N730", "version": FORMAT_VERSION, "project": "N730",
               "model_id": self.model_id, "total_layers": len(self.seek_table),
               "total_params": self.total_params,
               "original_mb": round(self.total_orig / (1024 ** 2), 2),
               "stored_mb": round(self.total_stored / (1024 ** 2), 2),
               "compression": round(self.total_orig / max(self.total_stored, 1), 2),
               "page_size": PAGE_SIZE, "seek_table": self.seek_table}
        hj = json.dumps(hdr, indent=2).encode("utf-8")
        pre = MAGIC + struct.pack(">II", FORMAT_VERSION, len(hj)) + hj
        if len(pre) > self.data_start:
            self.f.close()
            raise ValueError(f"header ({len(pre)} B) exceeds the reserved {self.data_start} B")
        self.f.seek(0)
        self.f.write(pre)
        self.f.close()
        return hdr


def inspect_n730(path: Path):
    h = read_header(path)
    print(f"  Model {h['model_id']}  tensors {h['total_layers']}  "
          f"stored {h['stored_mb']} MB  compression {h['compression']}x")
    for e in h["seek_table"][:5]:
        g = f" g{e['group_size']}" if e.get("group_size") else ""
        print(f"    [{e['precision']:<5}{g}] offset={e['file_offset']:>12,}  "
              f"{e['rows']}x{e['cols']}  {e['layer_name']}")
    return h


def _unpack(raw: np.ndarray, bits: int, n: int) -> np.ndarray:
    if bits == 8:
        return raw[:n]
    per = 8 // bits
    out = np.empty(raw.size * per, np.uint8)
    for i in range(per):
        out[i::per] = (raw >> (bits * i)) & ((1 << bits) - 1)
    return out[:n]


def read_layer(path: Path, layer_idx: int, header: dict = None) -> np.ndarray:
    """Read and dequantise one tensor to fp32 [rows, cols] (converter.py:316-376).

    Per-tensor: ``(float(q) - zp) * scale``.  Grouped: the same per element
    with the group's fp16 scale and zero.  This is the host-side utility; the
    device path never dequantises to fp32 memory.
    """
    if header is None:
        header = read_header(path)
    e = header["seek_table"][layer_idx]
    b = read_block(path, e["file_offset"])
    n = b.rows * b.cols
    if e["precision"] == "FP16":
        w = np.frombuffer(b.payload, np.float16).astype(np.float32)
    elif e["precision"] in ("INT2", "INT4", "INT8"):
        q = _unpack(np.frombuffer(b.payload, np.uint8), PRECISION_BITS[e["precision"]], n)
        w = (q.astype(np.float32) - b.zero_point) * b.scale
    elif b.grouped:
        q = _unpack(b.codes, PRECISION_BITS[e["precision"]], n).reshape(b.rows, b.cols)
        g = b.group_size
        s = np.repeat(b.scales16.astype(np.float32), g, axis=1)
        z = np.repeat(b.zeros16.astype(np.float32), g, axis=1)
        w = (q.astype(np.float32) - z) * s
    else:
        raise ValueError(f"Unknown precision: {e['precision']}")
    return w.reshape(b.rows, b.cols)


def generate_synthetic_weights(sensitivity_map: dict) -> list:
    """Capped synthetic shapes from a sensitivity map (converter.py:378-389)."""
    layers = []
    rng = np.random.default_rng(42)
    for profile in sensitivity_map["profiles"]:
        params = min(profile["param_count"], 1_000_000)
        cols = min(1024, params)
        rows = max(1, params // cols)
        std = profile.get("weight_std") or 0.02
        layers.append((profile["layer_name"], rng.normal(0, std, (rows, cols)).astype(np.float32)))
    return layers


def main(argv=None):
    ap = argparse.ArgumentParser(description="N730 format converter")
    ap.add_argument("--synthetic", action="store_true")
    ap.add_argument("--sensitivity", default="sensitivity_map.json")
    ap.add_argument("--output", default="model.n730")
    ap.add_argument("--inspect")
    ap.add_argument("--read-layer", type=int)
    ap.add_argument("--quiet", action="store_true")
    args = ap.parse_args(argv)
    if args.inspect:
        inspect_n730(Path(args.inspect))
        if args.read_layer is not None:
            w = read_layer(Path(args.inspect), args.read_layer)
            print(f"  Shape {w.shape}  mean {w.mean():.6f}  std {w.std():.6f}  "
                  f"min {w.min():.6f}  max {w.max():.6f}")
        return 0
    with open(args.sensitivity) as f:
        smap = json.load(f)
    layers = generate_synthetic_weights(smap)
    convert(layers, smap, Path(args.output), verbose=not args.quiet)
    return 0


if __name__ == "__main__":
    sys.exit(main())
