"""The ``.n730`` packed-weight format: constants, block headers, raw block access.

File layout (``src-code/converter.py:1-21``)::

    [MAGIC 8B "N730\\0\\1\\0\\0"][>I version][>I header_size][JSON header][pad to 4 KiB]
    [block 0][pad to 4 KiB][block 1][pad to 4 KiB] ...

Block = 29-byte big-endian header ``>4sIBIIffi`` (magic ``LYR\\0``, layer index,
precision id, rows, cols, scale f32, zero point f32, data_size) followed by
``data_size`` payload bytes (``converter.py:149-159``, C mirror
``src-code/cpp/n730core.cpp:144-155``).

Per-tensor precision ids 2/4/8/16 are the reference's, byte for byte.  The
group-wise extension adds ids ``0x42/0x44/0x48`` (INT2/INT4/INT8 grouped).
Their header scale/zero are 1.0/0.0 and their payload is::

    codes  (same packing as per-tensor: flattened row-major [rows, cols],
            element 0 in the least-significant bits)
    scale  fp16 little-endian [rows, cols/group]
    zero   fp16 little-endian [rows, cols/group]

``data_size`` covers all three, so the group size follows from the block
alone: ``group = cols / ((data_size - code_bytes) / (4 * rows))``.  The seek
table entry also records ``"group_size"``.  A reader that only knows the
reference ids rejects the new ids (n730core returns BAD_PREC -5; the
reference ``read_layer`` raises "Unknown precision").
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"N730\x00\x01\x00\x00"
LAYER_MAGIC = b"LYR\x00"
FORMAT_VERSION = 1
PAGE_SIZE = 4096
BLOCK_HEADER = ">4sIBIIffi"
BLOCK_HEADER_SIZE = struct.calcsize(BLOCK_HEADER)  # 29

PREC_INT2, PREC_INT4, PREC_INT8, PREC_FP16 = 2, 4, 8, 16
PREC_INT2_G, PREC_INT4_G, PREC_INT8_G = 0x42, 0x44, 0x48

PRECISION_ID = {"INT2": 2, "INT4": 4, "INT8": 8, "FP16": 16,
                "INT2G": PREC_INT2_G, "INT4G": PREC_INT4_G, "INT8G": PREC_INT8_G}
PRECISION_NAME = {v: k for k, v in PRECISION_ID.items()}
PRECISION_BITS = {"INT2": 2, "INT4": 4, "INT8": 8, "FP16": 16,
                  "INT2G": 2, "INT4G": 4, "INT8G": 8}
GROUPED = {PREC_INT2_G, PREC_INT4_G, PREC_INT8_G}


def prec_bits(prec_id: int) -> int:
    return PRECISION_BITS[PRECISION_NAME[prec_id]]


def code_bytes(prec_id: int, n_elements: int) -> int:
    bits = prec_bits(prec_id)
    return (n_elements * bits + 7) // 8


def min_group_multiple(bits: int) -> int:
    """Elements per 16 bytes of codes: the group size must be a multiple of this."""
    return 128 // bits


def pad_to_page(data: bytes) -> bytes:
    rem = len(data) % PAGE_SIZE
    return data if rem == 0 else data + bytes(PAGE_SIZE - rem)


@dataclass
class RawBlock:
    """One tensor block as stored: codes plus its dequant parameters."""
    layer_idx: int
    prec_id: int
    rows: int
    cols: int
    scale: float          # per-tensor scale (1.0 for grouped)
    zero_point: float     # per-tensor zero point (0.0 for grouped)
    payload: bytes        # data_size bytes
    group_size: int = 0   # 0 for per-tensor formats

    @property
    def n_elements(self) -> int:
        return self.rows * self.cols

    @property
    def grouped(self) -> bool:
        return self.prec_id in GROUPED

    @property
    def codes(self) -> np.ndarray:
        n = code_bytes(self.prec_id, self.n_elements)
        return np.frombuffer(self.payload, np.uint8, count=n)

    @property
    def scales16(self) -> np.ndarray:
        n = code_bytes(self.prec_id, self.n_elements)
        g = self.rows * (self.cols // self.group_size)
        return np.frombuffer(self.payload, np.float16, count=g, offset=n).reshape(self.rows, -1)

    @property
    def zeros16(self) -> np.ndarray:
        n = code_bytes(self.prec_id, self.n_elements)
        g = self.rows * (self.cols // self.group_size)
        return np.frombuffer(self.payload, np.float16, count=g, offset=n + 2 * g).reshape(self.rows, -1)


def group_size_from_block(prec_id: int, rows: int, cols: int, data_size: int) -> int:
    """Derive the group size of a grouped block from its sizes; raise if inconsistent."""
    n_codes = code_bytes(prec_id, rows * cols)
    extra = data_size - n_codes
    if rows <= 0 or extra <= 0 or extra % (4 * rows):
        raise ValueError(f"grouped block sizes inconsistent (rows={rows} cols={cols} "
                         f"data_size={data_size})")
    G = extra // (4 * rows)
    if cols % G:
        raise ValueError(f"grouped block: {G} groups do not divide cols={cols}")
    return cols // G


def read_header(path) -> dict:
    with open(path, "rb") as f:
        magic = f.read(8)
        if magic != MAGIC:
            raise ValueError(f"Not a valid .n730 file (bad magic: {magic!r})")
        _version, header_size = struct.unpack(">II", f.read(8))
        return json.loads(f.read(header_size))


def read_block(path, file_offset: int, f=None) -> RawBlock:
    """Read one block's header and payload at an absolute offset (no dequant)."""
    own = f is None
    if own:
        f = open(path, "rb")
    try:
        f.seek(file_offset)
        magic = f.read(4)
        if magic != LAYER_MAGIC:
            raise ValueError(f"Bad layer magic at offset {file_offset}")
        idx, prec, rows, cols, scale, zp, dsz = struct.unpack(
            BLOCK_HEADER[0] + BLOCK_HEADER[3:], f.read(BLOCK_HEADER_SIZE - 4))
        payload = f.read(dsz)
        if len(payload) != dsz:
            raise ValueError(f"short read at offset {file_offset}")
    finally:
        if own:
            f.close()
    if prec not in PRECISION_NAME:
        raise ValueError(f"Unknown precision id: {prec}")
    g = group_size_from_block(prec, rows, cols, dsz) if prec in GROUPED else 0
    return RawBlock(idx, prec, rows, cols, scale, zp, payload, g)


def pack_block(layer_idx: int, prec_id: int, rows: int, cols: int, scale: float,
               zero_point: float, payload: bytes) -> bytes:
    header = struct.pack(BLOCK_HEADER, LAYER_MAGIC, layer_idx, prec_id, rows, cols,
                         scale, zero_point, len(payload))
    return pad_to_page(header + payload)
