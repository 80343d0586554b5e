"""The rebuilt file core (n730core.so) against the reference's outputs and error codes."""
import ctypes as C

import numpy as np
import pytest

from conftest import GOLDEN, REPO
from n730_b200 import _lib
from n730_b200.formats import read_header


@pytest.fixture(scope="module")
def core():
    from n730_b200 import build
    build.build()
    return _lib.core()


def _read(core, h, off, n):
    out = np.zeros(n, np.float32)
    r, c, p = C.c_int32(), C.c_int32(), C.c_int32()
    rc = core.n730_read_layer(h, off, out.ctypes.data_as(C.POINTER(C.c_float)), C.byref(r),
                              C.byref(c), C.byref(p))
    return rc, out, (r.value, c.value, p.value)


def test_read_layer_bit_exact_vs_reference(core, golden):
    hdr = read_header(GOLDEN / "ref_small.n730")
    h = core.n730_open(str(GOLDEN / "ref_small.n730").encode())
    assert h > 0
    for e in hdr["seek_table"]:
        k = e["layer_name"].replace(".", "_")
        rc, out, meta = _read(core, h, e["file_offset"], e["rows"] * e["cols"])
        assert rc == 0
        assert list(meta) == list(golden[k + "__meta"])
        ref = golden[k + "__n730core"].reshape(-1)
        assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), e["layer_name"]
        assert core.n730_layer_elements(h, e["file_offset"]) == e["rows"] * e["cols"]
    core.n730_close(h)


def test_error_codes(core, tmp_path):
    bad = tmp_path / "bad.n730"
    bad.write_bytes(b"NOTN730!" + bytes(100))
    assert core.n730_open(str(bad).encode()) == -1           # BAD_MAGIC
    assert core.n730_open(str(tmp_path / "missing").encode()) == -2  # FILE
    h = core.n730_open(str(GOLDEN / "ref_small.n730").encode())
    out = np.zeros(16, np.float32)
    r = C.c_int32()
    assert core.n730_read_layer(h, 5, out.ctypes.data_as(C.POINTER(C.c_float)), C.byref(r), None, None) == -4
    assert core.n730_read_layer(0, 0, out.ctypes.data_as(C.POINTER(C.c_float)), None, None, None) == -6
    core.n730_close(h)
    # unknown precision id: patch a copy of the first block's prec byte
    data = bytearray((GOLDEN / "ref_small.n730").read_bytes())
    off = read_header(GOLDEN / "ref_small.n730")["seek_table"][0]["file_offset"]
    data[off + 8] = 3
    p = tmp_path / "prec.n730"
    p.write_bytes(bytes(data))
    h = core.n730_open(str(p).encode())
    big = np.zeros(64 * 96, np.float32)
    assert core.n730_read_layer(h, off, big.ctypes.data_as(C.POINTER(C.c_float)), None, None, None) == -5
    core.n730_close(h)


def test_grouped_blocks_read(core, tmp_path):
    from n730_b200 import converter
    from oracle import quant as oq
    rng = np.random.default_rng(5)
    layers = [("a.weight", rng.normal(0, 0.02, (32, 256)).astype(np.float32)),
              ("b.weight", rng.normal(0, 0.02, (16, 512)).astype(np.float32)),
              ("c.weight", rng.normal(0, 0.02, (8, 128)).astype(np.float32))]
    smap = {"model_id": "g", "total_params": 0, "profiles": [
        {"layer_name": "a.weight", "assigned_precision": "INT4G128"},
        {"layer_name": "b.weight", "assigned_precision": "INT2G64"},
        {"layer_name": "c.weight", "assigned_precision": "INT8PC"}]}
    path = tmp_path / "g.n730"
    converter.convert(layers, smap, path, verbose=False)
    hdr = read_header(path)
    h = core.n730_open(str(path).encode())
    for (name, w), e, (bits, g) in zip(layers, hdr["seek_table"], [(4, 128), (2, 64), (8, 128)]):
        codes, s16, z16 = oq.quantize_grouped(w, bits, g)
        ref = oq.dequant_grouped(codes, s16, z16, bits, *w.shape)
        rc, out, meta = _read(core, h, e["file_offset"], w.size)
        assert rc == 0 and meta[2] == {4: 0x44, 2: 0x42, 8: 0x48}[bits]
        assert np.array_equal(out.view(np.uint32), ref.reshape(-1).view(np.uint32)), name
        np_out = converter.read_layer(path, e["layer_idx"], hdr)
        assert np.array_equal(np_out.view(np.uint32), ref.view(np.uint32))
        hdr8 = np.zeros(8, np.int64)
        assert core.n730_read_block(h, e["file_offset"], hdr8.ctypes.data_as(C.POINTER(C.c_int64)), None, 0) == 0
        assert hdr8[5] == g
    core.n730_close(h)
