"""Pin the oracle against the reference's own outputs (golden fixtures)."""
import hashlib

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import quant as oq
from oracle.model import rope_table

from n730_b200.formats import read_header, read_block


def _bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_reference_readers_agree(golden):
    """Reference numpy read_layer and reference n730core are bit-identical (fixture sanity)."""
    hdr = read_header(GOLDEN / "ref_small.n730")
    for e in hdr["seek_table"]:
        k = e["layer_name"].replace(".", "_")
        assert _bits_equal(golden[k + "__read_layer"], golden[k + "__n730core"]), k


@pytest.mark.parametrize("use_c", [False, True])
def test_oracle_dequant_matches_reference(golden, oracle_c, use_c):
    hdr = read_header(GOLDEN / "ref_small.n730")
    for e in hdr["seek_table"]:
        b = read_block(GOLDEN / "ref_small.n730", e["file_offset"])
        n = b.rows * b.cols
        if use_c:
            out = np.zeros(n, np.float32)
            raw = np.frombuffer(b.payload, np.uint8).copy()
            rc = oracle_c.oracle_dequant_tensor(raw.ctypes.data, b.prec_id, n, b.scale,
                                                b.zero_point, out.ctypes.data)
            assert rc == 0
        else:
            out = oq.dequant_tensor(b.payload, b.prec_id, n, b.scale, b.zero_point)
        k = e["layer_name"].replace(".", "_")
        assert _bits_equal(out.reshape(b.rows, b.cols), golden[k + "__read_layer"]), e["layer_name"]


def test_oracle_quantisers_match_reference_blocks(golden):
    """Re-quantising the fixture inputs reproduces the reference's codes/scale/zp."""
    hdr = read_header(GOLDEN / "ref_small.n730")
    qf = {"INT8": oq.quantize_int8, "INT4": oq.quantize_int4, "INT2": oq.quantize_int2,
          "FP16": oq.quantize_fp16}
    for e in hdr["seek_table"]:
        k = e["layer_name"].replace(".", "_")
        w = golden[k + "__w"]
        b = read_block(GOLDEN / "ref_small.n730", e["file_offset"])
        codes, scale, zp = qf[e["precision"]](w)
        assert np.float32(scale) == np.float32(b.scale) and np.float32(zp) == np.float32(b.zero_point)
        if e["layer_name"] == "t.int4_odd":
            # the reference's np.append(uint8, 0) promotes to int64 for odd-length
            # INT4 tensors and stores 8 bytes per packed byte; the packed values agree.
            ref = np.frombuffer(b.payload, np.int64).astype(np.uint8)
            assert np.array_equal(np.frombuffer(codes, np.uint8), ref)
        else:
            assert codes == b.payload, e["layer_name"]


def test_linear4096_config_pin():
    """The single-linear workload: the oracle reproduces the reference's INT4 codes,
    scale, zero point and dequant exactly, and its GEMV."""
    g = np.load(GOLDEN / "ref_linear4096.npz")
    W = np.random.default_rng(0).normal(0, 0.02, (4096, 4096)).astype(np.float32)
    codes, scale, zp = oq.quantize_int4(W)
    assert hashlib.sha256(codes).digest() == g["codes_sha256"].tobytes()
    assert scale == float(g["scale"]) and zp == float(g["zero_point"])
    Wd = oq.dequant_tensor(codes, 4, W.size, scale, zp)
    assert _bits_equal(Wd[g["sample_idx"]], g["sample_dequant"])
    assert Wd.astype(np.float64).sum() == float(g["dequant_sum"])
    y = oq.gemv(Wd.reshape(4096, 4096), g["x"].astype(np.float32))
    assert np.max(np.abs(y - g["y"])) <= 1e-5 * np.max(np.abs(g["y"]))


def test_half_to_float_exhaustive(oracle_c):
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle_c.oracle_half_to_float(int(v)) for v in h[::7]], np.float32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))


@pytest.mark.parametrize("bits,group", [(4, 128), (4, 32), (2, 64), (8, 32), (8, 256)])
def test_grouped_roundtrip_and_c(bits, group, oracle_c):
    rng = np.random.default_rng(bits * 1000 + group)
    rows, cols = 24, 512
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    w[3, :group] = 0.0                      # a degenerate group
    codes, s16, z16 = oq.quantize_grouped(w, bits, group)
    d = oq.dequant_grouped(codes, s16, z16, bits, rows, cols)
    assert np.all(d[3, :group] == 0)
    qmax = {2: 3, 4: 15, 8: 254}[bits]
    step = np.repeat(s16.astype(np.float32), group, axis=1)
    # quantisation error is at most about one step (half a step plus fp16 scale rounding)
    assert np.all(np.abs(d - w) <= step * 0.51 + 1e-6 * qmax)
    out = np.zeros(rows * cols, np.float32)
    rc = oracle_c.oracle_dequant_grouped(codes.ctypes.data, s16.ctypes.data, z16.ctypes.data,
                                         bits, rows, cols, group, out.ctypes.data)
    assert rc == 0 and _bits_equal(out.reshape(rows, cols), d)


def test_grouped_dequant_is_reference_formula_per_group():
    """With one group per tensor and the tensor's own (scale, zero), the grouped
    formula is the reference per-tensor dequant, bit for bit."""
    g = np.load(GOLDEN / "ref_small.npz")
    w = g["t_int4__w"]
    codes, scale, zp = oq.quantize_int4(w)
    ref = g["t_int4__read_layer"]
    q = oq.unpack_codes(np.frombuffer(codes, np.uint8), 4, w.size).astype(np.float32)
    per_group = (q - np.float32(zp)) * np.float32(scale)
    assert _bits_equal(per_group.reshape(w.shape), ref)


def test_rope_table_numpy_vs_c(oracle_c):
    cos, sin = rope_table(512, 128, 1e6)
    cc = np.zeros_like(cos)
    ss = np.zeros_like(sin)
    oracle_c.oracle_rope_table(512, 128, 1e6, cc.ctypes.data, ss.ctypes.data)
    # numpy float32 power differs from glibc powf by an ulp; the error grows with pos
    assert np.max(np.abs(cos - cc)) < 1e-4 and np.max(np.abs(sin - ss)) < 1e-4
