"""GPU parity of the packed-weight kernels against the oracle, through the C ABI.

Bars: dequantised weights bit-exact; GPU quantiser codes/scales/zeros
bit-exact; GEMV outputs within max|y - y_ref| / max|y_ref| <= 1e-4 (fp32
accumulation in a different order; the decoder's end-to-end bar is 1e-2).
"""
import ctypes as C
import hashlib

import numpy as np
import pytest

from conftest import GOLDEN
from gpu_util import dev, ptr, qweight_from_oracle, rel_err, torch
from oracle import quant as oq
from n730_b200 import _lib
from n730_b200.formats import read_block, read_header

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def lib():
    return _lib.cuda()


def _dequant(lib, qw, rows, cols):
    out = torch().zeros(rows, cols, dtype=torch().float32, device="cuda")
    _lib.check(lib.n730_dequant_to_f32(qw, ptr(out), None), "dequant")
    torch().cuda.synchronize()
    return out.cpu().numpy()


def test_dequant_bit_exact_reference_blocks(lib, golden):
    hdr = read_header(GOLDEN / "ref_small.n730")
    for e in hdr["seek_table"]:
        b = read_block(GOLDEN / "ref_small.n730", e["file_offset"])
        if e["layer_name"] == "t.int4_odd":
            continue  # the reference wrote int64-expanded codes for this tensor (odd INT4)
        qw = qweight_from_oracle(b.prec_id, b.rows, b.cols, b.payload, b.scale, b.zero_point)
        got = _dequant(lib, qw, b.rows, b.cols)
        ref = golden[e["layer_name"].replace(".", "_") + "__read_layer"]
        assert np.array_equal(got.view(np.uint32), ref.reshape(b.rows, b.cols).view(np.uint32)), e["layer_name"]
        lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("bits,group,rows,cols", [(4, 128, 40, 512), (2, 64, 24, 640), (8, 32, 17, 96),
                                                  (8, 256, 8, 256), (4, 32, 3, 32)])
def test_dequant_bit_exact_grouped(lib, bits, group, rows, cols):
    rng = np.random.default_rng(bits * 7 + rows)
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    codes, s16, z16 = oq.quantize_grouped(w, bits, group)
    qw = qweight_from_oracle(0x40 | bits, rows, cols, codes, s16=s16, z16=z16, group=group)
    got = _dequant(lib, qw, rows, cols)
    ref = oq.dequant_grouped(codes, s16, z16, bits, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("bits,group", [(4, 128), (2, 64), (8, 32), (8, 512)])
def test_gpu_quantiser_bit_exact(lib, bits, group):
    rng = np.random.default_rng(100 + bits)
    rows, cols = 64, 1024
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    w[5, :group] = 0.3           # degenerate group (constant)
    w[6, :group] *= 1e-3         # small range
    codes, s16, z16 = oq.quantize_grouped(w, bits, group)
    t = torch()
    dw = dev(w)
    dc = t.zeros(rows * cols * bits // 8, dtype=t.uint8, device="cuda")
    ds = t.zeros(rows, cols // group, dtype=t.float16, device="cuda")
    dz = t.zeros_like(ds)
    _lib.check(lib.n730_quantize_grouped(ptr(dw), rows, cols, bits, group, ptr(dc), ptr(ds), ptr(dz), None), "quantize")
    t.cuda.synchronize()
    assert np.array_equal(dc.cpu().numpy(), codes.reshape(-1))
    assert np.array_equal(ds.cpu().numpy().view(np.uint16), s16.view(np.uint16))
    assert np.array_equal(dz.cpu().numpy().view(np.uint16), z16.view(np.uint16))


def _qlinear(lib, qw, x, n_out, bias=None, resid=None, norm=None, eps=1e-6, swiglu=0):
    t = torch()
    dx = dev(x.astype(np.float32))
    B, K = x.shape
    dy = t.zeros(B, n_out, dtype=t.float32, device="cuda")
    db = dev(bias) if bias is not None else None
    dr = dev(resid) if resid is not None else None
    dn = dev(norm) if norm is not None else None
    _lib.check(lib.n730_qlinear(qw, ptr(dx), K, B, ptr(dy), n_out, ptr(db), ptr(dr), n_out if resid is not None else 0,
                                ptr(dn), eps, swiglu, None), "qlinear")
    t.cuda.synchronize()
    return dy.cpu().numpy()


def test_linear4096_config(lib):
    """The single-linear workload: W[4096x4096] ~ N(0,0.02) seed 0, reference per-tensor
    INT4 packing; y = x . dequant(W)^T checked against the reference's golden y."""
    g = np.load(GOLDEN / "ref_linear4096.npz")
    W = np.random.default_rng(0).normal(0, 0.02, (4096, 4096)).astype(np.float32)
    codes, scale, zp = oq.quantize_int4(W)
    assert hashlib.sha256(codes).digest() == g["codes_sha256"].tobytes()
    qw = qweight_from_oracle(4, 4096, 4096, codes, scale, zp)
    y = _qlinear(lib, qw, g["x"].astype(np.float32), 4096)
    assert rel_err(y, g["y"]) <= TOL
    lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("bits,group,rows,cols,batch", [
    (4, 128, 4096, 4096, 1), (4, 128, 512, 3584, 1), (4, 128, 3584, 18944, 1), (4, 128, 258, 896, 3),
    (2, 64, 1000, 4864, 1), (2, 64, 96, 18944, 2), (8, 32, 896, 896, 1), (8, 896, 130, 896, 5),
    (4, 32, 7, 64, 4), (8, 16, 33, 48, 2)])
def test_qlinear_grouped(lib, bits, group, rows, cols, batch):
    rng = np.random.default_rng(rows + cols + bits)
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    codes, s16, z16 = oq.quantize_grouped(w, bits, group)
    wd = oq.dequant_grouped(codes, s16, z16, bits, rows, cols)
    qw = qweight_from_oracle(0x40 | bits, rows, cols, codes, s16=s16, z16=z16, group=group)
    y = _qlinear(lib, qw, x, rows)
    assert rel_err(y, oq.gemv(wd, x)) <= TOL
    lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("prec,rows,cols,batch", [(8, 896, 896, 1), (8, 128, 4864, 2), (4, 64, 96, 1),
                                                  (2, 48, 80, 3), (16, 256, 896, 1), (16, 40, 72, 2),
                                                  (4, 33, 70, 1), (8, 5, 13, 2)])
def test_qlinear_per_tensor(lib, prec, rows, cols, batch):
    rng = np.random.default_rng(prec * 31 + rows)
    w = rng.normal(0, 0.05, (rows, cols)).astype(np.float32)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    q = {2: oq.quantize_int2, 4: oq.quantize_int4, 8: oq.quantize_int8, 16: oq.quantize_fp16}[prec]
    codes, scale, zp = q(w)
    wd = oq.dequant_tensor(codes, prec, w.size, scale, zp).reshape(rows, cols)
    qw = qweight_from_oracle(prec, rows, cols, codes, scale, zp)
    y = _qlinear(lib, qw, x, rows)
    assert rel_err(y, oq.gemv(wd, x)) <= TOL
    lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("B", [1, 2, 3, 4, 7])
def test_qlinear_epilogues(lib, B):
    """Fused RMSNorm prologue, bias, residual, and SwiGLU on interleaved gate/up rows."""
    from oracle.model import rms_norm, swiglu
    rng = np.random.default_rng(9 + B)
    K, N = 896, 640
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, K).astype(np.float32)
    bias = rng.normal(0, 0.02, N).astype(np.float32)
    res = rng.normal(0, 1, (B, N)).astype(np.float32)
    codes, s16, z16 = oq.quantize_grouped(w, 4, 128)
    wd = oq.dequant_grouped(codes, s16, z16, 4, N, K)
    qw = qweight_from_oracle(0x44, N, K, codes, s16=s16, z16=z16, group=128)
    xn = rms_norm(x, nw, 1e-6)
    y = _qlinear(lib, qw, x, N, bias=bias, resid=res, norm=nw)
    assert rel_err(y, res + xn @ wd.T + bias) <= TOL
    # swiglu: rows 2i = gate_i, 2i+1 = up_i
    y2 = _qlinear(lib, qw, x, N // 2, bias=bias, norm=nw, swiglu=1)
    full = xn @ wd.T + bias
    ref = swiglu(full[:, 0::2], full[:, 1::2])
    assert rel_err(y2, ref) <= TOL
    lib.n730_qweight_destroy(qw)


def test_bad_group_rejected(lib):
    codes = np.zeros(64 * 100 // 2, np.uint8)
    s = np.ones((64, 4), np.float16)
    out = C.c_void_p()
    rc = lib.n730_qweight_create(0x44, 64, 100, 25, 1.0, 0.0, codes.ctypes.data_as(C.c_void_p),
                                 s.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p), 0, None,
                                 C.byref(out))
    assert rc == -13 and b"group" in lib.n730_last_error()


@pytest.mark.parametrize("rows,cols,group,batch", [(4096, 4096, 128, 1), (4608, 3584, 128, 1), (3584, 18944, 128, 1),
                                                   (40, 256, 64, 3), (37, 512, 128, 9), (300, 1024, 256, 16),
                                                   (64, 3584, 128, 20)])
def test_qlinear_tensor_core_layout(lib, rows, cols, group, batch):
    """INT4 group-wise weights in the tensor-core fragment layout: dequant stays
    bit-exact; the GEMV (x rounded to fp16, fp32 accumulation) is within 2e-3."""
    rng = np.random.default_rng(rows * 7 + batch)
    w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    codes, s16, z16 = oq.quantize_grouped(w, 4, group)
    wd = oq.dequant_grouped(codes, s16, z16, 4, rows, cols)
    qw = qweight_from_oracle(0x44, rows, cols, codes, s16=s16, z16=z16, group=group)
    _lib.check(lib.n730_qweight_set_layout(qw, 1, None), "set_layout")
    assert np.array_equal(_dequant(lib, qw, rows, cols).view(np.uint32), wd.view(np.uint32))
    y = _qlinear(lib, qw, x, rows)
    assert rel_err(y, oq.gemv(wd, x)) <= 2e-3
    lib.n730_qweight_destroy(qw)


@pytest.mark.parametrize("B", [1, 2, 5])
def test_tensor_core_epilogues(lib, B):
    from oracle.model import rms_norm, swiglu
    rng = np.random.default_rng(90 + B)
    K, N = 1024, 640
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    x = rng.normal(0, 1, (B, K)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, K).astype(np.float32)
    bias = rng.normal(0, 0.02, N).astype(np.float32)
    res = rng.normal(0, 1, (B, N)).astype(np.float32)
    codes, s16, z16 = oq.quantize_grouped(w, 4, 128)
    wd = oq.dequant_grouped(codes, s16, z16, 4, N, K)
    qw = qweight_from_oracle(0x44, N, K, codes, s16=s16, z16=z16, group=128)
    _lib.check(lib.n730_qweight_set_layout(qw, 1, None), "set_layout")
    xn = rms_norm(x, nw, 1e-6)
    assert rel_err(_qlinear(lib, qw, x, N, bias=bias, resid=res, norm=nw), res + xn @ wd.T + bias) <= 2e-3
    full = xn @ wd.T + bias
    assert rel_err(_qlinear(lib, qw, x, N // 2, bias=bias, norm=nw, swiglu=1),
                   swiglu(full[:, 0::2], full[:, 1::2])) <= 2e-3
    lib.n730_qweight_destroy(qw)
