"""tcgen05 GEMM (n730_qgemm) against the tensor-core GEMV on the same weights.

Both read INT4 group-wise weights in fragment tiles and round x to fp16; the
GEMM also rounds the dequantised weights to fp16 (one more 2^-11 relative error
per weight), so the bar is 3e-3 of max|y|.  Covers token counts below, at and
across the 128- and 256-token tiles (256-token tiles are taken when there are
enough row tiles to fill the SMs: 150 x 2 here), partial row tiles, groups of
64, 128 and 256 columns, and every epilogue.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import rel_err
from n730_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 3e-3


def _weight(rows, cols, seed, group=128):
    import torch
    lib = _lib.cuda()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
    s16 = torch.empty(rows, cols // group, dtype=torch.float16, device="cuda")
    z16 = torch.empty_like(s16)
    P = lambda t: C.c_void_p(t.data_ptr())
    _lib.check(lib.n730_quantize_grouped(P(w), rows, cols, 4, group, P(codes), P(s16), P(z16), None), "quantize")
    q = C.c_void_p()
    _lib.check(lib.n730_qweight_create(0x44, rows, cols, group, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                       C.byref(q)), "create")
    _lib.check(lib.n730_qweight_set_layout(q, 1, None), "layout")
    torch.cuda.synchronize()
    return q


@pytest.mark.parametrize("rows,cols,tokens,group", [(256, 512, 128, 128), (400, 512, 33, 128), (384, 1024, 300, 128),
                                                    (160, 256, 1, 128), (512, 3584, 200, 128), (19200, 512, 300, 128),
                                                    (19200, 512, 256, 128), (1024, 1024, 200, 64),
                                                    (1024, 1024, 200, 256), (19200, 1024, 270, 256)])
@pytest.mark.parametrize("epi", ["plain", "bias_resid", "norm_swiglu"])
def test_qgemm_matches_gemv(rows, cols, tokens, group, epi):
    import torch
    lib = _lib.cuda()
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    q = _weight(rows, cols, seed=rows + cols, group=group)
    g = torch.Generator(device="cuda")
    g.manual_seed(tokens)
    x = torch.randn(tokens, cols, generator=g, device="cuda")
    bias = torch.randn(rows, generator=g, device="cuda") * 0.1 if epi == "bias_resid" else None
    nw = (1 + 0.1 * torch.randn(cols, generator=g, device="cuda")) if epi == "norm_swiglu" else None
    sw = 1 if epi == "norm_swiglu" else 0
    out_cols = rows // 2 if sw else rows
    res = torch.randn(tokens, out_cols, generator=g, device="cuda") if epi == "bias_resid" else None
    ws = torch.empty(tokens, device="cuda")
    y_ref = torch.empty(tokens, out_cols, device="cuda")
    y = torch.full((tokens, out_cols), float("nan"), device="cuda")
    # reference: the GEMV in chunks of 16 tokens
    for t0 in range(0, tokens, 16):
        n = min(16, tokens - t0)
        _lib.check(lib.n730_qlinear(q, C.c_void_p(x[t0].data_ptr()), cols, n, C.c_void_p(y_ref[t0].data_ptr()),
                                    out_cols, P(bias), C.c_void_p(res[t0].data_ptr()) if res is not None else None,
                                    out_cols, P(nw), 1e-6, sw, None), "qlinear")
    _lib.check(lib.n730_qgemm(q, P(x), cols, tokens, P(y), out_cols, P(bias), P(res), out_cols, P(nw), 1e-6, sw,
                              P(ws), None), "qgemm")
    torch.cuda.synchronize()
    lib.n730_qweight_destroy(q)
    a, b = y.cpu().numpy(), y_ref.cpu().numpy()
    assert np.isfinite(a).all()
    assert rel_err(a, b) <= TOL


def test_qgemm_rejects_row_major_weights():
    import torch
    lib = _lib.cuda()
    codes = torch.zeros(64 * 128 // 2, dtype=torch.uint8, device="cuda")
    s16 = torch.ones(64, 1, dtype=torch.float16, device="cuda")
    z16 = torch.zeros(64, 1, dtype=torch.float16, device="cuda")
    q = C.c_void_p()
    P = lambda t: C.c_void_p(t.data_ptr())
    _lib.check(lib.n730_qweight_create(0x44, 64, 128, 128, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                       C.byref(q)), "create")
    x = torch.zeros(40, 128, device="cuda")
    y = torch.zeros(40, 64, device="cuda")
    assert lib.n730_qgemm(q, P(x), 128, 40, P(y), 64, None, None, 0, None, 1e-6, 0, None, None) == -14
    lib.n730_qweight_destroy(q)
