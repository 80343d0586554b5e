"""The reference's CUDA ABI, driven the way src-code/diagnose_binary.py drives it:
each sub-step compared with the oracle restatement of the reference math.
Bar: max|y - y_ref| / max|y_ref| <= 1e-4 (fp32 throughout)."""
import ctypes as C

import numpy as np
import pytest

from gpu_util import rel_err
from oracle import quant as oq
from oracle.model import apply_rope, attention, rms_norm, rope_table, swiglu
from n730_b200 import _lib

pytestmark = pytest.mark.gpu
FP = C.POINTER(C.c_float)


def fptr(a):
    return a.ctypes.data_as(FP)


class Buf:
    def __init__(self, lib, n):
        self.lib, self.n = lib, n
        self.p = C.c_void_p()
        _lib.check(lib.n730_device_alloc(n, C.byref(self.p)), "alloc")

    def fp(self):
        return C.cast(self.p, FP)

    def pull(self):
        out = np.zeros(self.n, np.float32)
        _lib.check(self.lib.n730_memcpy_d2h(fptr(out), self.p, self.n), "d2h")
        return out

    def push(self, a):
        a = np.ascontiguousarray(a, np.float32).reshape(-1)
        _lib.check(self.lib.n730_memcpy_h2d(self.p, fptr(a), a.size), "h2d")

    def __del__(self):
        self.lib.n730_device_free(self.p)


@pytest.mark.parametrize("prec", [8, 4, 2, 16])
def test_layer_walk(prec):
    lib = _lib.cuda()
    rng = np.random.default_rng(prec)
    h, nh, nkv, hd, inter, seq, eps, theta = 256, 4, 2, 64, 512, 6, 1e-6, 1e6
    ctx = C.c_void_p()
    _lib.check(lib.n730_cuda_init(h, nh, hd, 1000, 64, inter * h, C.byref(ctx)), "init")
    q_fn = {8: oq.quantize_int8, 4: oq.quantize_int4, 2: oq.quantize_int2, 16: oq.quantize_fp16}[prec]

    def upload(w):
        codes, s, z = q_fn(w)
        raw = np.frombuffer(codes, np.uint8).copy()
        _lib.check(lib.n730_upload_weight(ctx, raw.ctypes.data_as(C.POINTER(C.c_uint8)), prec, w.size, s, z), "upload")
        return oq.dequant_tensor(codes, prec, w.size, s, z).reshape(w.shape)

    x = rng.normal(0, 1, (seq, h)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, h).astype(np.float32)
    dn = C.c_void_p()
    _lib.check(lib.n730_upload_norm_weight(fptr(nw), h, C.byref(dn)), "norm")
    dcos, dsin = C.c_void_p(), C.c_void_p()
    _lib.check(lib.n730_rope_precompute(512, hd, theta, C.byref(dcos), C.byref(dsin)), "rope table")
    cos, sin = rope_table(512, hd, theta)
    _lib.check(lib.n730_load_activations(ctx, fptr(x), seq, h), "load")
    _lib.check(lib.n730_rmsnorm(ctx, dn, seq, eps), "rmsnorm")
    xn = rms_norm(x, nw, eps)

    dq, dk, dv = Buf(lib, seq * nh * hd), Buf(lib, seq * nkv * hd), Buf(lib, seq * nkv * hd)
    outs = {}
    for name, buf, n in (("q", dq, nh * hd), ("k", dk, nkv * hd), ("v", dv, nkv * hd)):
        w = rng.normal(0, 0.05, (n, h)).astype(np.float32)
        wd = upload(w)
        _lib.check(lib.n730_linear(ctx, buf.p, seq, h, n), "linear")
        ref = xn @ wd.T
        assert rel_err(buf.pull().reshape(seq, n), ref) <= 1e-4, name
        outs[name] = ref
    bias = rng.normal(0, 0.02, nh * hd).astype(np.float32)
    db = C.c_void_p()
    _lib.check(lib.n730_upload_norm_weight(fptr(bias), bias.size, C.byref(db)), "bias")
    _lib.check(lib.n730_add_bias(ctx, dq.fp(), C.cast(db, FP), seq, nh * hd), "add_bias")
    outs["q"] = outs["q"] + bias
    assert rel_err(dq.pull().reshape(seq, -1), outs["q"]) <= 1e-4

    _lib.check(lib.n730_apply_rope(dq.p, dcos, dsin, seq, nh, hd, 0), "rope q")
    _lib.check(lib.n730_apply_rope(dk.p, dcos, dsin, seq, nkv, hd, 0), "rope k")
    qr = apply_rope(outs["q"], nh, hd, 0, cos, sin)
    kr = apply_rope(outs["k"], nkv, hd, 0, cos, sin)
    assert rel_err(dq.pull().reshape(seq, -1), qr) <= 1e-4
    assert rel_err(dk.pull().reshape(seq, -1), kr) <= 1e-4

    da = Buf(lib, seq * nh * hd)
    _lib.check(lib.n730_attention_forward(ctx, dq.fp(), dk.fp(), dv.fp(), da.fp(), seq, seq, nh, nkv, hd, 0), "attn")
    aref = attention(qr, kr, outs["v"], nh, nkv, hd, 0)
    assert rel_err(da.pull().reshape(seq, -1), aref) <= 1e-4
    sc = np.zeros(nh * seq * seq, np.float32)
    _lib.check(lib.n730_get_scores(ctx, fptr(sc), nh, seq, seq), "scores")
    assert np.allclose(sc.reshape(nh, seq, seq).sum(-1), 1.0, atol=1e-5)
    assert np.all(np.triu(sc.reshape(nh, seq, seq)[0], 1) < 1e-6)  # causal

    wo = rng.normal(0, 0.05, (h, nh * hd)).astype(np.float32)
    wod = upload(wo)
    do = Buf(lib, seq * h)
    _lib.check(lib.n730_linear_from_buf(ctx, da.fp(), do.fp(), seq, nh * hd, h), "o_proj")
    o_ref = aref @ wod.T
    assert rel_err(do.pull().reshape(seq, h), o_ref) <= 1e-4
    _lib.check(lib.n730_residual_add(ctx, do.p, seq), "residual")
    act = np.zeros(seq * h, np.float32)
    _lib.check(lib.n730_get_activations(ctx, fptr(act), seq, h), "get")
    assert rel_err(act.reshape(seq, h), x + o_ref) <= 1e-4

    g = rng.normal(0, 1, (seq, inter)).astype(np.float32)
    u = rng.normal(0, 1, (seq, inter)).astype(np.float32)
    dg, du = Buf(lib, g.size), Buf(lib, u.size)
    dg.push(g)
    du.push(u)
    _lib.check(lib.n730_swiglu(dg.p, du.p, seq, inter), "swiglu")
    assert rel_err(dg.pull().reshape(seq, inter), swiglu(g, u)) <= 1e-5

    lib.n730_free_device_buf(dn)
    lib.n730_free_device_buf(db)
    lib.n730_free_device_buf(dcos)
    lib.n730_free_device_buf(dsin)
    lib.n730_cuda_destroy(ctx)
    assert lib.n730_sync() == 0


def test_decode_offset_attention():
    """seq_q = 1 against a longer cache (no mask), cache_offset > 0."""
    lib = _lib.cuda()
    rng = np.random.default_rng(3)
    nh, nkv, hd, total = 8, 2, 64, 37
    ctx = C.c_void_p()
    _lib.check(lib.n730_cuda_init(nh * hd, nh, hd, 100, 64, 16, C.byref(ctx)), "init")
    q = rng.normal(0, 1, (1, nh * hd)).astype(np.float32)
    k = rng.normal(0, 1, (total, nkv * hd)).astype(np.float32)
    v = rng.normal(0, 1, (total, nkv * hd)).astype(np.float32)
    dq, dk, dv, do = Buf(lib, q.size), Buf(lib, k.size), Buf(lib, v.size), Buf(lib, q.size)
    dq.push(q); dk.push(k); dv.push(v)
    _lib.check(lib.n730_attention_forward(ctx, dq.fp(), dk.fp(), dv.fp(), do.fp(), 1, total, nh, nkv, hd, total - 1), "attn")
    assert rel_err(do.pull().reshape(1, -1), attention(q, k, v, nh, nkv, hd, total - 1)) <= 1e-4
    lib.n730_cuda_destroy(ctx)
