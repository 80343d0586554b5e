"""n730_attention_forward_noalloc against the context-based n730_attention_forward.

Both run the same kernels; the no-allocation entry point keeps the score
matrix in a fixed device array instead of the context's buffer.  Each case
calls it twice in a row (the scratch is reused) and requires bit-identical
outputs to the context path, and to the oracle's attention within 1e-4.
The file sorts last so the check also runs after every other GPU test.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import dev, ptr, rel_err
from oracle.model import attention
from n730_b200 import _lib

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 1 << 20


def fp(t):  # the reference ABI binds float* arguments
    return C.cast(C.c_void_p(t.data_ptr()), C.POINTER(C.c_float))


def _case(seq_q, total, nh, nkv, hd, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((seq_q, nh, hd)).astype(np.float32)
    k = rng.standard_normal((total, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((total, nkv, hd)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("seq_q,total,nh,nkv,hd", [(1, 300, 8, 2, 64), (16, 48, 14, 2, 64), (1, 2048, 28, 4, 128),
                                                   (5, 5, 4, 4, 128)])
def test_noalloc_matches_context_path(seq_q, total, nh, nkv, hd):
    import torch
    lib = _lib.cuda()
    q, k, v = _case(seq_q, total, nh, nkv, hd, seed=seq_q * 7 + total)
    off = total - seq_q
    dq, dk, dv = dev(q), dev(k), dev(v)
    ctx = C.c_void_p()
    _lib.check(lib.n730_cuda_init(nh * hd, nh, hd, 100, total, 16, C.byref(ctx)), "init")
    try:
        ref = torch.empty(seq_q, nh * hd, device="cuda")
        _lib.check(lib.n730_attention_forward(ctx, fp(dq), fp(dk), fp(dv), fp(ref), seq_q, total, nh, nkv, hd,
                                              off), "attention_forward")
        torch.cuda.synchronize()
        outs = []
        for _ in range(2):  # two calls in a row reuse the same scratch
            o = torch.full((seq_q, nh * hd), float("nan"), device="cuda")
            _lib.check(lib.n730_attention_forward_noalloc(ptr(dq), ptr(dk), ptr(dv), ptr(o), seq_q, total, nh, nkv,
                                                          hd, off, None), "attention_forward_noalloc")
            torch.cuda.synchronize()
            outs.append(o.cpu().numpy())
        r = ref.cpu().numpy()
        assert np.array_equal(outs[0], r) and np.array_equal(outs[1], r)
        want = attention(q.reshape(seq_q, -1), k.reshape(total, -1), v.reshape(total, -1), nh, nkv, hd, off)
        assert rel_err(outs[1], want) <= 1e-4
    finally:
        lib.n730_cuda_destroy(ctx)


def test_noalloc_on_a_stream():
    import torch
    lib = _lib.cuda()
    q, k, v = _case(1, 200, 8, 2, 64, seed=3)
    dq, dk, dv = dev(q), dev(k), dev(v)
    s = torch.cuda.Stream()
    o = torch.empty(1, 8 * 64, device="cuda")
    with torch.cuda.stream(s):
        _lib.check(lib.n730_attention_forward_noalloc(ptr(dq), ptr(dk), ptr(dv), ptr(o), 1, 200, 8, 2, 64, 199,
                                                      C.c_void_p(s.cuda_stream)), "noalloc on stream")
    s.synchronize()
    want = attention(q.reshape(1, -1), k.reshape(200, -1), v.reshape(200, -1), 8, 2, 64, 199)
    assert rel_err(o.cpu().numpy(), want) <= 1e-4


def test_noalloc_rejects_oversize_and_null():
    lib = _lib.cuda()
    one = C.c_void_p(16)  # never dereferenced: the size check returns first
    heads, total = 64, SCRATCH_FLOATS // 64 + 1
    assert lib.n730_attention_forward_noalloc(one, one, one, one, 1, total, heads, 8, 128, total - 1, None) == -13
    assert lib.n730_attention_forward_noalloc(None, one, one, one, 1, 10, 8, 2, 64, 9, None) == -12
    assert lib.n730_attention_forward_noalloc(one, one, one, one, 1, 10, 8, 3, 64, 9, None) == -13
    # within the scratch but beyond the launch-grid limit of 65535 queries / heads
    assert lib.n730_attention_forward_noalloc(one, one, one, one, 65536, 1, 1, 1, 64, 0, None) == -13
    assert lib.n730_attention_forward_noalloc(one, one, one, one, 1, 1, 65536, 1, 64, 0, None) == -13
