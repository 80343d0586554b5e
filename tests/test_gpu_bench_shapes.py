"""Parity at the benchmarked shapes, with the engine planning as the benchmark does.

The other model tests use small shapes and force the decode path.  Here the
engine keeps its automatic choices (``per_op_decode=0``, ``ffn_fuse=0``, the
settings ``bench.py`` runs) at the widths of the benchmark configurations, and
its logits are checked against the oracle decoder (max relative error 1e-2,
the bar of the reference's own check, ``src-code/diagnose_binary.py:28-35``)
on the codes the GPU quantiser produced (exported by ``build_on_device``):

* Qwen2-7B width (hidden 3584, 28/4 heads, head_dim 128, FFN 18944, vocab
  152064, all INT4 g128), 2 layers: the persistent kernel with the fused FFN
  (148 down_proj groups, one per SM), the lm_head's 152064 rows over the grid,
  37 KV splits per head; prefill chunks of 512 tokens through the tcgen05 GEMM;
  decode at contexts 2360-2371 (the step where a split starts to span two KV
  pages, position 2368) and 4084-4089.
* Qwen2-72B width (hidden 8192, 64/8 heads, FFN 29568), 1 layer, one GPU: 231
  down_proj groups spread unevenly over 148 CTAs in the fused FFN.
* Qwen2-0.5B width with the mixed map (INT8 per-tensor attention, INT4 g128
  FFN, FP16 tied embedding / lm_head), 2 layers: the per-op path the automatic
  choice takes, and the persistent kernel with INT8 / FP16 tiles.
* ``n730_qgemm`` (the tcgen05 GEMM) against the oracle's dequantised weights
  and numpy fp32 GEMM, with every epilogue.
"""
import ctypes as C
import dataclasses

import numpy as np
import pytest

from gpu_util import rel_err
from oracle import quant as oq
from oracle.model import OracleDecoder, rms_norm, swiglu
from n730_b200 import _lib, synthetic
from n730_b200.engine import Engine

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _dequant(item):
    if item["kind"] == "vector":
        return np.asarray(item["v"], np.float32)
    if item["kind"] == "block":
        b = item["block"]
        return oq.dequant_tensor(b.payload, b.prec_id, b.rows * b.cols, b.scale, b.zero_point).reshape(b.rows, b.cols)
    rows, cols = item["rows"], item["cols"]
    out = np.empty((rows, cols), np.float32)
    for r0 in range(0, rows, 8192):  # bounded temporaries for the 152k-row tables
        r1 = min(rows, r0 + 8192)
        out[r0:r1] = oq.dequant_grouped(item["codes"][r0:r1], item["s16"][r0:r1], item["z16"][r0:r1], item["bits"],
                                        r1 - r0, cols)
    return out


class _EmbedRows:
    """An untied embedding table dequantised one looked-up row at a time."""

    def __init__(self, item):
        self.item = item

    def __getitem__(self, ids):
        it = self.item
        ids = np.asarray(ids)
        return oq.dequant_grouped(it["codes"][ids], it["s16"][ids], it["z16"][ids], it["bits"], len(ids), it["cols"])


def _build(shape, pmap, seed, **engine_kw):
    """Engine built by build_on_device (the benchmark's builder) + the oracle's weights."""
    import torch
    torch.cuda.set_device(0)
    items = {}
    e = Engine(shape, **engine_kw)
    synthetic.build_on_device(shape, pmap, e, seed=seed, export=lambda n, it: items.__setitem__(n, it))
    e.finalize()
    w = {}
    for name, it in items.items():
        if name == "model.embed_tokens.weight" and not shape.tie_embeddings and it["kind"] == "grouped":
            w[name] = _EmbedRows(it)
        else:
            w[name] = _dequant(it)
    return e, w


def _prefill(e, orc, prompt, chunk=512):
    y = e.forward(prompt)
    for i in range(0, len(prompt), chunk):
        yr = orc.forward(prompt[i:i + chunk])
    return y, yr


def _decode(e, orc, tok, steps, label):
    for s in range(steps):
        y, yr = e.forward([tok]), orc.forward([tok])
        err = rel_err(y, yr)
        assert err <= TOL, f"{label}: step {s} at position {orc.seq_len - 1}: {err:.3g}"
        tok = int(np.argmax(yr))
    return tok


def test_7b_width_auto_plan_long_context():
    shape = dataclasses.replace(synthetic.SHAPES["qwen2-7b"], layers=2)
    e, w = _build(shape, "int4_g128", seed=7, max_ctx=4096, max_batch=1, max_prefill=512)
    info = e.info()
    assert info["persistent_decode"] and info["ffn_fused"], info  # what bench.py runs at this width
    assert not info["phase_table_global"]
    orc = OracleDecoder(shape, w, max_pos=4096)
    rng = np.random.default_rng(70)
    y, yr = _prefill(e, orc, rng.integers(0, shape.vocab, 512))
    assert rel_err(y, yr) <= TOL
    tok = _decode(e, orc, int(rng.integers(0, shape.vocab)), 3, "ctx 512")
    # to 2360 cached positions: 37 splits of one page each, then two pages per split from 2368 on
    y, yr = _prefill(e, orc, rng.integers(0, shape.vocab, 2360 - orc.seq_len))
    assert rel_err(y, yr) <= TOL
    tok = _decode(e, orc, tok, 12, "ctx 2360-2371")
    y, yr = _prefill(e, orc, rng.integers(0, shape.vocab, 4084 - orc.seq_len))
    assert rel_err(y, yr) <= TOL
    _decode(e, orc, tok, 6, "ctx 4084-4089")
    assert e.seq_len(0) == 4090
    e.close()


@pytest.mark.parametrize("B", [24, 32])
def test_7b_width_batched_decode_gemm(B):
    """Decode batches at 7B width: every linear takes the tcgen05 GEMM with a 32-token tile,
    K split over CTAs for q|k|v / o_proj / down_proj; at 32 sequences their folds also hand
    the sums of squares of the residual stream to the next RMSNorm (gate|up, the final norm),
    at 24 a 1/rms kernel runs.  Two of the sequences are replayed on the oracle, and the
    steps replay bit-identically."""
    shape = dataclasses.replace(synthetic.SHAPES["qwen2-7b"], layers=1)
    e, w = _build(shape, "int4_g128", seed=11, max_ctx=128, max_batch=B, max_prefill=64)
    rng = np.random.default_rng(24)
    picks = (0, 17)
    orcs = {b: OracleDecoder(shape, w, max_pos=128) for b in picks}
    for b in range(B):
        p = rng.integers(0, shape.vocab, 9 + b % 4)
        y = e.forward(p, seq=b)
        if b in orcs:
            assert rel_err(y, orcs[b].forward(p)) <= TOL
    toks = rng.integers(0, shape.vocab, B)
    lens = [e.seq_len(b) for b in range(B)]
    steps = []
    for step in range(2):
        y = e.decode(toks)
        steps.append((toks.copy(), y.copy()))
        for b in picks:
            assert rel_err(y[b], orcs[b].forward([int(toks[b])])) <= TOL, (step, b)
        toks = np.argmax(y, axis=1)
    # split-K folds and the per-slice sums of squares are reduced in a fixed order
    for b in range(B):
        e.set_seq_len(b, lens[b])
    for t, y0 in steps:
        assert np.array_equal(e.decode(t), y0)
    e.close()


def test_72b_width_uneven_fused_ffn():
    shape = dataclasses.replace(synthetic.SHAPES["qwen2-72b"], layers=1, vocab=4096)
    e, w = _build(shape, "int4_g128", seed=9, max_ctx=512, max_batch=1, max_prefill=512)
    info = e.info()
    # 231 down groups over 148 CTAs: the two-phase FFN does not fit, the fused one runs
    assert info["persistent_decode"] and info["ffn_fused"], info
    orc = OracleDecoder(shape, w, max_pos=512)
    rng = np.random.default_rng(72)
    y, yr = _prefill(e, orc, rng.integers(0, shape.vocab, 300))
    assert rel_err(y, yr) <= TOL
    _decode(e, orc, int(rng.integers(0, shape.vocab)), 8, "72b width")
    e.close()


@pytest.mark.parametrize("per_op", [0, -1], ids=["auto", "persistent"])
def test_05b_width_mixed(per_op):
    shape = dataclasses.replace(synthetic.SHAPES["qwen2-0.5b"], layers=2)
    e, w = _build(shape, "mixed_05b", seed=5, max_ctx=1024, max_batch=1, max_prefill=512, per_op_decode=per_op)
    info = e.info()
    # auto: 8 MB layers decode faster through the per-op kernels; forced: INT8 / FP16 persistent tiles,
    # two GEMV phases for the FFN (38 down groups do not divide over the SMs)
    assert info["persistent_decode"] == (per_op == -1), info
    assert not info["ffn_fused"]
    orc = OracleDecoder(shape, w, max_pos=1024)
    rng = np.random.default_rng(5)
    y, yr = _prefill(e, orc, rng.integers(0, shape.vocab, 700))
    assert rel_err(y, yr) <= TOL
    _decode(e, orc, int(rng.integers(0, shape.vocab)), 10, f"0.5b mixed, per_op_decode={per_op}")
    e.close()


def _gpu_weight(rows, cols, seed):
    import torch
    lib = _lib.cuda()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
    s16 = torch.empty(rows, cols // 128, dtype=torch.float16, device="cuda")
    z16 = torch.empty_like(s16)
    P = lambda t: C.c_void_p(t.data_ptr())
    _lib.check(lib.n730_quantize_grouped(P(w), rows, cols, 4, 128, P(codes), P(s16), P(z16), None), "quantize")
    q = C.c_void_p()
    _lib.check(lib.n730_qweight_create(0x44, rows, cols, 128, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                       C.byref(q)), "create")
    _lib.check(lib.n730_qweight_set_layout(q, 1, None), "layout")
    torch.cuda.synchronize()
    W = oq.dequant_grouped(codes.cpu().numpy(), s16.cpu().numpy(), z16.cpu().numpy(), 4, rows, cols)
    return q, W


@pytest.mark.parametrize("rows,cols,tokens,epi", [(1024, 3584, 512, "plain"), (3584, 18944, 256, "bias_resid"),
                                                  (19200, 3584, 300, "norm_swiglu"), (37888, 3584, 512, "plain"),
                                                  (3584, 18944, 32, "bias_resid"), (4608, 3584, 40, "plain"),
                                                  (37888, 3584, 24, "norm_swiglu"),
                                                  (2048, 3584, 300, "norm_swiglu"), (640, 8192, 129, "plain")])
def test_qgemm_matches_oracle(rows, cols, tokens, epi):
    """The tcgen05 GEMM rounds x and the dequantised weights to fp16 and accumulates in fp32:
    within 5e-3 of max|y| of the oracle's fp32 product of the exact dequantised weights.
    Decode-sized calls (< 128 tokens) of the narrow down_proj / q|k|v shapes split K over
    CTAs and fold the parts; the wide SwiGLU one does not split."""
    import torch
    lib = _lib.cuda()
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    q, W = _gpu_weight(rows, cols, seed=rows * 7 + cols)
    rng = np.random.default_rng(tokens)
    x = rng.normal(0, 1, (tokens, cols)).astype(np.float32)
    sw = epi == "norm_swiglu"
    out_cols = rows // 2 if sw else rows
    bias = rng.normal(0, 0.1, rows).astype(np.float32) if epi == "bias_resid" else None
    res = rng.normal(0, 1, (tokens, out_cols)).astype(np.float32) if epi == "bias_resid" else None
    nw = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32) if sw else None
    T = lambda a: torch.from_numpy(a).cuda() if a is not None else None
    dx, db, dr, dn = T(x), T(bias), T(res), T(nw)
    y = torch.full((tokens, out_cols), float("nan"), device="cuda")
    ws = torch.empty(tokens, device="cuda")
    _lib.check(lib.n730_qgemm(q, P(dx), cols, tokens, P(y), out_cols, P(db), P(dr), out_cols, P(dn), 1e-6,
                              int(sw), P(ws), None), "qgemm")
    torch.cuda.synchronize()
    lib.n730_qweight_destroy(q)
    xin = rms_norm(x, nw, 1e-6) if sw else x
    full = oq.gemv(W, xin)
    if bias is not None:
        full = full + bias
    ref = swiglu(full[:, 0::2], full[:, 1::2]) if sw else full   # gate|up rows interleaved
    if res is not None:
        ref = ref + res
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_err(got, ref) <= 5e-3


@pytest.mark.parametrize("batch", [1, 8])
def test_lm_head_gemv_matches_oracle(batch):
    """The tensor-core GEMV at lm_head size (152064 x 3584 INT4 g128, 65 row tiles per CTA) with
    the final RMSNorm folded in: the per-op decode and prefill logits path, against the oracle."""
    import torch
    lib = _lib.cuda()
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    rows, cols = 152064, 3584
    q, W = _gpu_weight(rows, cols, seed=11)
    rng = np.random.default_rng(batch)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    nw = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    dx, dn = torch.from_numpy(x).cuda(), torch.from_numpy(nw).cuda()
    y = torch.full((batch, rows), float("nan"), device="cuda")
    _lib.check(lib.n730_qlinear(q, P(dx), cols, batch, P(y), rows, None, None, 0, P(dn), 1e-6, 0, None), "qlinear")
    torch.cuda.synchronize()
    lib.n730_qweight_destroy(q)
    ref = oq.gemv(W, rms_norm(x, nw, 1e-6))
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    for b in range(batch):
        assert rel_err(got[b], ref[b]) <= 2e-3, b
