"""Paths that the small test shapes do not reach with their default engines:

* split-K batched GEMV: a one-layer decoder with a 7B-wide FFN (down_proj K = 18944, whose x
  fragments for 8 batch columns exceed shared memory), decoded at batch 8;
* the tcgen05 GEMM inside the model: prefill chunks of >= 128 tokens (max_prefill 256);
* the persistent decode kernel with a phase table too large for shared memory (200 layers,
  1001 phases): read from global memory.

Both against the oracle decoder within the 1e-2 logit bar.
"""
import dataclasses

import numpy as np
import pytest

from gpu_util import rel_err
from oracle.model import OracleDecoder
from test_gpu_model import _blocks, _oracle_weights
from n730_b200 import synthetic
from n730_b200.engine import Engine, ModelShape, load_tensors

pytestmark = pytest.mark.gpu
TOL = 1e-2
WIDE = ModelShape(256, 1, 4, 2, 64, 18944, 1000, 1e6, 1e-6, False)


def _model(tmp_path, shape, seed):
    path = tmp_path / "m.n730"
    synthetic.write_n730(path, shape, "int4_g128", seed=seed)
    blocks = _blocks(path)
    return blocks, _oracle_weights(blocks)


def test_batch8_decode_split_k(tmp_path):
    blocks, w = _model(tmp_path, WIDE, seed=41)
    B = 8
    e = Engine(WIDE, max_ctx=128, max_batch=B, max_prefill=64)
    load_tensors(e, blocks)
    e.finalize()
    rng = np.random.default_rng(8)
    oracles = [OracleDecoder(WIDE, w, max_pos=128) for _ in range(B)]
    for b in range(B):
        p = rng.integers(0, WIDE.vocab, 5 + 3 * b)
        assert rel_err(e.forward(p, seq=b), oracles[b].forward(p)) <= TOL
    toks = rng.integers(0, WIDE.vocab, B)
    for step in range(4):
        y = e.decode(toks.astype(np.int32))
        for b in range(B):
            assert rel_err(y[b], oracles[b].forward([int(toks[b])])) <= TOL, (step, b)
        toks = np.argmax(y, axis=1)
    e.close()


@pytest.mark.parametrize("shape_name", ["tiny", "tiny-128"])
def test_long_prefill_uses_gemm(tmp_path, shape_name):
    shape = synthetic.SHAPES[shape_name]
    blocks, w = _model(tmp_path, shape, seed=43)
    e = Engine(shape, max_ctx=512, max_batch=1, max_prefill=256)
    load_tensors(e, blocks)
    e.finalize()
    orc = OracleDecoder(shape, w, max_pos=512)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, shape.vocab, 300)  # chunks of 256 and 44 tokens
    assert rel_err(e.forward(prompt), orc.forward(prompt)) <= TOL
    for t in (3, 17):
        assert rel_err(e.forward([t]), orc.forward([t])) <= TOL
    e.close()


def test_persistent_phase_table_in_global_memory(tmp_path):
    shape = dataclasses.replace(synthetic.SHAPES["tiny"], layers=200)
    blocks, w = _model(tmp_path, shape, seed=45)
    e = Engine(shape, max_ctx=256, max_batch=1, max_prefill=64, per_op_decode=-1)
    load_tensors(e, blocks)
    e.finalize()
    assert e.info()["persistent_decode"] and e.info()["phase_table_global"]
    orc = OracleDecoder(shape, w, max_pos=256)
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, shape.vocab, 80)
    assert rel_err(e.forward(prompt), orc.forward(prompt)) <= TOL
    tok = 7
    for step in range(5):
        y, yr = e.forward([tok]), orc.forward([tok])
        assert rel_err(y, yr) <= TOL, step
        tok = int(np.argmax(yr))
    e.close()
