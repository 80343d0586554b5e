"""Continuous batching on the engine (n730_b200.batching) against the oracle.

Nine requests of different prompt lengths and token counts share an engine of
3 slots whose KV pool holds 10 pages of 64 positions (a third of 3 x 512):
requests are admitted as pages free up, finished ones release their pages
(reused by later requests) and the last active request moves into the freed
slot.  Every emitted token's logits, replayed on a per-request oracle decoder
with the same tokens, must be within the 1e-2 bar.
"""
import numpy as np
import pytest

from gpu_util import rel_err
from oracle.model import OracleDecoder
from test_gpu_model import _blocks, _oracle_weights
from n730_b200 import synthetic
from n730_b200.batching import ContinuousBatcher
from n730_b200.engine import Engine, load_tensors

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape_name", ["tiny", "tiny-128"])
def test_continuous_batching_matches_oracle(tmp_path, shape_name):
    shape = synthetic.SHAPES[shape_name]
    path = tmp_path / "m.n730"
    synthetic.write_n730(path, shape, "int4_g128", seed=19)
    blocks = _blocks(path)
    w = _oracle_weights(blocks)
    e = Engine(shape, max_ctx=512, max_batch=3, max_prefill=64, kv_pool_pages=10)
    load_tensors(e, blocks)
    e.finalize()
    assert e.kv_pages() == (10, 10)
    b = ContinuousBatcher(e, keep_logits=True)
    rng = np.random.default_rng(4)
    reqs = {}
    for _ in range(9):
        p = rng.integers(0, shape.vocab, int(rng.integers(5, 150)))
        reqs[b.submit(p, int(rng.integers(3, 60)))] = p
    out = b.run()
    assert sorted(out) == sorted(reqs)
    assert e.kv_pages() == (10, 10)  # every page back in the pool
    for rid, p in reqs.items():
        r = out[rid]
        orc = OracleDecoder(shape, w, max_pos=512)
        assert rel_err(r.logits[0], orc.forward(p)) <= 1e-2, (rid, 0)
        for k, tok in enumerate(r.tokens[:-1]):
            assert rel_err(r.logits[k + 1], orc.forward([tok])) <= 1e-2, (rid, k + 1)
        assert r.tokens == [int(np.argmax(lg)) for lg in r.logits]
    e.close()


def test_pool_exhaustion_and_release(tmp_path):
    shape = synthetic.SHAPES["tiny"]
    path = tmp_path / "m.n730"
    synthetic.write_n730(path, shape, "int4_g128", seed=3)
    e = Engine(shape, max_ctx=512, max_batch=2, max_prefill=64, kv_pool_pages=4)
    load_tensors(e, _blocks(path))
    e.finalize()
    e.forward(np.arange(200) % shape.vocab, seq=0)           # 4 pages
    assert e.kv_pages() == (0, 4)
    with pytest.raises(RuntimeError, match="pool exhausted"):
        e.forward([1, 2, 3], seq=1)
    e.seq_release(0)
    assert e.kv_pages() == (4, 4) and e.seq_len(0) == 0
    y1 = e.forward([1, 2, 3], seq=1)                          # pages of sequence 0 reused
    e.seq_move(0, 1)
    assert e.seq_len(0) == 3 and e.seq_len(1) == 0
    y2 = e.forward([4], seq=0)                                # continues in its new slot
    orc = OracleDecoder(shape, _oracle_weights(_blocks(path)), max_pos=64)
    assert rel_err(y1, orc.forward([1, 2, 3])) <= 1e-2 and rel_err(y2, orc.forward([4])) <= 1e-2
    e.close()
