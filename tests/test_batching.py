"""Continuous batching bookkeeping (n730_b200.batching) against a stand-in engine on the CPU:
slots stay compact (finished requests are replaced by the last active one), the KV pool is
reserved so an admitted request always runs to completion, every request gets its tokens."""
import numpy as np
import pytest

from n730_b200.batching import ContinuousBatcher

V = 50


class _Cfg:
    page_size = 4


class FakeEngine:
    """Greedy 'model': the next token is the last one + 1 (mod V).  Tracks per-slot lengths and
    pages the way the engine does (pages handed out as a sequence grows, returned on release)."""

    def __init__(self, max_batch=3, max_ctx=64, pool_pages=12):
        self.max_batch, self.max_ctx, self.cfg = max_batch, max_ctx, _Cfg()
        self.len = [0] * max_batch
        self.pages = [0] * max_batch
        self.pool = pool_pages
        self.moves = []

    def _grow(self, s, n):
        self.len[s] += n
        need = -(-self.len[s] // 4)
        assert sum(self.pages) - self.pages[s] + need <= self.pool, "pool exhausted"
        self.pages[s] = need

    def kv_pages(self):
        return self.pool - sum(self.pages), self.pool

    def forward(self, prompt, seq=0):
        assert self.len[seq] == 0
        self._grow(seq, len(prompt))
        out = np.zeros(V, np.float32)
        out[(int(prompt[-1]) + 1) % V] = 1
        return out

    def decode(self, toks):
        assert all(self.len[b] > 0 for b in range(len(toks)))
        out = np.zeros((len(toks), V), np.float32)
        for b, t in enumerate(toks):
            self._grow(b, 1)
            out[b, (int(t) + 1) % V] = 1
        return out

    def seq_release(self, s):
        self.len[s] = 0
        self.pages[s] = 0

    def seq_move(self, dst, src):
        assert self.len[dst] == 0 and self.pages[dst] == 0
        self.len[dst], self.pages[dst] = self.len[src], self.pages[src]
        self.len[src] = self.pages[src] = 0
        self.moves.append((dst, src))


def test_continuous_batching_bookkeeping():
    e = FakeEngine()
    b = ContinuousBatcher(e)
    rng = np.random.default_rng(0)
    reqs = {}
    for _ in range(9):
        p = rng.integers(0, V, int(rng.integers(1, 12)))
        n = int(rng.integers(1, 14))
        reqs[b.submit(p, n)] = (p, n)
    out = b.run()
    assert sorted(out) == sorted(reqs)
    for rid, (p, n) in reqs.items():
        assert out[rid].tokens == [(int(p[-1]) + k) % V for k in range(1, n + 1)]
    assert e.moves and e.kv_pages()[0] == e.pool and e.len == [0] * 3


def test_eos_and_rejections():
    e = FakeEngine(max_batch=2, pool_pages=5)
    b = ContinuousBatcher(e)
    rid = b.submit([7], 15, eos=10)               # stops at token 10
    with pytest.raises(ValueError):
        b.submit([1] * 30, 40)                    # beyond the context
    with pytest.raises(ValueError):
        b.submit([1] * 15, 10)                    # needs 7 pages, the pool has 5
    out = b.run()
    assert out[rid].tokens == [8, 9, 10]
