"""GPU next-token sampling (n730_sample) against the host sampler.

The host sampler is the reference's (``src-code/inference.py:674-682``),
restated in ``n730_b200.inference.sample``: argmax for temperature <= 0, else
temperature + nucleus (top-p) and ``choice``.  The GPU draws u from a hash of
(seed, counter, row) and reports it, so the host side is replayed with the same
u: numpy's choice rule is ``searchsorted(cumsum(q) / sum(q), u, 'right')``.

* greedy: bit-exact (the first index of the maximum, ties included);
* sampled: a pick of the rule under a float64 restatement (tokens by
  probability descending, ties by index): inside the nucleus, with u times the
  nucleus mass between the masses ahead of and through the token, where
  probabilities within 1e-6 of each other (fp32 exp rounding) may come in
  either order and boundaries carry 2e-6 of the total mass; the numpy float32
  sampler, replayed with the same u, picks the same token on rows where one
  token carries 99 % of the mass; over a large nucleus its sequential float32
  cumulative sums drift by up to ~n 2^-24 of the mass, too far to compare
  token by token.
"""
import ctypes as C

import numpy as np
import pytest

from n730_b200 import _lib
from n730_b200.inference import sample as host_sample

pytestmark = pytest.mark.gpu
V = 152064


def _gpu(logits, temp, top_p, seed, counter=0):
    import torch
    lib = _lib.cuda()
    B = logits.shape[0]
    d = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    u = torch.empty(B, dtype=torch.float32, device="cuda")
    _lib.check(lib.n730_sample(C.c_void_p(d.data_ptr()), B, logits.shape[1], logits.shape[1], temp, top_p, seed, counter,
                               C.c_void_p(tok.data_ptr()), C.c_void_p(u.data_ptr()), None), "sample")
    torch.cuda.synchronize()
    return tok.cpu().numpy(), u.cpu().numpy()


def _valid(row, temp, top_p, u, tok, eps=1e-6, tol=2e-6):
    """Is `tok` the pick of the rule for draw u, up to rounding?  In float64 from the same fp32
    z: tokens ahead of it have at least mass A (p above p_tok (1 + eps)) and at most B - p_tok
    (p above p_tok (1 - eps)); it must sit inside the nucleus and u * M must fall in [A, B]
    (tol of the total mass either way)."""
    z = (row.astype(np.float32) - row.max()) / np.float32(temp)
    p = np.exp(z.astype(np.float64))
    S = p.sum()
    order = np.lexsort((np.arange(len(p)), -p))  # p descending, index ascending
    c = np.cumsum(p[order])
    k = len(p) - 1 if top_p >= 1 else int(np.searchsorted(c, top_p * S, side="left"))
    M = c[min(k, len(p) - 1)]
    pt = p[tok]
    A = p[p > pt * (1 + eps)].sum()
    B = p[p >= pt * (1 - eps)].sum()
    in_nucleus = top_p >= 1 or A <= top_p * S + tol * S
    return bool(in_nucleus and A - tol * S <= u * M <= B + tol * S)


class _ReplayRng:
    """Stands in for numpy's Generator in the host sampler: choice() with a given u."""

    def __init__(self, u):
        self.u = float(u)

    def choice(self, a, p):
        cdf = np.cumsum(p)
        cdf /= cdf[-1]
        return a[int(np.searchsorted(cdf, self.u, side="right"))]


def _rows(kind, B, rng):
    if kind == "normal":
        return rng.normal(0, 2.0, (B, V)).astype(np.float32)
    if kind == "peaked":
        x = rng.normal(0, 1.0, (B, V)).astype(np.float32)
        x[np.arange(B), rng.integers(0, V, B)] += 20.0  # > 99.9 % of the mass on one token
        return x
    if kind == "flat":
        return (rng.normal(0, 0.01, (B, V))).astype(np.float32)
    if kind == "ties":  # whole rows of equal logits: order by index
        return np.zeros((B, V), np.float32)
    raise ValueError(kind)


def test_greedy_is_argmax():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (5, V)).astype(np.float32)
    x[1, [17, 99, 50000]] = 9.0        # ties: the first index wins, as np.argmax
    x[2, :] = -3.0
    tok, _ = _gpu(x, 0.0, 0.9, seed=1)
    assert np.array_equal(tok, x.argmax(axis=1))
    tok, _ = _gpu(x, -1.0, 0.5, seed=1)
    assert np.array_equal(tok, x.argmax(axis=1))


@pytest.mark.parametrize("kind", ["normal", "peaked", "flat", "ties"])
@pytest.mark.parametrize("temp,top_p", [(0.7, 0.9), (1.0, 1.0), (0.3, 0.5), (1.5, 0.99)])
def test_sampled_matches_host(kind, temp, top_p):
    rng = np.random.default_rng(hash((kind, temp, top_p)) % 2**32)
    B = 8
    x = _rows(kind, B, rng)
    for counter in range(3):
        tok, u = _gpu(x, temp, top_p, seed=1234, counter=counter)
        assert ((u >= 0) & (u < 1)).all()
        for b in range(B):
            assert _valid(x[b], temp, top_p, float(u[b]), int(tok[b])), (kind, b, int(tok[b]))
            # the host sampler sums float32 probabilities sequentially, so its cumulative mass
            # drifts by up to ~n 2^-24 over a large nucleus, and numpy's argsort leaves equal
            # values in any order: it must pick the same token where one token carries the mass
            z = (x[b].astype(np.float64) - x[b].max()) / temp
            if 1.0 / np.exp(z).sum() >= 0.99:
                assert int(tok[b]) == host_sample(x[b], temp, top_p, rng=_ReplayRng(u[b])), (kind, b)


def test_draws_differ_by_counter_and_row():
    x = np.zeros((4, V), np.float32)
    _, u0 = _gpu(x, 1.0, 1.0, seed=7, counter=0)
    _, u1 = _gpu(x, 1.0, 1.0, seed=7, counter=1)
    _, u2 = _gpu(x, 1.0, 1.0, seed=8, counter=0)
    assert len(set(u0.tolist())) == 4 and not np.array_equal(u0, u1) and not np.array_equal(u0, u2)
    tok, _ = _gpu(x, 1.0, 1.0, seed=7, counter=0)
    # equal logits: uniform over the vocabulary in index order
    assert np.array_equal(tok, np.minimum((u0.astype(np.float64) * V).astype(np.int64), V - 1))


def test_rejects_bad_arguments():
    lib = _lib.cuda()
    one = C.c_void_p(16)  # never dereferenced: the checks return first
    assert lib.n730_sample(None, 1, 10, 10, 1.0, 0.9, 0, 0, one, None, None) == -12
    assert lib.n730_sample(one, 1, 10, 5, 1.0, 0.9, 0, 0, one, None, None) == -13
    assert lib.n730_sample(one, 1, 10, 10, 1.0, 0.0, 0, 0, one, None, None) == -13
