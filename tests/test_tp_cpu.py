"""Tensor-parallel sharding and dataflow on CPU: two gloo ranks.

Each rank holds the shards ``n730_b200.tp`` assigns (q/k/v by heads, gate/up by
FFN groups, o/down by the matching input columns, lm_head by vocabulary) and
runs the numpy decoder of the oracle with one allreduce after o_proj and after
down_proj and an all-gather of the logits - the exchange steps the engine
issues through NCCL.  The result must match the unsharded oracle.
"""
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.model import OracleDecoder, apply_rope, attention, rms_norm, swiglu
from n730_b200 import synthetic, tp

FFN_GROUP = 128


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class TPOracle(OracleDecoder):
    def __init__(self, shape, weights, rank, size, max_pos=256):
        super().__init__(tp.local_shape(shape, size, rank, FFN_GROUP), weights, max_pos)
        self.vocab_split = tp.lm_head_split(shape, size)

    @staticmethod
    def _sum(y):
        t = torch.from_numpy(np.ascontiguousarray(y, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    def layer(self, i, x, offset):
        c = self.cfg
        p = f"model.layers.{i}"
        h = rms_norm(x, self._norm(f"{p}.input_layernorm.weight"), c.rms_norm_eps)
        q = apply_rope(self._lin(h, f"{p}.self_attn.q_proj"), c.num_attention_heads, c.head_dim, offset, self.cos, self.sin)
        k = apply_rope(self._lin(h, f"{p}.self_attn.k_proj"), c.num_kv_heads, c.head_dim, offset, self.cos, self.sin)
        v = self._lin(h, f"{p}.self_attn.v_proj")
        self.k[i] = np.concatenate([self.k[i], k])
        self.v[i] = np.concatenate([self.v[i], v])
        a = attention(q, self.k[i], self.v[i], c.num_attention_heads, c.num_kv_heads, c.head_dim, offset)
        x = (x + self._sum(self._lin(a, f"{p}.self_attn.o_proj"))).astype(np.float32)
        h2 = rms_norm(x, self._norm(f"{p}.post_attention_layernorm.weight"), c.rms_norm_eps)
        m = swiglu(self._lin(h2, f"{p}.mlp.gate_proj"), self._lin(h2, f"{p}.mlp.up_proj"))
        return (x + self._sum(self._lin(m, f"{p}.mlp.down_proj"))).astype(np.float32)

    def forward(self, ids):
        y = super().forward(ids)
        if not self.vocab_split:
            return y
        parts = [torch.empty(len(y)) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, torch.from_numpy(y))
        return torch.cat(parts).numpy()


class TPPushOracle(TPOracle):
    """The persistent kernel's exchange: every rank's partial sums land in one slot per rank
    (here an all-gather) and each rank adds them to its residual in rank order,
    ((x + p_0) + p_1) + ..., so the new residual is bit-identical on every rank."""

    def _resid(self, x, y):
        t = torch.from_numpy(np.ascontiguousarray(y, np.float32))
        parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
        dist.all_gather(parts, t)
        acc = x.astype(np.float32)
        for part in parts:
            acc = (acc + part.numpy()).astype(np.float32)
        return acc

    def layer(self, i, x, offset):
        c = self.cfg
        p = f"model.layers.{i}"
        h = rms_norm(x, self._norm(f"{p}.input_layernorm.weight"), c.rms_norm_eps)
        q = apply_rope(self._lin(h, f"{p}.self_attn.q_proj"), c.num_attention_heads, c.head_dim, offset, self.cos, self.sin)
        k = apply_rope(self._lin(h, f"{p}.self_attn.k_proj"), c.num_kv_heads, c.head_dim, offset, self.cos, self.sin)
        v = self._lin(h, f"{p}.self_attn.v_proj")
        self.k[i] = np.concatenate([self.k[i], k])
        self.v[i] = np.concatenate([self.v[i], v])
        a = attention(q, self.k[i], self.v[i], c.num_attention_heads, c.num_kv_heads, c.head_dim, offset)
        x = self._resid(x, self._lin(a, f"{p}.self_attn.o_proj"))
        h2 = rms_norm(x, self._norm(f"{p}.post_attention_layernorm.weight"), c.rms_norm_eps)
        m = swiglu(self._lin(h2, f"{p}.mlp.gate_proj"), self._lin(h2, f"{p}.mlp.up_proj"))
        return self._resid(x, self._lin(m, f"{p}.mlp.down_proj"))


def _push_worker(rank, size, port, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size)
    try:
        shape = synthetic.SHAPES["tiny"]
        full = dict(synthetic.host_tensors(shape, seed=6))
        local = {n: np.ascontiguousarray(s) for n, w in full.items()
                 if (s := tp.shard(n, w, shape, size, rank, FFN_GROUP)) is not None}
        o = TPPushOracle(shape, local, rank, size)
        rng = np.random.default_rng(4)
        ys = [o.forward(rng.integers(0, shape.vocab, 7))] + [o.forward([t]) for t in (2, 9)]
        # every rank must hold the same logits, bit for bit
        t = torch.from_numpy(np.concatenate(ys))
        gathered = [torch.empty_like(t) for _ in range(size)]
        dist.all_gather(gathered, t)
        same = all(torch.equal(gathered[0], g) for g in gathered)
        if rank == 0:
            ref = OracleDecoder(shape, full, max_pos=256)
            rng = np.random.default_rng(4)
            refs = [ref.forward(rng.integers(0, shape.vocab, 7))] + [ref.forward([t]) for t in (2, 9)]
            out.put((same, max(float(np.max(np.abs(a - b)) / np.max(np.abs(b))) for a, b in zip(ys, refs))))
    finally:
        dist.destroy_process_group()


def test_tp2_rank_order_push_sums():
    """The persistent decode kernel's exchange (partials pushed to per-rank slots, summed into
    the residual in rank order on every rank): identical on both ranks, = unsharded <= 1e-5."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_push_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    same, err = q.get(timeout=5)
    assert same and err <= 1e-5


class _FakeEngine:
    """Stands in for Engine in the communicator handshake (no GPU): records the calls."""

    def __init__(self, rank, sig=(896, 2, 7, 1, 64, 1000)):
        self.rank, self.calls, self.sig = rank, [], sig

    def tp_signature(self):
        return self.sig

    def tp_unique_id(self):
        return b"id-of-rank-0".ljust(128, b"\0")

    def tp_init(self, uid, rank, size):
        self.calls.append(("init", uid[:12], rank, size))

    def tp_ipc_handle(self):
        return bytes([self.rank]) * 64

    def tp_ipc_open(self, handles, size):
        self.calls.append(("open", handles, size))


def _handshake_worker(rank, size, port, map_peers, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size)
    try:
        e = _FakeEngine(rank)
        tp.init_engine_comm(e, rank, size, map_peers=map_peers)
        out.put((rank, e.calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("map_peers", [True, False])
def test_engine_comm_handshake(map_peers):
    """Rank 0's NCCL id reaches every rank; with map_peers every rank opens all ranks'
    exchange-region handles in rank order (the persistent kernel's peer pointers)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_handshake_worker, args=(r, 2, port, map_peers, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(q.get(timeout=5) for _ in range(2))
    for rank, calls in got.items():
        assert calls[0] == ("init", b"id-of-rank-0", rank, 2)
        if map_peers:
            assert calls[1] == ("open", bytes([0]) * 64 + bytes([1]) * 64, 2) and len(calls) == 2
        else:
            assert len(calls) == 1


def _worker(rank, size, port, shape_name, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size)
    try:
        shape = synthetic.SHAPES[shape_name]
        full = dict(synthetic.host_tensors(shape, seed=5))
        local = {}
        for n, w in full.items():
            s = tp.shard(n, w, shape, size, rank, FFN_GROUP)
            if s is not None:
                local[n] = np.ascontiguousarray(s)
        o = TPOracle(shape, local, rank, size)
        rng = np.random.default_rng(2)
        ys = [o.forward(rng.integers(0, shape.vocab, 9))]
        for t in (3, 8, 1):
            ys.append(o.forward([t]))
        if rank == 0:
            ref = OracleDecoder(shape, full, max_pos=256)
            rng = np.random.default_rng(2)
            refs = [ref.forward(rng.integers(0, shape.vocab, 9))] + [ref.forward([t]) for t in (3, 8, 1)]
            out.put(max(float(np.max(np.abs(a - b)) / np.max(np.abs(b))) for a, b in zip(ys, refs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape_name", ["tiny", "tiny-gqa7"])
def test_tp2_matches_unsharded(shape_name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) <= 1e-5


def test_shard_geometry():
    s72 = synthetic.SHAPES["qwen2-72b"]
    # 231 groups of 128 over 8 ranks: 28 or 29 whole groups each, covering the FFN exactly
    spans = [tp.span(s72.ffn, 8, r, 128) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == s72.ffn
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert sorted({(hi - lo) // 128 for lo, hi in spans}) == [28, 29]
    loc = tp.local_shape(s72, 8, 3, 128)
    assert (loc.heads, loc.kv_heads, loc.hidden, loc.vocab) == (8, 1, 8192, 152064)
    assert tp.lm_head_split(s72, 8) and not tp.lm_head_split(synthetic.SHAPES["qwen2-0.5b"], 2)
    with pytest.raises(ValueError):
        tp.check_shape(synthetic.SHAPES["qwen2-7b"], 8, 128)  # 4 KV heads over 8 ranks
    with pytest.raises(ValueError, match="o_proj"):
        tp.check_shape(synthetic.SHAPES["tiny-gqa7"], 2, 128)  # 7 heads x 64 = 448 columns per rank
    tp.check_shape(synthetic.SHAPES["qwen2-72b"], 8, 128)


@pytest.mark.parametrize("name,rows,cols", [("model.layers.0.mlp.down_proj.weight", 256, 512),
                                            ("model.layers.0.mlp.gate_proj.weight", 512, 256),
                                            ("model.layers.0.self_attn.o_proj.weight", 256, 256),
                                            ("model.layers.0.self_attn.k_proj.weight", 128, 256),
                                            ("lm_head.weight", 1000, 256)])
def test_shard_block_matches_sliced_dequant(name, rows, cols):
    """A packed group-wise block sharded in place dequantises to the slice of the full tensor."""
    import struct

    from oracle import quant as oq
    from n730_b200.converter import serialize_layer
    from n730_b200.formats import RawBlock, group_size_from_block
    shape = synthetic.SHAPES["tiny"]
    w = np.random.default_rng(rows + cols).normal(0, .02, (rows, cols)).astype(np.float32)
    blk, _ = serialize_layer(0, "INT4G", w, name, 128)
    _, _, pid, r, c, sc, zp, dsz = struct.unpack(">4sIBIIffi", blk[:29])
    b = RawBlock(0, pid, r, c, sc, zp, blk[29:29 + dsz], group_size_from_block(pid, r, c, dsz))
    full = oq.dequant_grouped(b.codes, b.scales16, b.zeros16, 4, r, c)
    for rank in range(2):
        sb = tp.shard_block(name, b, shape, 2, rank, FFN_GROUP)
        r0, r1, c0, c1 = tp.shard_ranges(name, r, c, shape, 2, rank, FFN_GROUP)
        part = oq.dequant_grouped(sb.codes, sb.scales16, sb.zeros16, 4, sb.rows, sb.cols)
        assert np.array_equal(part, full[r0:r1, c0:c1])


def _missing_rank_worker(rank, size, port, out):
    from datetime import timedelta
    import time
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size,
                            timeout=timedelta(seconds=3))
    if rank == 1:  # joins the process group but never the engine communicator
        time.sleep(12)
        out.put((1, None, 0.0))
        return
    t0 = time.monotonic()
    e = _FakeEngine(rank)
    try:
        tp.init_engine_comm(e, rank, size)
        out.put((0, "returned", time.monotonic() - t0))
    except Exception as ex:  # the process group's timeout ends the handshake
        out.put((0, type(ex).__name__, time.monotonic() - t0, e.calls))


def test_engine_comm_rank_never_joins():
    """A rank that never calls init_engine_comm: the other rank's handshake ends with an error
    at the process group's timeout (3 s here), before it enters NCCL's set-up (which has no
    timeout of its own): no tp_init call was made."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_missing_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=60)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
    kind, elapsed, calls = res[0][1], res[0][2], res[0][3]
    assert kind != "returned" and elapsed < 11.0, res[0]
    assert calls == []


def _mismatch_worker(rank, size, port, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size)
    try:
        e = _FakeEngine(rank, sig=(896, 2, 7, 1, 64, 1000 + rank))  # rank 1 built another vocabulary
        try:
            tp.init_engine_comm(e, rank, size)
            out.put((rank, "returned", e.calls))
        except ValueError as ex:
            out.put((rank, str(ex), e.calls))
    finally:
        dist.destroy_process_group()


def test_engine_comm_config_mismatch():
    """Ranks configured differently: every rank raises ValueError before any NCCL set-up."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_mismatch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    got = dict((r, (msg, calls)) for r, msg, calls in (q.get(timeout=5) for _ in range(2)))
    for rank in range(2):
        msg, calls = got[rank]
        assert "configured differently" in msg and calls == []
