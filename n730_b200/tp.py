"""Tensor-parallel sharding of a Qwen-like decoder over ``size`` ranks.

Column split (each rank computes whole output rows, no exchange): q/k/v by
attention heads / KV heads, gate/up by FFN rows in whole quantisation groups
of down_proj's input.  Row split (each rank a slice of the input columns, the
partial outputs are summed by one allreduce per projection): o_proj by the
rank's heads, down_proj by the rank's FFN rows.  The lm_head is split by
vocabulary rows (logits all-gathered) when the vocabulary divides evenly,
else replicated; embeddings and norms are replicated.  Biases of the row-split
projections are added by rank 0 only, so the allreduce counts them once.
The KV cache is sharded with the KV heads.
"""
from __future__ import annotations

import dataclasses

import numpy as np


def span(n: int, size: int, rank: int, unit: int = 1):
    """[lo, hi) of rank's share of n items split in whole ``unit``s (first ranks take the extra units)."""
    units = n // unit
    assert units * unit == n, (n, unit)
    lo = rank * units // size
    hi = (rank + 1) * units // size
    return lo * unit, hi * unit


def check_shape(shape, size: int, ffn_group: int, attn_group: int = 128):
    """Raise unless the shape splits over ``size`` ranks: whole heads and KV heads per
    rank, o_proj's per-rank input columns a whole number of its quant groups, and
    at least one FFN group per rank."""
    if shape.heads % size or shape.kv_heads % size:
        raise ValueError(f"{shape.heads} heads / {shape.kv_heads} KV heads do not split over {size} ranks")
    if size > 1 and (shape.heads // size * shape.head_dim) % attn_group:
        raise ValueError(f"o_proj input columns per rank ({shape.heads // size * shape.head_dim}) are not whole "
                         f"groups of {attn_group}")
    if (shape.ffn // ffn_group) < size:
        raise ValueError(f"FFN {shape.ffn} has fewer than {size} groups of {ffn_group}")


def lm_head_split(shape, size: int) -> bool:
    return size > 1 and not shape.tie_embeddings and shape.vocab % size == 0


def local_shape(shape, size: int, rank: int, ffn_group: int):
    """This rank's ModelShape: local heads, KV heads and FFN rows; hidden and vocab stay global."""
    if size == 1:
        return shape
    lo, hi = span(shape.ffn, size, rank, ffn_group)
    return dataclasses.replace(shape, heads=shape.heads // size, kv_heads=shape.kv_heads // size, ffn=hi - lo)


def shard_ranges(name: str, rows: int, cols: int, shape, size: int, rank: int, ffn_group: int):
    """(r0, r1, c0, c1) of tensor ``name`` [rows, cols] (cols = 1 for vectors) kept by
    ``rank``; None when the rank drops it (row-split biases on ranks > 0)."""
    full = (0, rows, 0, cols)
    if size == 1:
        return full
    hd = shape.head_dim
    qh = span(shape.heads, size, rank)
    kvh = span(shape.kv_heads, size, rank)
    f0, f1 = span(shape.ffn, size, rank, ffn_group)
    if name == "lm_head.weight":
        return (*span(shape.vocab, size, rank), 0, cols) if lm_head_split(shape, size) else full
    if not name.startswith("model.layers."):
        return full  # embeddings, final norm
    tail = name.split(".", 3)[3]
    if tail.startswith("self_attn.q_proj."):
        return qh[0] * hd, qh[1] * hd, 0, cols
    if tail.startswith(("self_attn.k_proj.", "self_attn.v_proj.")):
        return kvh[0] * hd, kvh[1] * hd, 0, cols
    if tail == "self_attn.o_proj.weight":
        return 0, rows, qh[0] * hd, qh[1] * hd
    if tail.startswith(("mlp.gate_proj.", "mlp.up_proj.")):
        return f0, f1, 0, cols
    if tail == "mlp.down_proj.weight":
        return 0, rows, f0, f1
    if tail in ("self_attn.o_proj.bias", "mlp.down_proj.bias"):
        return full if rank == 0 else None
    return full  # layer norms


def shard(name: str, w, shape, size: int, rank: int, ffn_group: int):
    """This rank's slice of tensor ``name`` (numpy or torch, [rows, cols] or [n]); None drops it."""
    cols = w.shape[1] if w.ndim == 2 else 1
    rg = shard_ranges(name, w.shape[0], cols, shape, size, rank, ffn_group)
    if rg is None:
        return None
    r0, r1, c0, c1 = rg
    return w[r0:r1] if w.ndim == 1 else w[r0:r1, c0:c1]


def shard_block(name: str, b, shape, size: int, rank: int, ffn_group: int):
    """Shard a stored ``.n730`` block (group-wise 0x42/0x44/0x48, or FP16) like
    ``shard``: rows, and columns at whole quant groups, re-packed into a block
    of the same format; None drops it."""
    from .formats import GROUPED, RawBlock
    if size == 1:
        return b
    rg = shard_ranges(name, b.rows, b.cols, shape, size, rank, ffn_group)
    if rg is None:
        return None
    r0, r1, c0, c1 = rg
    if b.prec_id == 16:
        w = np.frombuffer(b.payload, np.float16).reshape(b.rows, b.cols)[r0:r1, c0:c1]
        return RawBlock(b.layer_idx, 16, r1 - r0, c1 - c0, 1.0, 0.0, np.ascontiguousarray(w).tobytes(), 0)
    if b.prec_id not in GROUPED:
        raise ValueError(f"{name}: tensor-parallel loading needs group-wise or FP16 blocks (precision {b.prec_id})")
    bits = {0x42: 2, 0x44: 4, 0x48: 8}[b.prec_id]
    g, per = b.group_size, 8 // bits
    if c0 % g or (c1 - c0) % g:
        raise ValueError(f"{name}: column split {c0}:{c1} is not at group-{g} boundaries")
    codes = b.codes.reshape(b.rows, b.cols // per)[r0:r1, c0 // per:c1 // per]
    s16 = b.scales16[r0:r1, c0 // g:c1 // g]
    z16 = b.zeros16[r0:r1, c0 // g:c1 // g]
    payload = b"".join(np.ascontiguousarray(a).tobytes() for a in (codes, s16, z16))
    return RawBlock(b.layer_idx, b.prec_id, r1 - r0, c1 - c0, 1.0, 0.0, payload, g)


def init_engine_comm(engine, rank: int, size: int, group=None, map_peers: bool = True):
    """Share rank 0's NCCL id over torch.distributed (any backend) and join the engine's
    communicator; with ``map_peers`` (ranks on one node) also exchange the exchange-region
    handles and map every rank's region: the persistent batch-1 decode kernel pushes its
    row-split sums there, and with tp_allreduce=0 so does the one-shot allreduce.  Without it
    every step uses the per-op kernels and NCCL.

    First every rank's (rank, size, engine configuration) is all-gathered over the process
    group: NCCL's communicator set-up has no timeout, so a rank that never arrives (or joins
    with another tensor-parallel configuration) is caught here, where the process group's
    timeout ends the wait with an error (RuntimeError), before any rank enters NCCL.
    Configurations that differ raise ValueError on every rank."""
    import torch.distributed as dist
    sig = (rank, size, engine.tp_signature())
    sigs = [None] * size
    dist.all_gather_object(sigs, sig, group=group)
    if [s[0] for s in sigs] != list(range(size)) or any(s[1] != size for s in sigs):
        raise ValueError(f"tensor-parallel ranks disagree on rank numbering / size: {[s[:2] for s in sigs]}")
    bad = [s[0] for s in sigs if s[2] != sigs[0][2]]
    if bad:
        raise ValueError(f"tensor-parallel ranks {bad} were configured differently from rank 0: "
                         f"{sigs[bad[0]][2]} vs {sigs[0][2]}")
    ids = [engine.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0, group=group)
    engine.tp_init(ids[0], rank, size)
    if map_peers:
        handles = [None] * size
        dist.all_gather_object(handles, engine.tp_ipc_handle(), group=group)
        engine.tp_ipc_open(b"".join(handles), size)
        dist.barrier(group=group)  # every region is mapped and zeroed before the first push


def ffn_group_of(pmap_fn, down_name: str, default: int = 128) -> int:
    """Quant group of down_proj's columns (the FFN split unit) from a precision map entry."""
    spec = pmap_fn(down_name)
    if spec.startswith("INT2G") or spec.startswith("INT4G") or spec.startswith("INT8G"):
        digits = "".join(ch for ch in spec[5:] if ch.isdigit())
        return int(digits) if digits else default
    return default


__all__ = ["span", "check_shape", "lm_head_split", "local_shape", "shard_ranges", "shard", "shard_block",
           "init_engine_comm", "ffn_group_of"]
