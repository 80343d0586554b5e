"""Python wrapper of the C model engine (include/n730_cuda.h, "whole-model engine").

Weights enter as packed ``QWeight`` handles (``qweight_from_block`` for
``.n730`` blocks, ``qweight_from_device`` for device buffers); the engine
fuses q|k|v and gate/up, owns the paged KV cache, and runs prefill and the
graph-replayed decode step.  Torch is not required here.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from .formats import RawBlock, GROUPED, read_block, read_header

W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_EMBED, W_LMHEAD = range(9)
V_INPUT_NORM, V_POST_NORM, V_Q_BIAS, V_K_BIAS, V_V_BIAS, V_O_BIAS, V_GATE_BIAS, V_UP_BIAS, V_DOWN_BIAS, \
    V_FINAL_NORM = range(10)

PROJ_SLOTS = {"self_attn.q_proj": W_Q, "self_attn.k_proj": W_K, "self_attn.v_proj": W_V,
              "self_attn.o_proj": W_O, "mlp.gate_proj": W_GATE, "mlp.up_proj": W_UP,
              "mlp.down_proj": W_DOWN}
BIAS_SLOTS = {"self_attn.q_proj": V_Q_BIAS, "self_attn.k_proj": V_K_BIAS, "self_attn.v_proj": V_V_BIAS,
              "self_attn.o_proj": V_O_BIAS, "mlp.gate_proj": V_GATE_BIAS, "mlp.up_proj": V_UP_BIAS,
              "mlp.down_proj": V_DOWN_BIAS}


class N730ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float)] + \
               [(n, C.c_int32) for n in ("max_ctx", "max_batch", "page_size", "max_prefill", "tie_embeddings",
                                         "tp_rank", "tp_size", "use_graphs", "use_pdl", "exact_gemv",
                                         "per_op_decode", "stream_depth", "ffn_fuse", "tp_allreduce",
                                         "kv_pool_pages")]


def _sigs(lib):
    if getattr(lib, "_model_sigs", False):
        return lib
    vp, i32, i64p = C.c_void_p, C.c_int32, C.POINTER(C.c_int64)
    lib.n730_model_create.argtypes = [C.POINTER(N730ModelConfig), C.POINTER(vp)]
    lib.n730_model_create.restype = i32
    lib.n730_model_destroy.argtypes = [vp]
    lib.n730_model_destroy.restype = None
    lib.n730_model_set_qweight.argtypes = [vp, i32, i32, vp]
    lib.n730_model_set_qweight.restype = i32
    lib.n730_model_set_vector.argtypes = [vp, i32, i32, vp, i32, i32]
    lib.n730_model_set_vector.restype = i32
    for f in ("n730_model_finalize", "n730_model_reset"):
        getattr(lib, f).argtypes = [vp]
        getattr(lib, f).restype = i32
    lib.n730_model_seq_len.argtypes = [vp, i32]
    lib.n730_model_seq_len.restype = i32
    lib.n730_model_set_seq_len.argtypes = [vp, i32, i32]
    lib.n730_model_set_seq_len.restype = i32
    lib.n730_model_forward.argtypes = [vp, i32, vp, i32, vp]
    lib.n730_model_forward.restype = i32
    lib.n730_model_decode.argtypes = [vp, vp, i32, vp]
    lib.n730_model_decode.restype = i32
    lib.n730_host_alloc.argtypes = [C.c_size_t, C.POINTER(vp)]
    lib.n730_host_alloc.restype = i32
    lib.n730_host_free.argtypes = [vp]
    lib.n730_host_free.restype = i32
    lib.n730_model_decode_sample.argtypes = [vp, vp, i32, C.c_float, C.c_float, C.c_uint64, vp, vp]
    lib.n730_model_decode_sample.restype = i32
    lib.n730_model_decode_device.argtypes = [vp, vp, i32, vp, vp]
    lib.n730_model_decode_device.restype = i32
    lib.n730_model_info.argtypes = [vp, i64p]
    lib.n730_model_info.restype = i32
    lib.n730_model_stream.argtypes = [vp]
    lib.n730_model_stream.restype = vp
    lib.n730_tp_unique_id.argtypes = [vp]
    lib.n730_tp_unique_id.restype = i32
    lib.n730_model_tp_init.argtypes = [vp, vp, i32, i32]
    lib.n730_model_tp_init.restype = i32
    lib.n730_model_tp_ipc_handle.argtypes = [vp, vp]
    lib.n730_model_tp_ipc_handle.restype = i32
    lib.n730_model_tp_ipc_open.argtypes = [vp, vp, i32]
    lib.n730_model_tp_ipc_open.restype = i32
    lib.n730_model_run_step_kernel.argtypes = [vp, vp]
    lib.n730_model_run_step_kernel.restype = i32
    lib.n730_model_run_linear.argtypes = [vp, i32, i32, vp, i32, vp, vp]
    lib.n730_model_run_linear.restype = i32
    lib.n730_model_linear_bytes.argtypes = [vp, i32, i32, i32]
    lib.n730_model_linear_bytes.restype = C.c_int64
    lib.n730_model_seq_release.argtypes = [vp, i32]
    lib.n730_model_seq_release.restype = i32
    lib.n730_model_seq_move.argtypes = [vp, i32, i32]
    lib.n730_model_seq_move.restype = i32
    lib.n730_model_kv_pages.argtypes = [vp, C.POINTER(i32), C.POINTER(i32)]
    lib.n730_model_kv_pages.restype = i32
    lib.n730_model_trace_step.argtypes = [vp, vp, vp, C.c_int64, vp, C.POINTER(i32), C.POINTER(i32)]
    lib.n730_model_trace_step.restype = i32
    lib._model_sigs = True
    return lib


def qweight_from_block(b: RawBlock):
    """Register a .n730 block's packed codes on the current device."""
    lib = _lib.cuda()
    out = C.c_void_p()
    payload = np.frombuffer(b.payload, np.uint8)
    if b.prec_id in GROUPED:
        s16 = np.ascontiguousarray(b.scales16)
        z16 = np.ascontiguousarray(b.zeros16)
        rc = lib.n730_qweight_create(b.prec_id, b.rows, b.cols, b.group_size, 1.0, 0.0,
                                     payload.ctypes.data_as(C.c_void_p), s16.ctypes.data_as(C.c_void_p),
                                     z16.ctypes.data_as(C.c_void_p), 0, None, C.byref(out))
    else:
        rc = lib.n730_qweight_create(b.prec_id, b.rows, b.cols, 0, b.scale, b.zero_point,
                                     payload.ctypes.data_as(C.c_void_p), None, None, 0, None, C.byref(out))
    _lib.check(rc, "qweight_create")
    return out


def qweight_from_device(prec_id, rows, cols, group, d_codes, d_s16=None, d_z16=None, scale=1.0, zero=0.0,
                        stream=None):
    lib = _lib.cuda()
    out = C.c_void_p()
    _lib.check(lib.n730_qweight_create(prec_id, rows, cols, group, scale, zero, C.c_void_p(d_codes),
                                       C.c_void_p(d_s16) if d_s16 else None, C.c_void_p(d_z16) if d_z16 else None,
                                       1, C.c_void_p(stream) if stream else None, C.byref(out)),
               "qweight_create")
    return out


@dataclass
class ModelShape:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    tie_embeddings: bool = False


class _PinnedBlock:
    """Page-locked host memory from n730_host_alloc, freed when the last array viewing it goes."""

    def __init__(self, lib, nbytes: int):
        self.lib, self.ptr = lib, C.c_void_p()
        _lib.check(lib.n730_host_alloc(nbytes, C.byref(self.ptr)), "host_alloc")

    def __del__(self):
        try:
            if self.ptr:
                self.lib.n730_host_free(self.ptr)
        except Exception:
            pass


def _pinned_f32(lib, n: int) -> np.ndarray:
    """A float32 array of n zeros in page-locked memory: n730_model_decode copies the logits
    straight into it.  The array keeps the block alive (numpy base -> ctypes array -> block)."""
    blk = _PinnedBlock(lib, n * 4)
    arr = (C.c_float * n).from_address(blk.ptr.value)
    arr._block = blk
    out = np.frombuffer(arr, np.float32)
    out[:] = 0.0
    return out


class Engine:
    """Owns one C model; all methods raise ``N730Error`` on a negative code."""

    def __init__(self, shape: ModelShape, max_ctx: int = 4096, max_batch: int = 1, page_size: int = 64,
                 max_prefill: int = 512, use_graphs: bool = True, use_pdl: bool = True,
                 tp_rank: int = 0, tp_size: int = 1, exact_gemv: bool = False, per_op_decode: int = 0,
                 stream_depth: int = 0, ffn_fuse: int = 0, tp_allreduce: int = 1, kv_pool_pages: int = 0):
        self.lib = _sigs(_lib.cuda())
        self.shape = shape
        c = N730ModelConfig(shape.hidden, shape.layers, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn,
                            shape.vocab, shape.rms_eps, shape.rope_theta, max_ctx, max_batch, page_size,
                            max_prefill, int(shape.tie_embeddings), tp_rank, tp_size, int(use_graphs),
                            int(use_pdl), int(exact_gemv), int(per_op_decode), int(stream_depth), int(ffn_fuse),
                            int(tp_allreduce), int(kv_pool_pages))
        self.cfg = c
        self.h = C.c_void_p()
        _lib.check(self.lib.n730_model_create(C.byref(c), C.byref(self.h)), "model_create")
        self.max_batch = max_batch
        self.max_ctx = max_ctx
        self._logits = _pinned_f32(self.lib, max_batch * shape.vocab).reshape(max_batch, shape.vocab)

    def set_qweight(self, layer: int, slot: int, qw):
        _lib.check(self.lib.n730_model_set_qweight(self.h, layer, slot, qw), "model_set_qweight")

    def set_vector(self, layer: int, slot: int, v):
        v = np.ascontiguousarray(v, np.float32)
        _lib.check(self.lib.n730_model_set_vector(self.h, layer, slot, v.ctypes.data_as(C.c_void_p), v.size, 0),
                   "model_set_vector")

    def finalize(self):
        _lib.check(self.lib.n730_model_finalize(self.h), "model_finalize")

    def reset(self):
        _lib.check(self.lib.n730_model_reset(self.h), "model_reset")

    def seq_len(self, seq: int = 0) -> int:
        return _lib.check(self.lib.n730_model_seq_len(self.h, seq), "model_seq_len")

    def set_seq_len(self, seq: int, n: int):
        _lib.check(self.lib.n730_model_set_seq_len(self.h, seq, n), "model_set_seq_len")

    def forward(self, token_ids, seq: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, np.int32).reshape(-1)
        out = np.empty(self.shape.vocab, np.float32)
        _lib.check(self.lib.n730_model_forward(self.h, seq, ids.ctypes.data_as(C.c_void_p), ids.size,
                                               out.ctypes.data_as(C.c_void_p)), "model_forward")
        return out

    def seq_release(self, seq: int):
        _lib.check(self.lib.n730_model_seq_release(self.h, seq), "model_seq_release")

    def seq_move(self, dst: int, src: int):
        _lib.check(self.lib.n730_model_seq_move(self.h, dst, src), "model_seq_move")

    def kv_pages(self):
        """(free, total) pages of the KV pool."""
        f, t = C.c_int32(), C.c_int32()
        _lib.check(self.lib.n730_model_kv_pages(self.h, C.byref(f), C.byref(t)), "model_kv_pages")
        return f.value, t.value

    def decode(self, tokens) -> np.ndarray:
        ids = np.ascontiguousarray(tokens, np.int32).reshape(-1)
        B = ids.size
        _lib.check(self.lib.n730_model_decode(self.h, ids.ctypes.data_as(C.c_void_p), B,
                                              self._logits.ctypes.data_as(C.c_void_p)), "model_decode")
        return self._logits[:B]

    def decode_sample(self, tokens, temperature: float = 0.7, top_p: float = 0.9, seed: int = 0,
                      return_u: bool = False):
        """One decode step for sequences [0, len(tokens)) with the next tokens sampled on the GPU
        (n730_model_decode_sample): host ids in, next ids out (4 bytes per sequence)."""
        ids = np.ascontiguousarray(tokens, np.int32).reshape(-1)
        nxt = np.empty(ids.size, np.int32)
        u = np.empty(ids.size, np.float32)
        _lib.check(self.lib.n730_model_decode_sample(self.h, ids.ctypes.data_as(C.c_void_p), ids.size, temperature,
                                                     top_p, seed, nxt.ctypes.data_as(C.c_void_p),
                                                     u.ctypes.data_as(C.c_void_p)), "model_decode_sample")
        return (nxt, u) if return_u else nxt

    def decode_device(self, d_tokens: int, batch: int, d_logits: int, stream: int = 0):
        _lib.check(self.lib.n730_model_decode_device(self.h, C.c_void_p(d_tokens) if d_tokens else None, batch,
                                                     C.c_void_p(d_logits) if d_logits else None,
                                                     C.c_void_p(stream) if stream else None), "model_decode_device")

    def info(self) -> dict:
        a = (C.c_int64 * 16)()
        _lib.check(self.lib.n730_model_info(self.h, a), "model_info")
        return {"weight_bytes": a[0], "kv_bytes_per_pos": a[1], "kv_capacity_bytes": a[2], "n_split": a[3],
                "qkv_dim": a[4], "pages_per_seq": a[5], "persistent_decode": bool(a[7]),
                "embed_bytes": a[8], "streamed_bytes": a[9], "ffn_fused": bool(a[10]),
                "phase_table_global": bool(a[11]), "tp_plan_mismatch": bool(a[12]), "persistent_grid": a[13]}

    def tp_signature(self) -> tuple:
        """Configuration fields every tensor-parallel rank must share (its FFN share may differ:
        whole quantisation groups split unevenly, and tp_rank differs by definition)."""
        c = self.cfg
        return tuple(getattr(c, f) for f in ("hidden", "layers", "heads", "kv_heads", "head_dim", "vocab",
                                              "max_ctx", "max_batch", "page_size", "max_prefill",
                                              "tie_embeddings", "tp_size", "use_graphs", "use_pdl",
                                              "exact_gemv", "per_op_decode", "ffn_fuse", "tp_allreduce")) + \
            (round(float(c.rms_eps), 12), float(c.rope_theta))

    @staticmethod
    def tp_unique_id() -> bytes:
        """128-byte NCCL unique id (rank 0 makes it, every rank passes it to tp_init)."""
        buf = (C.c_uint8 * 128)()
        _lib.check(_sigs(_lib.cuda()).n730_tp_unique_id(buf), "tp_unique_id")
        return bytes(buf)

    def tp_init(self, id_bytes: bytes, rank: int, size: int):
        buf = (C.c_uint8 * 128).from_buffer_copy(id_bytes)
        _lib.check(self.lib.n730_model_tp_init(self.h, buf, rank, size), "model_tp_init")

    IPC_HANDLE_BYTES = 64

    def tp_ipc_handle(self) -> bytes:
        """This rank's exchange-region handle for the one-shot allreduce (after tp_init)."""
        buf = (C.c_uint8 * self.IPC_HANDLE_BYTES)()
        _lib.check(self.lib.n730_model_tp_ipc_handle(self.h, buf), "model_tp_ipc_handle")
        return bytes(buf)

    def tp_ipc_open(self, handles: bytes, size: int):
        """Map every rank's exchange region (handles concatenated in rank order)."""
        assert len(handles) == size * self.IPC_HANDLE_BYTES
        buf = (C.c_uint8 * len(handles)).from_buffer_copy(handles)
        _lib.check(self.lib.n730_model_tp_ipc_open(self.h, buf, size), "model_tp_ipc_open")

    def run_step_kernel(self, stream: int = 0):
        """Launch only the persistent decode kernel of a batch-1 step (timing hook)."""
        _lib.check(self.lib.n730_model_run_step_kernel(self.h, C.c_void_p(stream) if stream else None),
                   "model_run_step_kernel")

    def trace_step(self, stream: int = 0):
        """One persistent-kernel launch with per-phase timing: (times [6 n_phases + 1, grid] ns,
        kinds [n_phases]); see include/n730_cuda.h."""
        st = C.c_void_p(stream) if stream else None
        npz, grid = C.c_int32(), C.c_int32()
        _lib.check(self.lib.n730_model_trace_step(self.h, st, None, 0, None, C.byref(npz), C.byref(grid)),
                   "model_trace_step")
        times = np.zeros((6 * npz.value + 1, grid.value), np.uint64)
        kinds = np.zeros(npz.value, np.int8)
        _lib.check(self.lib.n730_model_trace_step(self.h, st, times.ctypes.data_as(C.c_void_p), times.size,
                                                  kinds.ctypes.data_as(C.c_void_p), C.byref(npz), C.byref(grid)),
                   "model_trace_step")
        return times, kinds

    def run_linear(self, layer: int, which: int, d_x: int, batch: int, d_y: int, stream: int = 0):
        _lib.check(self.lib.n730_model_run_linear(self.h, layer, which, C.c_void_p(d_x), batch, C.c_void_p(d_y),
                                                  C.c_void_p(stream) if stream else None), "model_run_linear")

    def linear_bytes(self, layer: int, which: int, batch: int = 1) -> int:
        return int(self.lib.n730_model_linear_bytes(self.h, layer, which, batch))

    @property
    def stream(self) -> int:
        return self.lib.n730_model_stream(self.h) or 0

    def close(self):
        if self.h:
            self.lib.n730_model_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_tensors(engine: Engine, named_blocks, norms: dict | None = None):
    """Hand a model's tensors to the engine by HF name.

    ``named_blocks``: iterable of (name, RawBlock) for every 2-D weight and
    1-D FP16 bias / norm vector; ``norms``: name -> fp32 vector, overriding
    norm blocks of the file (absent norms default to ones, the reference's
    identity fallback, inference.py:398-406).
    """
    norms = dict(norms or {})
    for name, b in named_blocks:
        if name == "model.embed_tokens.weight":
            engine.set_qweight(-1, W_EMBED, qweight_from_block(b))
        elif name == "lm_head.weight":
            engine.set_qweight(-1, W_LMHEAD, qweight_from_block(b))
        elif name.endswith("norm.weight") and b.prec_id == 16 and name not in norms:
            norms[name] = np.frombuffer(b.payload, np.float16).astype(np.float32)
        elif name.startswith("model.layers."):
            rest = name[len("model.layers."):]
            i, _, tail = rest.partition(".")
            layer = int(i)
            base, _, kind = tail.rpartition(".")
            if kind == "weight" and base in PROJ_SLOTS:
                engine.set_qweight(layer, PROJ_SLOTS[base], qweight_from_block(b))
            elif kind == "bias" and base in BIAS_SLOTS:
                if b.prec_id != 16:
                    raise ValueError(f"bias {name} must be stored FP16 (as the reference converter writes it)")
                engine.set_vector(layer, BIAS_SLOTS[base], np.frombuffer(b.payload, np.float16).astype(np.float32))
    for name, v in norms.items():
        if name == "model.norm.weight":
            engine.set_vector(-1, V_FINAL_NORM, v)
        elif name.startswith("model.layers.") and name.endswith("input_layernorm.weight"):
            engine.set_vector(int(name.split(".")[2]), V_INPUT_NORM, v)
        elif name.startswith("model.layers.") and name.endswith("post_attention_layernorm.weight"):
            engine.set_vector(int(name.split(".")[2]), V_POST_NORM, v)

def _weight_slot(name: str):
    """(layer, slot) of a 2-D weight tensor the engine holds, else None."""
    if name == "model.embed_tokens.weight":
        return -1, W_EMBED
    if name == "lm_head.weight":
        return -1, W_LMHEAD
    if name.startswith("model.layers.") and name.endswith(".weight"):
        i, _, tail = name[len("model.layers."):].partition(".")
        base = tail.rpartition(".")[0]
        if base in PROJ_SLOTS:
            return int(i), PROJ_SLOTS[base]
    return None


def qweights_from_file(path, offsets, stream=None):
    """Packed weights of the blocks at `offsets` through the native loader (n730_qweight_load_blocks:
    pread into pinned staging, asynchronous copies to HBM); returns handles and bytes read."""
    lib = _lib.cuda()
    n = len(offsets)
    offs = np.ascontiguousarray(offsets, np.int64)
    out = (C.c_void_p * max(n, 1))()
    nbytes = C.c_int64()
    _lib.check(lib.n730_qweight_load_blocks(str(path).encode(), n, offs.ctypes.data_as(C.c_void_p),
                                            C.c_void_p(stream) if stream else None, out, C.byref(nbytes)),
               "qweight_load_blocks")
    return [C.c_void_p(out[i]) for i in range(n)], int(nbytes.value)


def load_file(engine: Engine, path, norms: dict | None = None) -> dict:
    """Hand a ``.n730`` file's tensors to the engine: every 2-D weight through the native block
    loader in one call, 1-D vectors (q/k/v biases, FP16 norm weights) read in Python.  A
    per-tensor block the native loader leaves to Python (the reference's odd-length INT4/INT2
    packing) is read by ``read_block``.  Returns {"native_blocks", "native_bytes", "python_blocks"}."""
    hdr = read_header(path)
    big, small = [], []
    for e in hdr["seek_table"]:
        slot = _weight_slot(e["layer_name"])
        (big if slot else small).append((e["layer_name"], e["file_offset"], slot))
    stats = {"native_blocks": 0, "native_bytes": 0, "python_blocks": len(small)}
    try:
        handles, nbytes = qweights_from_file(path, [off for _, off, _ in big])
        stats.update(native_blocks=len(big), native_bytes=nbytes)
    except _lib.N730Error as ex:
        if ex.code != -14:
            raise
        handles = []
        for _, off, _ in big:  # one by one, the blocks the native reader declines through Python
            try:
                h, nb = qweights_from_file(path, [off])
                handles.append(h[0])
                stats["native_blocks"] += 1
                stats["native_bytes"] += nb
            except _lib.N730Error as e2:
                if e2.code != -14:
                    raise
                handles.append(qweight_from_block(read_block(path, off)))
                stats["python_blocks"] += 1
    for (_, _, (layer, slot)), h in zip(big, handles):
        engine.set_qweight(layer, slot, h)
    load_tensors(engine, [(name, read_block(path, off)) for name, off, _ in small], norms)
    return stats
