"""Benchmark: decode tok/s at Qwen2-7B shape, INT4 g128, batch 1, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--ctx C]
    python bench.py --impl reference ...          # the reference's CPU path

Workload (one "step" = one decode step of the whole model for B sequences):
a Qwen2-7B-shape decoder (hidden 3584, 28 layers, 28/4 heads, head_dim 128,
FFN 18944, vocab 152064), random-init N(0, 0.02) weights quantised on the GPU
to INT4 with group 128 (fp16 scale + zero), lm_head and embeddings included;
a 2048-token prompt of uniform-random ids is prefilled (untimed), then K
decode steps run at context 2048.. with the fp16 paged KV cache.

* ``value``: tok/s with token ids and logits resident in HBM (device-side
  decode graph), CUDA events on the model's stream.  Weights (3.76 GB) exceed
  L2 (126 MB), so every step streams them from HBM; no L2 flush is needed.
* ``e2e``: the same through the host C-ABI call ``n730_model_decode`` with host
  token ids in and host fp32 logits out (copies inside the timed region);
  ``e2e.sampled_ids_out`` times ``n730_model_decode_sample`` (the next ids
  sampled on the GPU, temperature 0.7 / top-p 0.9) beside it.
* ``roofline``: the dominant kernel, the persistent decode kernel (one
  cooperative launch runs all 28 layers and the lm_head of a batch-1 step),
  timed alone with CUDA events on the model's stream; algorithmic bytes per
  launch = every packed weight it streams (q|k|v, o, gate|up, down per layer
  and the lm_head: INT4 codes + fp16 scale/zero) + the fp16 K/V it reads
  (28 layers x 4 KV heads x 128 x 2 x 2 B per cached position), against the
  measured HBM peak in MEASURED_PEAKS.json.  For batch > 1 (per-op kernels)
  the gate|up dequant-GEMV is timed alone instead.
* ``cpu_baseline``: the reference's CPU path for whole decode tokens of this
  shape (its own n730core read+dequant, built from its source, on a reader
  thread pool, plus numpy fp32 GEMVs and the attention over an fp32 KV
  cache); per-tensor INT4 stands in for g128 (the reference has no
  group-wise format).

Launched by torchrun (any N, including 1): the Qwen2-72B-shape INT4 g128
model decodes at batch 1 tensor parallel over the N ranks (q/k/v, gate/up
column-split, o_proj/down_proj row-split with one exchange each, vocab-split
lm_head): one model, strong scaling, time the max over ranks.  So the
multi-GPU scaling points measure tensor-parallel decode of one 72B model, and
their N = 1 point is that model on one GPU.  ``--workload resident`` under
torchrun runs independent 7B replicas instead.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

SHAPE_NAME = "qwen2-7b"
METRIC = "decode tok/s at Qwen2-7B-shape INT4; dequant-GEMV HBM GB/s vs ~8 TB/s peak"
TP_METRIC = "decode tok/s, Qwen2-72B-shape INT4 g128, tensor parallel"


def _under_torchrun() -> bool:
    return "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ


def _tp_workload(a) -> bool:
    """The 72B tensor-parallel workload: asked for, or (by default) whenever torchrun launched us,
    at any N: the multi-GPU scaling points measure tensor-parallel decode of one 72B model."""
    return a.workload == "tp72b" or (a.workload == "auto" and _under_torchrun())


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=2048, help="prompt length prefilled before decoding")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small profiling cases)")
    ap.add_argument("--vocab", type=int, default=0, help="phases workload: override the vocabulary (profiling cases)")
    ap.add_argument("--linear-shape", default="4096x4096", help="linear / gemm workload: rows x cols of W")
    ap.add_argument("--tokens", type=int, default=512, help="gemm workload: tokens per call")
    ap.add_argument("--prefill-chunk", type=int, default=2048, help="tokens per prefill call (engine max_prefill)")
    ap.add_argument("--copies", type=int, default=0,
                    help="linear workload: weight copies rotated through (default: > 4x L2 of bytes)")
    ap.add_argument("--tp-allreduce", type=int, default=1, choices=[0, 1],
                    help="tp72b decode row-split sums: 0 one-shot over NVLink peer memory, 1 NCCL")
    ap.add_argument("--ffn-fuse", type=int, default=0, choices=[-1, 0, 1],
                    help="persistent decode FFN: 0 auto, 1 one fused phase, -1 two GEMV phases")
    ap.add_argument("--per-op", action="store_true",
                    help="batch-1 decode through the per-op kernels instead of the persistent kernel")
    ap.add_argument("--model", default=SHAPE_NAME, choices=["qwen2-7b", "qwen2-0.5b"],
                    help="resident workload: model shape")
    ap.add_argument("--pmap", default="int4_g128", choices=["int4_g128", "mixed_05b"],
                    help="resident workload: precision map (mixed_05b: INT8 attention, INT4 g128 FFN, fp16 tied "
                         "embedding/lm_head)")
    ap.add_argument("--workload", default="auto",
                    choices=["auto", "resident", "streamed", "tp72b", "linear", "gemm", "phases"],
                    help="auto: tp72b when launched by torchrun (any N), else resident (the 7B headline); "
                         "resident: the model resident in HBM (N ranks: independent replicas); "
                         "streamed: 7B aggressive mixed quant (FFN INT2 g64, attention INT4 g128, lm_head INT8 "
                         "per channel), layer weights in pinned host memory, 2-layer prefetch, 1024-token prompt; "
                         "tp72b: Qwen2-72B shape INT4 g128 split over the N ranks (tensor parallel, strong scaling); "
                         "phases: per-phase timing of the persistent decode kernel")
    return ap.parse_args()


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Clocks and throttle reasons sampled DURING the timed region.

    NVML is polled from a thread every millisecond (a short timed region of a few
    steps still gets samples; reading clocks changes no setting); where NVML is
    not importable, ``nvidia-smi -lms 20`` is read instead.  Only samples taken
    between ``__enter__`` and ``__exit__`` are summarised."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.p = None
        self.th = None
        self.rows = []        # (time, sm_mhz, sm_max_mhz, [reason names])
        self.stop = False

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll_nvml(self, nv, h):
        bits = [(nv.nvmlClocksEventReasonHwSlowdown, "hw_slowdown"),
                (nv.nvmlClocksEventReasonHwThermalSlowdown, "hw_thermal_slowdown"),
                (nv.nvmlClocksEventReasonSwThermalSlowdown, "sw_thermal_slowdown"),
                (nv.nvmlClocksEventReasonSwPowerCap, "sw_power_cap")]
        smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((time.time(), int(sm), int(smax), [n for b, n in bits if r & b]))
            except Exception:
                return
            time.sleep(0.001)

    def _read_smi(self):
        for line in self.p.stdout:
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9 and f[1].isdigit():
                self.rows.append((time.time(), int(f[1]), int(f[2]),
                                  [n for n, v in zip(self.NAMES, f[5:9]) if v.lower() == "active"]))

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.th = threading.Thread(target=self._poll_nvml, args=(nv, h), daemon=True)
        except Exception:
            try:
                self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                           "--format=csv,noheader,nounits", "-lms", "20"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.th = threading.Thread(target=self._read_smi, daemon=True)
            except Exception:
                self.th = None
        if self.th is not None:
            self.th.start()
            time.sleep(0.3 if self.p else 0.01)  # let the sampler start before the timed region
        self.t_start = time.time()
        return self

    def __exit__(self, *a):
        self.t_end = time.time()
        self.stop = True
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
        if self.th is not None:
            self.th.join(timeout=2)

    def summary(self):
        rows = [r for r in self.rows if self.t_start <= r[0] <= self.t_end]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({n for r in rows for n in r[3]})
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": rows[0][2],
                "reasons": reasons, "samples": len(rows), "source": "nvml" if self.p is None else "nvidia-smi"}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU path for a whole decode token
# ---------------------------------------------------------------------------
def _host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuReferenceDecoder:
    """The reference's CPU decode path for one token of a Qwen2-shape decoder.

    Per layer, the seven projection weights are read and dequantised from a
    ``.n730`` file by the reference core's ``n730_read_layer`` (built from its
    own source by oracle/Makefile; per-tensor INT4, the reference has no
    group-wise format), as its layer scheduler does (``scheduler.py:198-230``),
    then applied as numpy fp32 ``W @ x`` (``inference.py:668``, ``scheduler.py:324``)
    around the oracle's RMSNorm, RoPE, GQA attention over an fp32 KV cache of
    ``ctx`` positions and SwiGLU; then the final norm and the lm_head (read,
    dequantised, GEMV).  Reads run on a pool of ``threads`` workers, each with its
    own file handle (a handle is not thread-safe, ``scheduler.py:242-244``),
    up to ``ahead`` tensors ahead of the layer being computed; the GEMVs use
    OpenBLAS's threads.  The file holds one layer's seven tensors and the
    lm_head; every layer reads the same seven blocks (same sizes, same work;
    the codes are uniform random bytes: dequant and GEMV cost do not depend on
    the values).
    """

    def __init__(self, shape, ctx, threads=None, ahead=16, seed=0):
        import ctypes as C
        import struct
        import tempfile
        from concurrent.futures import ThreadPoolExecutor

        core_so = REPO / "oracle" / "_ref" / "n730core.so"
        if not core_so.exists():
            raise FileNotFoundError("oracle/_ref/n730core.so missing (built by __graft_entry__.build)")
        self.C = C
        core = C.CDLL(str(core_so))
        core.n730_open.argtypes = [C.c_char_p]
        core.n730_open.restype = C.c_int64
        core.n730_read_layer.argtypes = [C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        core.n730_read_layer.restype = C.c_int32
        core.n730_close.argtypes = [C.c_int64]
        self.core = core
        self.shape = s = shape
        self.ctx = ctx
        h, q, kv, f = s.hidden, s.heads * s.head_dim, s.kv_heads * s.head_dim, s.ffn
        self.tensors = [(q, h), (kv, h), (kv, h), (h, q), (f, h), (f, h), (h, f), (s.vocab, h)]
        rng = np.random.default_rng(seed)
        tmp = tempfile.NamedTemporaryFile(suffix=".n730", delete=False, dir=os.environ.get("TMPDIR"))
        self.path = tmp.name
        self.offs = []
        with open(self.path, "wb") as fo:
            fo.write(b"N730\x00\x01\x00\x00" + struct.pack(">II", 1, 2) + b"{}")
            fo.write(bytes(4096 - 18))
            for i, (r, c) in enumerate(self.tensors):
                codes = rng.integers(0, 256, (r * c + 1) // 2, dtype=np.uint8)
                self.offs.append(fo.tell())
                fo.write(struct.pack(">4sIBIIffi", b"LYR\x00", i, 4, r, c, 0.0025, 8.0, codes.size))
                codes.tofile(fo)
                fo.write(bytes((-(29 + codes.size)) % 4096))
        self.threads = threads or _host_cores()
        self.ahead = ahead
        self.handles = [core.n730_open(self.path.encode()) for _ in range(self.threads)]
        assert all(hd >= 0 for hd in self.handles), self.handles
        import threading
        self._tls = threading.local()
        self._hid = iter(range(self.threads))
        self._hlock = threading.Lock()
        self.pool = ThreadPoolExecutor(self.threads)
        from oracle.model import rope_table
        self.cos, self.sin = rope_table(ctx + 64, s.head_dim, s.rope_theta)
        self.kc = [rng.normal(0, 1, (ctx, kv)).astype(np.float32) for _ in range(s.layers)]
        self.vc = [rng.normal(0, 1, (ctx, kv)).astype(np.float32) for _ in range(s.layers)]
        self.bias = [rng.normal(0, 0.02, q + 2 * kv).astype(np.float32) for _ in range(s.layers)]
        self.ones = np.ones(h, np.float32)
        self.x0 = rng.normal(0, 1, h).astype(np.float32)
        try:
            import threadpoolctl
            self.blas = max(i.get("num_threads", 1) for i in threadpoolctl.threadpool_info())
        except Exception:
            self.blas = os.cpu_count() or 1

    def _handle(self):
        hd = getattr(self._tls, "h", None)
        if hd is None:
            with self._hlock:
                hd = self._tls.h = self.handles[next(self._hid)]
        return hd

    def _read(self, k):
        C = self.C
        r, c = self.tensors[k]
        buf = np.empty(r * c, np.float32)
        ro, co, po = C.c_int32(), C.c_int32(), C.c_int32()
        rc = self.core.n730_read_layer(self._handle(), self.offs[k], buf.ctypes.data, C.byref(ro), C.byref(co),
                                       C.byref(po))
        if rc != 0:
            raise RuntimeError(f"n730_read_layer failed: {rc}")
        return buf.reshape(r, c)

    def step(self):
        """One decode token at position ``ctx`` (the cache is not extended: every step is the same work)."""
        from collections import deque
        from oracle.model import apply_rope, attention, rms_norm, swiglu
        s = self.shape
        q_dim, kv_dim = s.heads * s.head_dim, s.kv_heads * s.head_dim
        order = [(l, k) for l in range(s.layers) for k in range(7)] + [(s.layers, 7)]
        pend = deque()
        nxt = 0

        def fill():
            nonlocal nxt
            while nxt < len(order) and len(pend) < self.ahead:
                pend.append(self.pool.submit(self._read, order[nxt][1]))
                nxt += 1

        def take():
            fill()
            w = pend.popleft().result()
            fill()
            return w

        x = self.x0.copy()
        for l in range(s.layers):
            hn = rms_norm(x[None], self.ones, s.rms_eps)[0]
            qkv = np.concatenate([take() @ hn, take() @ hn, take() @ hn]) + self.bias[l]
            qv = apply_rope(qkv[None, :q_dim], s.heads, s.head_dim, self.ctx, self.cos, self.sin)
            kv = apply_rope(qkv[None, q_dim:q_dim + kv_dim], s.kv_heads, s.head_dim, self.ctx, self.cos, self.sin)
            ks = np.concatenate([self.kc[l], kv])
            vs = np.concatenate([self.vc[l], qkv[None, q_dim + kv_dim:]])
            a = attention(qv, ks, vs, s.heads, s.kv_heads, s.head_dim, self.ctx)[0]
            x = x + take() @ a
            h2 = rms_norm(x[None], self.ones, s.rms_eps)[0]
            g, u = take() @ h2, take() @ h2
            x = x + take() @ swiglu(g, u)
        last = rms_norm(x[None], self.ones, s.rms_eps)[0]
        return take() @ last

    def close(self):
        self.pool.shutdown()
        for hd in self.handles:
            self.core.n730_close(hd)
        os.unlink(self.path)


def run_reference(a):
    world, rank, _ = _dist()
    if rank != 0:
        return
    from n730_b200.synthetic import SHAPES
    tp72 = _tp_workload(a)
    shape = SHAPES["qwen2-72b" if tp72 else SHAPE_NAME]
    if a.layers:
        shape = dataclasses.replace(shape, layers=a.layers)
    cs = CpuReferenceDecoder(shape, a.ctx)
    t0 = time.perf_counter()
    cs.step()
    t_first = time.perf_counter() - t0
    # every step is one whole token; the step count is capped so the arm ends within ~2 minutes
    steps = max(1, min(a.steps, int(120.0 / max(t_first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(steps):
        cs.step()
    t = (time.perf_counter() - t0) / steps
    cs.close()
    v = a.batch / t
    name = "qwen2-72b" if tp72 else "qwen2-7b"
    sample = (f"whole {name}-shape decode tokens at context {a.ctx} ({steps} timed, 1 warm-up): {shape.layers} "
              f"layers x 7 reference n730_read_layer reads (per-tensor INT4) on {cs.threads} reader threads + numpy "
              f"fp32 GEMVs on {cs.blas} OpenBLAS threads, attention over an fp32 KV cache, final norm + lm_head")
    out = {"impl": "reference", "metric": TP_METRIC if tp72 else METRIC, "value": round(v, 4), "unit": "tok/s",
           "n_gpus": a.gpus, "steps": steps, "warmup": 1, "ms_per_step": round(t * 1000, 1),
           "higher_is_better": True, "scaling": "strong" if tp72 else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic",
           "config": {"workload": f"{name}-shape decoder ({shape.layers} layers), INT4 (per-tensor: the reference "
                                  "has no group-wise format), batch 1 decode step on the host CPU (the reference "
                                  "has no tensor parallelism: one host at every N)",
                      "batch": a.batch, "ctx": a.ctx, "steps_requested": a.steps, "warmup_requested": a.warmup},
           "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": _host_cores(), "kind": "reference",
                            "blas_threads": cs.blas, "reader_threads": cs.threads, "sample": sample},
           "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(a):
    import torch
    world, rank, local = _dist()
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(0)
    from n730_b200.engine import Engine
    from n730_b200.synthetic import SHAPES, build_on_device
    shape = SHAPES[a.model]
    if a.layers:
        shape = dataclasses.replace(shape, layers=a.layers)
    headline = a.model == SHAPE_NAME and a.pmap == "int4_g128"
    B, ctx = a.batch, a.ctx
    max_ctx = ctx + 3 * (a.warmup + a.steps) + 64  # device-side steps, then the two e2e passes
    eng = Engine(shape, max_ctx=max_ctx, max_batch=B, max_prefill=a.prefill_chunk, ffn_fuse=a.ffn_fuse,
                 per_op_decode=a.per_op)
    build_on_device(shape, a.pmap, eng, seed=rank)
    eng.finalize()
    info = eng.info()
    # prefill every sequence with a 2048-token uniform-random prompt (timed separately, reported
    # under "prefill"; the decode metric below does not include it), after one untimed prefill
    # that loads the kernels and sizes the workspaces
    rng = np.random.default_rng(100 + rank)
    eng.forward(rng.integers(0, shape.vocab, min(ctx, a.prefill_chunk)), seq=0)
    torch.cuda.synchronize()
    eng.reset()
    t0 = time.perf_counter()
    for b in range(B):
        eng.forward(rng.integers(0, shape.vocab, ctx), seq=b)
    torch.cuda.synchronize()
    t_prefill = time.perf_counter() - t0
    st_ptr = eng.stream
    st = torch.cuda.ExternalStream(st_ptr)
    d_tok = torch.from_numpy(rng.integers(0, shape.vocab, B).astype(np.int32)).cuda()
    d_logits = torch.empty(B, shape.vocab, device="cuda")

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- roofline: the dominant kernel alone, at the prefilled context (the persistent kernel
    #      is launched without advancing the sequence) ----
    persistent = B == 1 and info["persistent_decode"]
    kv_read = info["kv_bytes_per_pos"] * (eng.seq_len(0) + 1)  # K and V of every layer, cached + new position
    if persistent:
        reps = max(3, a.steps // 2)
        for _ in range(2):
            eng.run_step_kernel(st_ptr)
        torch.cuda.synchronize()
        e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e4.record(st)
        for _ in range(reps):
            eng.run_step_kernel(st_ptr)
        e5.record(st)
        torch.cuda.synchronize()
        t_kern = e4.elapsed_time(e5) / 1000.0 / reps
        kern_bytes = info["weight_bytes"] - info["embed_bytes"] + kv_read
        kern_name = "persist_decode_kernel<8,128,0> (whole batch-1 step, 148 CTAs x 512 threads)"
        traffic_file = "decode_persist_7b_traffic.txt"
    else:
        x = torch.randn(B, shape.hidden, device="cuda")
        y = torch.empty(B, shape.ffn, device="cuda")
        for l in range(shape.layers):
            eng.run_linear(l, 2, x.data_ptr(), B, y.data_ptr(), st_ptr)
        torch.cuda.synchronize()
        reps = 5
        e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e4.record(st)
        for _ in range(reps):
            for l in range(shape.layers):
                eng.run_linear(l, 2, x.data_ptr(), B, y.data_ptr(), st_ptr)
        e5.record(st)
        torch.cuda.synchronize()
        t_kern = e4.elapsed_time(e5) / 1000.0 / (reps * shape.layers)
        kern_bytes = eng.linear_bytes(0, 2, B)
        kern_name = (f"gemm_tc_kernel (tcgen05, {32 if B <= 32 else 64 if B <= 64 else 128}-token tile, + x packing) "
                     if B > 8 else "gemv_mma2_kernel ") + \
            f"on gate|up {2 * shape.ffn}x{shape.hidden} INT4 g128 (+SwiGLU), batch {B}"
        traffic_file = "gemv_gateup_traffic.txt" if headline else "none"

    # ---- value: device-resident decode ----
    for _ in range(a.warmup):
        eng.decode_device(d_tok.data_ptr(), B, d_logits.data_ptr(), 0)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        e0.record(st)
        for _ in range(a.steps):
            eng.decode_device(0, B, 0, 0)
        e1.record(st)
        barrier()
    t_dev = e0.elapsed_time(e1) / 1000.0
    # ---- e2e: host ids in, host fp32 logits out (the reference's forward() contract), C ABI ----
    # (each leg restarts from the prefilled context, as the device-resident leg did)
    for b in range(B):
        eng.set_seq_len(b, ctx)
    host_tok = rng.integers(0, shape.vocab, B).astype(np.int32)
    for _ in range(2):
        eng.decode(host_tok)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for _ in range(a.steps):
        eng.decode(host_tok)
    e3.record(st)
    barrier()
    t_e2e = e2.elapsed_time(e3) / 1000.0
    # the same with the next ids sampled on the GPU (temperature 0.7 / top-p 0.9) instead of logits out
    for b in range(B):
        eng.set_seq_len(b, ctx)
    for _ in range(2):
        host_tok = eng.decode_sample(host_tok, 0.7, 0.9, 1234)
    barrier()
    e2.record(st)
    for _ in range(a.steps):
        host_tok = eng.decode_sample(host_tok, 0.7, 0.9, 1234)
    e3.record(st)
    barrier()
    t_e2e_sampled = e2.elapsed_time(e3) / 1000.0
    # max over ranks
    if world > 1:
        tt = torch.tensor([t_dev, t_e2e, t_kern, t_e2e_sampled], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_dev, t_e2e, t_kern, t_e2e_sampled = tt.tolist()
    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = kern_bytes / t_kern / 1e9
        traffic = None
        tf = REPO / "profiles" / traffic_file
        if tf.exists() and not a.layers:
            for line in tf.read_text().splitlines():
                if line.startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":", 1)[1])
        toks = B * a.steps * world
        kv_bytes = info["kv_bytes_per_pos"] * (ctx + a.warmup + a.steps // 2) * B
        step_bytes = info["weight_bytes"] + kv_bytes
        params = shape.layers * (shape.hidden * (shape.heads + 2 * shape.kv_heads) * shape.head_dim
                                 + shape.heads * shape.head_dim * shape.hidden
                                 + 3 * shape.hidden * shape.ffn) + shape.vocab * shape.hidden
        out = {
            "metric": METRIC if headline else f"decode tok/s at {a.model}-shape ({a.pmap})",
            "value": round(toks / t_dev, 2), "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t_dev / a.steps * 1000, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights (exact dequant); fp16 x, f32 accumulate",
            "data": "synthetic (random-init N(0,0.02) weights, uniform-random token ids)",
            "config": {"workload": f"{a.model}-shape decoder ({shape.layers} layers), "
                                   + ("all linears INT4 g128 (fp16 scale+zero)" if a.pmap == "int4_g128" else
                                      "attention INT8 per-tensor, FFN INT4 g128, fp16 tied embedding / lm_head")
                                   + f", batch {B} decode after a {ctx}-token prefill, fp16 paged KV",
                       "batch": B, "ctx_start": ctx, "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "decode_path": ("persistent kernel" + (", FFN fused" if info["ffn_fused"] else "")
                                       if persistent else "per-op kernels (graph)"),
                       "l2": f"no flush: {info['weight_bytes'] / 1e9:.2f} GB of weights stream from HBM every step "
                             "(L2 126 MB)"},
            "e2e": {"value": round(toks / t_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * B * shape.vocab, "call": "n730_model_decode (host logits out)",
                    "sampled_ids_out": {"value": round(toks / t_e2e_sampled, 2),
                                        "call": "n730_model_decode_sample (GPU temperature 0.7 / top-p 0.9)",
                                        "d2h_bytes_per_step": 8 * B}},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": kern_name,
                         "bytes_per_launch": kern_bytes, "ms_per_launch": round(t_kern * 1000, 4),
                         "peak_source": peak_kind},
            "step_roofline": {"bytes_per_step": step_bytes,
                              "achieved_gbs": round(step_bytes / (t_dev / a.steps) / 1e9, 1),
                              "frac": round(step_bytes / (t_dev / a.steps) / 1e9 / peak, 4)},
            "clocks": clk.summary(),
            "gpu_launches": a.steps * (3 if persistent else 5 * shape.layers + 3),
            "gpu_launches_e2e_per_step": (3 if persistent else 5 * shape.layers + 3) + 1,
            "prefill": {"tokens": B * ctx, "chunk": a.prefill_chunk, "s": round(t_prefill, 4), "tok_per_s": round(B * ctx / t_prefill, 1),
                        "tflops": round(2 * params * B * ctx / t_prefill / 1e12, 1),
                        "path": "tcgen05 GEMM (INT4 fragment tiles dequantised to fp16 into tensor memory as the "
                                "MMA's A operand, x from shared memory, TMEM accumulators, 256- or 128-token tiles) for "
                                f"every linear, prompt in chunks of {a.prefill_chunk} tokens; wall clock incl. host calls, "
                                "after one untimed prefill"},
        }
        if not a.no_cpu_baseline and headline:
            cs = CpuReferenceDecoder(shape, ctx)
            cs.step()
            t0 = time.perf_counter()
            for _ in range(2):
                cs.step()
            t_token = (time.perf_counter() - t0) / 2
            cs.close()
            out["cpu_baseline"] = {"value": round(1.0 / t_token, 4), "unit": "tok/s", "cores": _host_cores(),
                                   "kind": "reference", "blas_threads": cs.blas, "reader_threads": cs.threads,
                                   "sample": f"2 whole qwen2-7b-shape decode tokens at context {ctx} after 1 "
                                             f"warm-up ({t_token:.2f} s each): 28 layers x 7 reference "
                                             "n730_read_layer reads (per-tensor INT4) on a reader pool + numpy "
                                             "fp32 GEMVs, attention over an fp32 KV cache, final norm + lm_head"}
        print(json.dumps(out), flush=True)
    eng.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_streamed(a):
    """7B aggressive mixed quant with layer weights streamed from pinned host
    memory (depth-2 prefetch on a copy stream): decode tok/s, and the host->HBM
    link rate against a measured cudaMemcpyAsync peak."""
    import torch
    torch.cuda.set_device(0)
    from n730_b200.engine import Engine
    from n730_b200.synthetic import SHAPES, build_on_device
    shape = SHAPES[SHAPE_NAME]
    if a.layers:
        shape = dataclasses.replace(shape, layers=a.layers)
    prompt = 1024
    eng = Engine(shape, max_ctx=prompt + a.warmup + a.steps + 16, max_batch=1, max_prefill=512, stream_depth=2)
    build_on_device(shape, "aggressive", eng)
    eng.finalize()
    info = eng.info()
    # host->HBM peak: one 1 GiB pinned copy, best of 3
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    best = 1e9
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1000)
    h2d_peak = (1 << 30) / best / 1e9
    del src, dst
    rng = np.random.default_rng(7)
    eng.forward(rng.integers(0, shape.vocab, prompt))
    tok = np.array([int(rng.integers(0, shape.vocab))], np.int32)
    st = torch.cuda.ExternalStream(eng.stream)
    for _ in range(a.warmup):
        eng.decode(tok)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        e0.record(st)
        for _ in range(a.steps):
            eng.decode(tok)
        e1.record(st)
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1000 / a.steps
    link = info["streamed_bytes"] / t / 1e9
    out = {"metric": "decode tok/s, 7B aggressive mixed quant, layers streamed host->HBM", "value": round(1 / t, 3),
           "unit": "tok/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t * 1e3, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "int2/int4/int8 weights (exact dequant), f32 math", "data": "synthetic",
           "config": {"workload": f"qwen2-7b-shape ({shape.layers} layers), FFN INT2 g64, attention INT4 g128, "
                                  "lm_head INT8 per channel, embeddings INT4 g128; layer weights in pinned host "
                                  f"memory, stream_depth 2; batch 1 decode after a {prompt}-token prompt",
                      "streamed_bytes_per_step": info["streamed_bytes"], "resident_bytes": info["weight_bytes"]},
           "e2e": {"value": round(1 / t, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 + info["streamed_bytes"],
                   "d2h_bytes_per_step": 4 * shape.vocab},
           "roofline": {"bound": "host->HBM link", "achieved": round(link, 2), "peak": round(h2d_peak, 2),
                        "unit": "GB/s", "frac": round(link / h2d_peak, 4), "traffic": None,
                        "peak_source": "measured here: 1 GiB pinned cudaMemcpyAsync H2D, best of 3"},
           "clocks": clk.summary()}
    print(json.dumps(out), flush=True)
    eng.close()


def run_tp(a):
    """Qwen2-72B-shape INT4 g128 decode, tensor parallel over the N ranks (one
    model; q/k/v, gate/up column-split, o/down row-split with an NCCL
    allreduce each, vocab-split lm_head).  Decoding starts at a context of
    --ctx cached positions (zero-filled KV; per-step work matches a real
    prefill of that length)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from n730_b200 import tp
    from n730_b200.engine import Engine
    from n730_b200.synthetic import SHAPES, build_on_device
    world, rank, local = _dist()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device(f"cuda:{local}"))
    shape = SHAPES["qwen2-72b"]
    if a.layers:
        shape = dataclasses.replace(shape, layers=a.layers)
    tp.check_shape(shape, world, 128)
    B, ctx = a.batch, a.ctx
    eng = Engine(tp.local_shape(shape, world, rank, 128), max_ctx=ctx + a.warmup + 2 * a.steps + 16, max_batch=B,
                 max_prefill=64, tp_rank=rank, tp_size=world, tp_allreduce=a.tp_allreduce,
                 per_op_decode=a.per_op, ffn_fuse=a.ffn_fuse)
    if world > 1:
        tp.init_engine_comm(eng, rank, world)
    build_on_device(shape, "int4_g128", eng, tp_rank=rank, tp_size=world)
    eng.finalize()
    info = eng.info()
    for b in range(B):
        eng.set_seq_len(b, ctx)
    st = torch.cuda.ExternalStream(eng.stream)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(a.warmup):
        eng.decode_device(0, B, 0, 0)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        e0.record(st)
        for _ in range(a.steps):
            eng.decode_device(0, B, 0, 0)
        e1.record(st)
        barrier()
    t = e0.elapsed_time(e1) / 1000.0
    # e2e: host token ids in, host logits (all-gathered over the ranks) out, through the C ABI
    host_tok = np.random.default_rng(3).integers(0, shape.vocab, B).astype(np.int32)
    eng.decode(host_tok)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for _ in range(a.steps):
        eng.decode(host_tok)
    e3.record(st)
    barrier()
    t_e2e = e2.elapsed_time(e3) / 1000.0
    if world > 1:
        tt = torch.tensor([t, t_e2e], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, t_e2e = tt.tolist()
    if rank == 0:
        peak, kind = _peaks()
        kv = info["kv_bytes_per_pos"] * (ctx + a.warmup + a.steps // 2) * B
        step_bytes = info["weight_bytes"] - info["embed_bytes"] + kv  # per rank
        out = {"metric": TP_METRIC, "value": round(B * a.steps / t, 3),
               "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
               "ms_per_step": round(t / a.steps * 1e3, 4), "higher_is_better": True, "scaling": "strong",
               "vs_baseline": None, "dtype": "int4 weights (exact dequant); fp16 x, f32 accumulate",
               "data": "synthetic (random-init N(0,0.02) weights)",
               "config": {"workload": f"qwen2-72b-shape ({shape.layers} layers) INT4 g128, batch {B} decode at "
                                      f"context {ctx}, tensor parallel over {world} GPU(s) (row-split sums after "
                                      "o_proj and down_proj, vocab-split lm_head)", "batch": B,
                          "allreduce": ("in-kernel: partial sums pushed to every rank over NVLink peer memory, "
                                        "cross-GPU barrier, rank-order sums" if info["persistent_decode"] else
                                        "one-shot push over NVLink peer memory, fused residual add"
                                        if a.tp_allreduce == 0 else "NCCL") if world > 1 else None,
                          "decode_path": ("persistent kernel" + (", phase table in global memory"
                                                                 if info["phase_table_global"] else "")
                                          if info["persistent_decode"] else "per-op kernels (graph)"),
                          "parallelism": f"tp{world}",
                          "scale_point": f"one qwen2-72b-shape model over {world} GPU(s); the N = 1 point is the "
                                         "same model on one GPU (strong scaling)",
                          "plan_mismatch": info["tp_plan_mismatch"],
                          "l2": f"no flush: {step_bytes / 1e9:.2f} GB per rank stream from HBM every step (L2 126 MB)"},
               "e2e": {"value": round(B * a.steps / t_e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                       "d2h_bytes_per_step": 4 * B * shape.vocab, "call": "n730_model_decode (host logits out)"},
               "roofline": {"bound": "hbm", "achieved": round(step_bytes / (t / a.steps) / 1e9, 1), "peak": peak,
                            "unit": "GB/s per GPU", "frac": round(step_bytes / (t / a.steps) / 1e9 / peak, 4),
                            "traffic": None, "kernel": "whole decode step, per-rank bytes", "peak_source": kind},
               "clocks": clk.summary(),
               "gpu_launches": a.steps * (4 if info["persistent_decode"] else 7 * shape.layers + 6)}
        print(json.dumps(out), flush=True)
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_linear(a):
    """Single INT4 g128 dequant-GEMV, W [4096, 4096] ~ N(0, 0.02) seed 0, batch 1 (the reference's
    single-linear configuration): launches rotate over enough weight copies to exceed 4x L2, one CUDA
    graph of the rotation is replayed, bytes per GEMV = codes + scale/zero + x + y."""
    import ctypes as C

    import torch
    from n730_b200 import _lib
    lib = _lib.cuda()
    torch.cuda.set_device(0)
    rows, cols = (int(v) for v in a.linear_shape.lower().split("x"))
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    w = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    P = lambda t: C.c_void_p(t.data_ptr())
    per = rows * cols // 2 + rows * (cols // 128) * 4
    copies = a.copies or max(4, -(-4 * 126 * 2**20 // per))
    qs = []
    for _ in range(copies):
        codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
        s16 = torch.empty(rows, cols // 128, dtype=torch.float16, device="cuda")
        z16 = torch.empty_like(s16)
        _lib.check(lib.n730_quantize_grouped(P(w), rows, cols, 4, 128, P(codes), P(s16), P(z16), None), "quantize")
        q = C.c_void_p()
        _lib.check(lib.n730_qweight_create(0x44, rows, cols, 128, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                           C.byref(q)), "qweight_create")
        _lib.check(lib.n730_qweight_set_layout(q, 1, None), "qweight_set_layout")
        qs.append(q)
    del w
    torch.cuda.synchronize()
    g1 = torch.Generator(device="cuda")
    g1.manual_seed(1)
    x = torch.randn(1, cols, generator=g1, device="cuda")
    y = torch.empty(copies, rows, device="cuda")
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for i in range(copies):  # warm-up outside capture
            _lib.check(lib.n730_qlinear(qs[i], P(x), cols, 1, P(y[i]), rows, None, None, 0, None, 1e-6, 0,
                                        C.c_void_p(side.cuda_stream)), "qlinear")
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st = torch.cuda.current_stream().cuda_stream
        for i in range(copies):
            _lib.check(lib.n730_qlinear(qs[i], P(x), cols, 1, P(y[i]), rows, None, None, 0, None, 1e-6, 0,
                                        C.c_void_p(st)), "qlinear")
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1000.0 / (a.steps * copies)
    bytes_per = rows * cols // 2 + rows * (cols // 128) * 4 + cols * 4 + rows * 4
    peak, kind = _peaks()
    out = {"metric": f"single-linear INT4 g128 dequant-GEMV bandwidth (W {rows}x{cols}, batch 1)",
           "value": round(bytes_per / t / 1e9, 1), "unit": "GB/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": round(t * 1e3, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "int4 weights (exact dequant); fp16 x, f32 accumulate",
           "data": "synthetic W ~ N(0, 0.02) seed 0, x ~ N(0, 1) seed 1",
           "config": {"workload": f"one {rows}x{cols} INT4 g128 GEMV per step (n730_qlinear, tensor-core GEMV)",
                      "copies": copies, "l2": f"rotation over {copies} weight copies = "
                                              f"{copies * bytes_per / 1e6:.0f} MB (L2 126 MB)", "graph": True},
           "roofline": {"bound": "hbm", "achieved": round(bytes_per / t / 1e9, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(bytes_per / t / 1e9 / peak, 4), "traffic": None,
                        "kernel": f"gemv_mma2_kernel<8,1,WARPS> ({rows} rows, K {cols}; 8 warps per CTA below 32 chunks per SM, else 16)", "bytes_per_launch": bytes_per,
                        "ms_per_launch": round(t * 1e3, 5), "peak_source": kind},
           "clocks": clk.summary(), "gpu_launches": a.steps * copies}
    print(json.dumps(out), flush=True)
    for q in qs:
        lib.n730_qweight_destroy(q)


def _tensor_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback (burst)"


def run_gemm(a):
    """The tcgen05 prefill GEMM alone (n730_qgemm: x packing + the GEMM kernel per call) on one
    INT4 g128 weight of --linear-shape for --tokens tokens, calls replayed from a CUDA graph over
    --copies weight copies; TFLOP/s = 2 rows cols tokens per call against the measured burst
    bf16 tensor peak (the kernel is kind::f16, the same rate)."""
    import ctypes as C
    import torch
    from n730_b200 import _lib
    lib = _lib.cuda()
    torch.cuda.set_device(0)
    rows, cols = (int(v) for v in a.linear_shape.lower().split("x"))
    T = a.tokens
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    w = torch.randn(rows, cols, generator=g, device="cuda") * 0.02
    P = lambda t: C.c_void_p(t.data_ptr())
    copies = a.copies or 2
    qs = []
    for _ in range(copies):
        codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
        s16 = torch.empty(rows, cols // 128, dtype=torch.float16, device="cuda")
        z16 = torch.empty_like(s16)
        _lib.check(lib.n730_quantize_grouped(P(w), rows, cols, 4, 128, P(codes), P(s16), P(z16), None), "quantize")
        q = C.c_void_p()
        _lib.check(lib.n730_qweight_create(0x44, rows, cols, 128, 1.0, 0.0, P(codes), P(s16), P(z16), 1, None,
                                           C.byref(q)), "qweight_create")
        _lib.check(lib.n730_qweight_set_layout(q, 1, None), "qweight_set_layout")
        qs.append(q)
    del w
    g1 = torch.Generator(device="cuda")
    g1.manual_seed(1)
    x = torch.randn(T, cols, generator=g1, device="cuda")
    y = torch.empty(copies, T, rows, device="cuda")
    side = torch.cuda.Stream()
    call = lambda i, st: _lib.check(lib.n730_qgemm(qs[i], P(x), cols, T, P(y[i]), rows, None, None, 0, None, 1e-6, 0,
                                                   None, C.c_void_p(st)), "qgemm")
    with torch.cuda.stream(side):
        for i in range(copies):  # warm-up outside capture (grows the packed-x workspace)
            call(i, side.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st = torch.cuda.current_stream().cuda_stream
        for i in range(copies):
            call(i, st)
    for _ in range(a.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1000.0 / (a.steps * copies)
    flops = 2.0 * rows * cols * T
    peak, kind = _tensor_peak()
    tf = flops / t / 1e12
    ntok = 256 if -(-rows // 128) * -(-T // 256) >= torch.cuda.get_device_properties(0).multi_processor_count else 128
    out = {"metric": f"INT4 g128 prefill GEMM throughput (W {rows}x{cols}, {T} tokens)",
           "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": round(t * 1e3, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "int4 weights dequantised to fp16; fp16 x; f32 accumulate (tcgen05 kind::f16)",
           "data": "synthetic W ~ N(0, 0.02) seed 0, x ~ N(0, 1) seed 1",
           "config": {"workload": f"one {rows}x{cols} INT4 g128 GEMM of {T} tokens per call (n730_qgemm)",
                      "copies": copies, "graph": True, "token_tile": ntok},
           "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tf / peak, 4), "traffic": None,
                        "kernel": f"gemm_tc_kernel<{ntok}> + x16_pack_kernel per call", "ms_per_launch": round(t * 1e3, 5),
                        "peak_source": kind},
           "clocks": clk.summary(), "gpu_launches": a.steps * copies * 2}
    print(json.dumps(out), flush=True)
    for q in qs:
        lib.n730_qweight_destroy(q)


def run_phases(a):
    """Per-phase timing of the persistent decode kernel (--model, batch 1, context --ctx): --steps
    traced launches (n730_model_trace_step, medians over them).  Per phase kind, averaged over the
    layers: the wall time (last CTA leaving the barrier that starts the phase to the last CTA
    leaving the next one), the algorithmic bytes per wall time, the arrival spread at the barrier
    that starts it (slowest minus fastest CTA) and its release latency (last arrival to first
    departure), the median CTA's time to the marks inside the phase (prologue done; FFN:
    gate|up done; attention: split written, all splits of the head published), and the mean
    time a warp spent waiting for its weight chunks.  Then the
    untraced kernel timed with CUDA events.  Prints one JSON line."""
    import torch
    torch.cuda.set_device(0)
    from n730_b200.engine import Engine
    from n730_b200.synthetic import SHAPES, build_on_device
    shape = SHAPES[a.model]
    if a.layers:
        shape = dataclasses.replace(shape, layers=a.layers)
    if a.vocab:
        shape = dataclasses.replace(shape, vocab=a.vocab)
    eng = Engine(shape, max_ctx=a.ctx + 64, max_batch=1, max_prefill=512, ffn_fuse=a.ffn_fuse)
    build_on_device(shape, a.pmap, eng)
    eng.finalize()
    info = eng.info()
    assert info["persistent_decode"], "the model does not decode through the persistent kernel"
    eng.set_seq_len(0, a.ctx)
    st = torch.cuda.ExternalStream(eng.stream)
    h, qd, kvd, f = shape.hidden, shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim, shape.ffn
    wb = lambda rows, cols: rows * cols // 2 + rows * (cols // 128) * 4  # INT4 g128 codes + fp16 scale/zero
    kv_layer = info["kv_bytes_per_pos"] // shape.layers * (a.ctx + 1)
    runs = []
    for _ in range(max(1, a.steps)):
        times, kinds = eng.trace_step(eng.stream)
        runs.append(times.astype(np.float64))
    R = 6  # trace rows per phase
    T = np.median(np.stack(runs), axis=0)  # [R n + 1][grid] ns
    n = len(kinds)
    arr = lambda p: T[R * p] if p < n else T[R * n]
    dep = np.array([T[R * p + 1].max() for p in range(n)] + [T[R * n].max()])

    def med(x):
        x = x[np.isfinite(x)]
        return float(np.median(x)) / 1e3 if x.size else None

    def since(row, start):  # per-CTA interval, CTAs without the mark left out
        d = np.where((row > 0) & (start > 0), row - start, np.nan)
        return med(d)

    rows = []
    gemv_i = 0
    for p in range(n):
        k = int(kinds[p])
        st0, m1, m2, nxt = T[R * p + 1], T[R * p + 2], T[R * p + 3], arr(p + 1)
        w1, w2 = float(np.mean(T[R * p + 4])) / 16e3, float(np.mean(T[R * p + 5])) / 16e3  # per warp, us
        r = {}
        if k == 1:
            name, nbytes = "attention", kv_layer
            r = {"split_us": since(m1, st0), "publish_wait_us": since(m2, m1), "merge_us": since(nxt, m2)}
        elif k == 2:
            name, nbytes = "ffn (gate|up + down)", wb(2 * f, h) + wb(h, f)
            r = {"prologue_us": since(m1, st0), "gate_up_us": since(m2, m1), "down_us": since(nxt, m2),
                 "gate_up_wait_us": w1, "down_wait_us": w2}
        else:
            if p == n - 1:
                name, nbytes = "lm_head", wb(shape.vocab, h)
            else:
                name, nbytes = ("qkv", wb(qd + 2 * kvd, h)) if gemv_i % 2 == 0 else ("o_proj", wb(h, qd))
                gemv_i += 1
            r = {"prologue_us": since(m1, st0), "stream_us": since(nxt, m1), "chunk_wait_us": w1}
        wall = (dep[p + 1] - dep[p]) / 1e3
        a_p = arr(p)
        r.update({"phase": name, "wall_us": wall, "gbs": nbytes / max(wall, 1e-9) / 1e3,
                  "spread_us": (a_p.max() - a_p.min()) / 1e3 if p else 0.0,
                  "release_us": (T[R * p + 1].min() - a_p.max()) / 1e3 if p else 0.0})
        rows.append(r)
    summary = {}
    for r in rows:
        d = summary.setdefault(r["phase"], {"n": 0})
        d["n"] += 1
        for key, v in r.items():
            if key != "phase" and v is not None:
                d[key] = d.get(key, 0.0) + v
    for d in summary.values():
        for key in list(d):
            if key != "n":
                d[key] = round(d[key] / d["n"], 3)
    total_us = (T[R * n].max() - T[0].min()) / 1e3
    for _ in range(3):
        eng.run_step_kernel(eng.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(20):
        eng.run_step_kernel(eng.stream)
    e1.record(st)
    torch.cuda.synchronize()
    out = {"workload": f"{a.model}-shape ({shape.layers} layers, {a.pmap}) persistent decode at context {a.ctx}",
           "traced_launches": len(runs), "traced_launch_us": round(total_us, 1),
           "untraced_ms_per_launch": round(e0.elapsed_time(e1) / 20, 4), "phases_per_layer": summary,
           "ffn_fused": info["ffn_fused"], "grid": info["persistent_grid"]}
    print(json.dumps(out), flush=True)
    eng.close()


def main():
    a = _args()
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "streamed":
        run_streamed(a)
    elif a.workload == "phases":
        run_phases(a)
    elif _tp_workload(a):
        run_tp(a)
    elif a.workload == "gemm":
        run_gemm(a)
    elif a.workload == "linear":
        run_linear(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
