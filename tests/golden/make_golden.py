"""Generate the golden fixtures for the packed-weight format from the reference itself.

Run in a container that has the reference tree (read-only) at REF_ROOT:

    make -C oracle REF_ROOT=<reference root>
    python tests/golden/make_golden.py --ref-root <reference root>

It imports the reference ``src-code/converter.py`` and calls its own
``convert()``/``read_layer()`` and quantisers, and loads the reference C core
``n730core.so`` built from ``src-code/cpp/n730core.cpp`` by ``oracle/Makefile``.
Outputs (small, committed):

* ``ref_small.n730``       - a .n730 file written by the reference ``convert()``:
                             INT8/INT4/INT2/FP16 tensors, odd element counts,
                             1-D bias, degenerate (constant) tensors.
* ``ref_small.npz``        - per tensor: the reference ``read_layer`` output,
                             the reference ``n730core`` ``n730_read_layer``
                             output, rows/cols/prec, and the input weights.
* ``ref_profiler.npz``     - the reference profiler's sensitivity scores and
                             statistics on seeded tensors (``profiler_cases``).
* ``ref_linear4096.npz``   - the single quantised linear W[4096x4096] ~ N(0,0.02)
                             (``default_rng(0)``) converted by the reference to
                             per-tensor INT4: code SHA-256, scale, zero point,
                             dequant samples at seeded indices and
                             ``y = x @ dequant(W).T`` for x[1x4096] fp16 ~ N(0,1)
                             (``default_rng(1)``).
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import io
import json
import sys
from contextlib import redirect_stdout
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _small_tensors():
    rng = np.random.default_rng(1234)
    t = {}
    t["t.int8"] = ("INT8", rng.normal(0, 0.02, (64, 96)).astype(np.float32))
    t["t.int4"] = ("INT4", rng.normal(0, 0.02, (64, 96)).astype(np.float32))
    t["t.int4_odd"] = ("INT4", rng.normal(0, 0.05, (7, 33)).astype(np.float32))
    t["t.int2"] = ("INT2", rng.normal(0, 0.02, (48, 80)).astype(np.float32))
    t["t.int2_odd"] = ("INT2", rng.normal(0, 0.02, (5, 13)).astype(np.float32))
    t["t.fp16"] = ("FP16", rng.normal(0, 1.0, (32, 64)).astype(np.float32))
    t["t.bias"] = ("FP16", rng.normal(0, 0.02, (64,)).astype(np.float32))
    t["t.const4"] = ("INT4", np.full((16, 32), 0.25, np.float32))
    t["t.const8"] = ("INT8", np.zeros((8, 16), np.float32))
    t["t.int8_wide"] = ("INT8", rng.uniform(-3, 3, (4, 260)).astype(np.float32))
    return t


def profiler_cases():
    """Seeded tensors for the sensitivity score: (seed, rows, cols, std, outlier share, layer, layers).
    ``profiler_tensor`` regenerates each one; the tests use the same two functions."""
    return [(1, 512, 256, 0.02, 0.0, 0, 32), (2, 512, 256, 0.035, 0.0, 16, 32), (3, 512, 256, 0.04, 0.06, 31, 32),
            (4, 3000, 1500, 0.03, 0.01, 5, 32), (5, 64, 64, 0.0, 0.0, 7, 9)]


def profiler_tensor(seed, rows, cols, std, outliers):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, std, (rows, cols)).astype(np.float32) if std > 0 else np.full((rows, cols), 0.5, np.float32)
    if outliers:
        n = int(w.size * outliers)
        idx = rng.choice(w.size, n, replace=False)
        w.flat[idx] = rng.choice([-1, 1], n) * rng.uniform(0.3, 0.8, n)
    return w


def write_profiler_golden(ref: Path):
    """The reference profiler's own sensitivity scores (src-code/profiler.py:50-89) on seeded tensors."""
    sys.path.insert(0, str(ref / "src-code"))
    import profiler  # the reference profiler, unmodified
    cases = profiler_cases()
    scores = [profiler.compute_sensitivity(profiler_tensor(*c[:5]), c[5], c[6]) for c in cases]
    prof = [profiler.profile_weight_tensor(profiler_tensor(*c[:5]), c[5], f"t{i}", c[6]) for i, c in enumerate(cases)]
    np.savez_compressed(HERE / "ref_profiler.npz", cases=np.array(cases, np.float64), scores=np.array(scores),
                        std=np.array([p.weight_std for p in prof]), kurtosis=np.array([p.weight_kurtosis for p in prof]),
                        outlier_ratio=np.array([p.outlier_ratio for p in prof]))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", required=True, help="root of the reference checkout (holds src-code/)")
    ap.add_argument("--only", choices=["profiler"], help="write one fixture only")
    args = ap.parse_args()
    ref = Path(args.ref_root)
    if args.only == "profiler":
        write_profiler_golden(ref)
        return
    sys.path.insert(0, str(ref / "src-code"))
    import converter  # the reference converter, unmodified

    core_path = REPO / "oracle" / "_ref" / "n730core.so"
    if not core_path.exists():
        raise SystemExit(f"build the reference core first: make -C {REPO / 'oracle'}")
    core = ctypes.CDLL(str(core_path))
    core.n730_open.argtypes = [ctypes.c_char_p]
    core.n730_open.restype = ctypes.c_int64
    core.n730_close.argtypes = [ctypes.c_int64]
    core.n730_read_layer.argtypes = [ctypes.c_int64, ctypes.c_int64,
                                     ctypes.POINTER(ctypes.c_float),
                                     ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32)]
    core.n730_read_layer.restype = ctypes.c_int32

    # ---- small mixed-precision file written by the reference convert() ----
    tensors = _small_tensors()
    smap = {"model_id": "golden-small", "total_params": int(sum(w.size for _, w in tensors.values())),
            "total_layers": len(tensors),
            "profiles": [{"layer_name": k, "assigned_precision": p} for k, (p, _) in tensors.items()]}
    out_file = HERE / "ref_small.n730"
    with redirect_stdout(io.StringIO()):
        header = converter.convert([(k, w) for k, (_, w) in tensors.items()], smap, out_file,
                                   verbose=False)
    arrays = {}
    h = core.n730_open(str(out_file).encode())
    assert h > 0, h
    for i, (name, (prec, w)) in enumerate(tensors.items()):
        entry = header["seek_table"][i]
        ref_np = converter.read_layer(out_file, i)
        n = entry["rows"] * entry["cols"]
        buf = np.zeros(n, np.float32)
        r, c, p = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        rc = core.n730_read_layer(h, entry["file_offset"],
                                  buf.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                  ctypes.byref(r), ctypes.byref(c), ctypes.byref(p))
        assert rc == 0, rc
        key = name.replace(".", "_")
        arrays[f"{key}__w"] = w
        arrays[f"{key}__read_layer"] = ref_np.astype(np.float32)
        arrays[f"{key}__n730core"] = buf.reshape(ref_np.shape)
        arrays[f"{key}__meta"] = np.array([r.value, c.value, p.value], np.int64)
    core.n730_close(h)
    np.savez_compressed(HERE / "ref_small.npz", **arrays)
    (HERE / "ref_small.header.json").write_text(json.dumps(header, indent=1))

    # ---- the single quantised linear 4096x4096 INT4 (per-tensor, reference format) ----
    W = np.random.default_rng(0).normal(0, 0.02, (4096, 4096)).astype(np.float32)
    x = np.random.default_rng(1).normal(0, 1, (1, 4096)).astype(np.float16)
    codes, scale, zp = converter.quantize_int4(W)
    smap1 = {"model_id": "linear4096", "total_params": W.size, "total_layers": 1,
             "profiles": [{"layer_name": "linear.weight", "assigned_precision": "INT4"}]}
    tmp = Path("/tmp/_golden_linear4096.n730")
    with redirect_stdout(io.StringIO()):
        converter.convert([("linear.weight", W)], smap1, tmp, verbose=False)
    Wd = converter.read_layer(tmp, 0)
    tmp.unlink()
    y = x.astype(np.float32) @ Wd.T
    idx = np.random.default_rng(7).integers(0, W.size, 4096)
    np.savez_compressed(
        HERE / "ref_linear4096.npz",
        codes_sha256=np.frombuffer(hashlib.sha256(codes).digest(), np.uint8),
        scale=np.float64(scale), zero_point=np.float64(zp),
        sample_idx=idx, sample_dequant=Wd.reshape(-1)[idx].astype(np.float32),
        dequant_sum=np.float64(Wd.astype(np.float64).sum()),
        x=x, y=y.astype(np.float32))
    write_profiler_golden(ref)
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".n730", ".npz", ".json")))


if __name__ == "__main__":
    main()
