"""Precision profiler: the reference's ``src-code/profiler.py`` surface, with a
real group-wise precision assignment.

The reference scores each weight tensor's sensitivity from three statistics
(``profiler.py:50-89``: the share of weights beyond 3 standard deviations, the
excess kurtosis, and a U-shaped position bias across the layers) and then
assigns INT8 to every tensor (``assign_precision``, ``profiler.py:92-93``).
``compute_sensitivity`` here keeps that score exactly (same statistics, same
4M-element sample, same weights 0.45 / 0.30 / 0.25).  The assignment is new:

* for each tensor the relative quantisation error ``|W - dq(q(W))| / |W|`` of
  every candidate is measured on a seeded sample of rows with the converter's
  own quantisers (the bytes the file will hold): ``INT2G64``, ``INT4G128``,
  ``INT8PC`` (per-channel) and ``FP16``;
* ``assign_precision`` takes the cheapest candidate whose error is within the
  tolerance ``TOL_MAX * (1 - sensitivity)^2 + TOL_MIN`` (about 0.5 for a score
  of 0, INT2 territory; 0.13 at 0.5, INT4; 0.01 at 1, INT8), so more sensitive
  tensors keep more bits; embeddings and the lm_head take at least INT4G128;
* ``allocate_bits`` instead meets a bits-per-weight budget: every tensor starts
  at its cheapest candidate and the upgrade with the largest sensitivity-
  weighted error reduction per added bit is taken until the budget is spent.

The map's ``assigned_precision`` strings are the converter's syntax, so
``converter.convert(layers, map, path)`` writes the file directly.
"""
from __future__ import annotations

import argparse
import json
import math
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np

from .converter import quantize_grouped

PRECISION_LEVELS = {"INT2": 2, "INT4": 4, "INT8": 8, "FP16": 16}
# candidates from cheapest to dearest: (name in converter syntax, bits per weight incl. fp16 scale + zero)
CANDIDATES = ("INT2G64", "INT4G128", "INT8PC", "FP16")
TOL_MAX, TOL_MIN = 0.5, 0.005
SAMPLE_ROWS = 256


def candidate_bits(name: str, cols: int) -> float:
    """Stored bits per weight: codes plus the fp16 scale and zero of each group (per row for INT8PC)."""
    return {"INT2G64": 2 + 32 / 64, "INT4G128": 4 + 32 / 128, "INT8PC": 8 + 32 / max(cols, 1),
            "FP16": 16.0}[name]


@dataclass
class LayerProfile:
    layer_idx: int
    layer_name: str
    param_count: int
    weight_std: float
    weight_kurtosis: float
    outlier_ratio: float
    sensitivity_score: float
    assigned_precision: str
    vram_bytes_original: int
    vram_bytes_n730: int
    compression_ratio: float
    quant_errors: dict = field(default_factory=dict)   # candidate -> relative error on the row sample
    bits_per_weight: float = 0.0


@dataclass
class SensitivityMap:
    model_id: str
    total_layers: int
    total_params: int
    profiles: list
    vram_original_mb: float
    vram_n730_mb: float
    overall_compression: float
    profiler_version: str = "0.2.0-b200"
    project: str = "N730"


def _sample(flat: np.ndarray, layer_idx: int) -> np.ndarray:
    # large tensors are sampled to 4M elements with the layer index as the seed (profiler.py:55-58)
    if flat.size > 4_000_000:
        rng = np.random.default_rng(seed=layer_idx)
        flat = rng.choice(flat, size=4_000_000, replace=False)
    return flat


def _stats(weights: np.ndarray, layer_idx: int):
    flat = _sample(weights.flatten().astype(np.float64), layer_idx)
    std = float(np.std(flat))
    mean = float(np.mean(flat))
    if std < 1e-9:
        return std, 0.0, 0.0
    normalised = np.clip((flat - mean) / std, -1e6, 1e6)
    kurtosis = float(np.mean(normalised ** 4)) - 3.0
    outlier_ratio = float(np.mean(np.abs(flat - mean) > (3.0 * std)))
    return std, kurtosis, outlier_ratio


def compute_sensitivity(weights: np.ndarray, layer_idx: int, total_layers: int) -> float:
    """The reference's score in [0, 1] (``profiler.py:50-89``)."""
    _, kurtosis, outlier_ratio = _stats(weights, layer_idx)
    relative_pos = layer_idx / max(total_layers - 1, 1)
    position_bias = 1.0 - math.sin(math.pi * relative_pos) ** 2
    outlier_score = min(outlier_ratio * 20.0, 1.0)
    kurtosis_score = min(max(kurtosis / 10.0, 0.0), 1.0)
    sensitivity = 0.45 * outlier_score + 0.30 * kurtosis_score + 0.25 * position_bias
    return float(np.clip(sensitivity, 0.0, 1.0))


def _unpack(codes: np.ndarray, bits: int, n: int) -> np.ndarray:
    per = 8 // bits
    raw = np.asarray(codes, np.uint8).reshape(-1)
    out = np.empty(raw.size * per, np.uint8)
    for i in range(per):
        out[i::per] = (raw >> (bits * i)) & ((1 << bits) - 1)
    return out[:n]


def quant_error(weights: np.ndarray, candidate: str, layer_idx: int = 0) -> float:
    """Relative Frobenius error of ``candidate`` on a seeded sample of up to SAMPLE_ROWS rows."""
    w = np.asarray(weights, np.float32)
    if w.ndim != 2:
        w = w.reshape(1, -1)
    rows, cols = w.shape
    if rows > SAMPLE_ROWS:
        idx = np.sort(np.random.default_rng(layer_idx).choice(rows, SAMPLE_ROWS, replace=False))
        w = w[idx]
        rows = SAMPLE_ROWS
    norm = float(np.linalg.norm(w.astype(np.float64)))
    if norm == 0.0:
        return 0.0
    if candidate == "FP16":
        dq = w.astype(np.float16).astype(np.float32)
    else:
        bits, group = {"INT2G64": (2, 64), "INT4G128": (4, 128), "INT8PC": (8, cols)}[candidate]
        if cols % group:
            return float("inf")  # the group does not tile the row
        codes, s16, z16 = quantize_grouped(w, bits, group)
        q = _unpack(codes, bits, rows * cols).reshape(rows, cols).astype(np.float32)
        s = np.repeat(s16.astype(np.float32), group, axis=1)
        z = np.repeat(z16.astype(np.float32), group, axis=1)
        dq = (q - z) * s
    return float(np.linalg.norm((w - dq).astype(np.float64)) / norm)


def tolerance(sensitivity: float) -> float:
    return TOL_MAX * (1.0 - sensitivity) ** 2 + TOL_MIN


def _floor_of(layer_name: str) -> int:
    """Index into CANDIDATES below which a tensor is never stored: embeddings and the lm_head
    (one row per token, every logit through it) keep at least INT4G128."""
    return 1 if layer_name.endswith(("embed_tokens.weight", "lm_head.weight")) else 0


def assign_precision(sensitivity: float, layer_name: str = "", errors: dict | None = None) -> str:
    """The cheapest candidate whose measured error is within ``tolerance(sensitivity)``.  Without
    errors (no tensor at hand) the tolerance is compared with typical errors of N(0, s) weights."""
    if errors is None:
        errors = {"INT2G64": 0.47, "INT4G128": 0.115, "INT8PC": 0.006, "FP16": 0.0003}
    tol = tolerance(sensitivity)
    for c in CANDIDATES[_floor_of(layer_name):]:
        if errors.get(c, float("inf")) <= tol:
            return c
    return "FP16"


def profile_weight_tensor(weights: np.ndarray, layer_idx: int, layer_name: str, total_layers: int,
                          measure: bool = True) -> LayerProfile:
    param_count = int(weights.size)
    std, kurtosis, outlier_ratio = _stats(weights, layer_idx)
    sensitivity = compute_sensitivity(weights, layer_idx, total_layers)
    errors = {c: quant_error(weights, c, layer_idx) for c in CANDIDATES} if measure else None
    precision = assign_precision(sensitivity, layer_name, errors)
    cols = weights.shape[-1] if weights.ndim >= 2 else weights.size
    bpw = candidate_bits(precision, cols)
    vram_original = param_count * 4
    vram_n730 = math.ceil(param_count * bpw / 8)
    return LayerProfile(layer_idx=layer_idx, layer_name=layer_name, param_count=param_count,
                        weight_std=round(std, 6), weight_kurtosis=round(kurtosis, 4),
                        outlier_ratio=round(outlier_ratio, 6), sensitivity_score=round(sensitivity, 4),
                        assigned_precision=precision, vram_bytes_original=vram_original, vram_bytes_n730=vram_n730,
                        compression_ratio=round(vram_original / max(vram_n730, 1), 2),
                        quant_errors={k: round(v, 6) for k, v in (errors or {}).items()}, bits_per_weight=bpw)


def allocate_bits(profiles: list, target_bits: float, cols_of: dict | None = None) -> list:
    """Re-assign precisions to meet an average of ``target_bits`` per weight (a target below the
    cheapest allowed assignment leaves that assignment): every tensor starts
    at its cheapest allowed candidate with a finite error; the upgrade with the largest
    (1 + 4 sensitivity) x error reduction per added bit is taken while the budget allows."""
    cols_of = cols_of or {}
    total = sum(p.param_count for p in profiles)
    level = []
    for p in profiles:
        lo = _floor_of(p.layer_name)
        while lo < len(CANDIDATES) - 1 and not math.isfinite(p.quant_errors.get(CANDIDATES[lo], float("inf"))):
            lo += 1
        level.append(lo)
    cols = [cols_of.get(p.layer_name, 4096) for p in profiles]
    bits = lambda i, lv: candidate_bits(CANDIDATES[lv], cols[i])
    used = sum(bits(i, level[i]) * p.param_count for i, p in enumerate(profiles))
    budget = target_bits * total
    while True:
        best, best_gain = None, 0.0
        for i, p in enumerate(profiles):
            if level[i] + 1 >= len(CANDIDATES):
                continue
            nxt = level[i] + 1
            while nxt < len(CANDIDATES) and not math.isfinite(p.quant_errors.get(CANDIDATES[nxt], float("inf"))):
                nxt += 1
            if nxt >= len(CANDIDATES):
                continue
            extra = (bits(i, nxt) - bits(i, level[i])) * p.param_count
            if used + extra > budget:
                continue
            gain = (1.0 + 4.0 * p.sensitivity_score) * (p.quant_errors[CANDIDATES[level[i]]] -
                                                  p.quant_errors[CANDIDATES[nxt]]) * p.param_count / extra
            if gain > best_gain:
                best, best_gain = (i, nxt, extra), gain
        if best is None:
            break
        i, nxt, extra = best
        level[i] = nxt
        used += extra
    for i, p in enumerate(profiles):
        p.assigned_precision = CANDIDATES[level[i]]
        p.bits_per_weight = bits(i, level[i])
        p.vram_bytes_n730 = math.ceil(p.param_count * p.bits_per_weight / 8)
        p.compression_ratio = round(p.vram_bytes_original / max(p.vram_bytes_n730, 1), 2)
    return profiles


def generate_synthetic_layers(num_layers: int, hidden_size: int = 4096, seed: int | None = None):
    """Synthetic transformer-like tensors with the reference generator's distributions
    (``profiler.py:143-172``): early layers N(0, 0.02), middle N(0, 0.035), the last ~12 % N(0, 0.04)
    with 6 % outliers of magnitude 0.3-0.8 (seeded here)."""
    rng = np.random.default_rng(seed)
    layers = []
    for i in range(num_layers):
        relative = i / max(num_layers - 1, 1)
        shape = (hidden_size, hidden_size // 4)
        if relative < 0.1:
            w = rng.normal(0, 0.02, shape).astype(np.float32)
        elif relative > 0.88:
            w = rng.normal(0, 0.04, shape).astype(np.float32)
            n_out = int(w.size * 0.06)
            idx = rng.choice(w.size, n_out, replace=False)
            w.flat[idx] = rng.choice([-1, 1], n_out) * rng.uniform(0.3, 0.8, n_out)
        else:
            w = rng.normal(0, 0.035, shape).astype(np.float32)
        layers.append((f"transformer.layer.{i}.weight", w))
    return layers


def load_model_layers(model_path: str):
    """Every >= 2-D parameter of a Hugging Face checkpoint (``profiler.py:174-193``)."""
    from transformers import AutoModelForCausalLM
    import torch
    model = AutoModelForCausalLM.from_pretrained(model_path, torch_dtype=torch.float32, device_map="cpu",
                                                 low_cpu_mem_usage=True)
    return [(n, p.detach().numpy()) for n, p in model.named_parameters() if p.ndim >= 2]


def run_profiler(model_id: str, weight_layers, verbose: bool = True, target_bits: float | None = None,
                 measure: bool = True) -> SensitivityMap:
    """Profile every tensor; with ``target_bits`` the precisions are then re-assigned to meet that
    average (``allocate_bits``)."""
    weight_layers = list(weight_layers)
    total_layers = len(weight_layers)
    t0 = time.time()
    profiles, cols_of = [], {}
    for idx, (name, w) in enumerate(weight_layers):
        p = profile_weight_tensor(w, idx, name, total_layers, measure=measure)
        profiles.append(p)
        cols_of[name] = w.shape[-1] if w.ndim >= 2 else w.size
        if verbose:
            print(f"  {idx + 1:>4}/{total_layers}  score={p.sensitivity_score:.2f}  {p.assigned_precision:<9} {name[:60]}")
    if target_bits is not None:
        if not measure:
            raise ValueError("a bits budget needs the measured errors (measure=True)")
        allocate_bits(profiles, target_bits, cols_of)
    orig = sum(p.vram_bytes_original for p in profiles)
    n730 = sum(p.vram_bytes_n730 for p in profiles)
    if verbose:
        print(f"  done in {time.time() - t0:.1f}s")
    return SensitivityMap(model_id=model_id, total_layers=total_layers, total_params=sum(p.param_count for p in profiles),
                          profiles=[asdict(p) for p in profiles], vram_original_mb=round(orig / 2**20, 2),
                          vram_n730_mb=round(n730 / 2**20, 2), overall_compression=round(orig / max(n730, 1), 2))


def print_summary(smap: SensitivityMap):
    counts = {}
    for p in smap.profiles:
        counts[p["assigned_precision"]] = counts.get(p["assigned_precision"], 0) + 1
    print(f"  N730 sensitivity report - {smap.model_id}")
    print(f"  tensors {smap.total_layers}, parameters {smap.total_params:,}")
    print(f"  {smap.vram_original_mb:.1f} MB fp32 -> {smap.vram_n730_mb:.1f} MB ({smap.overall_compression:.2f}x)")
    for k in CANDIDATES:
        if k in counts:
            print(f"    {k:<9} {counts[k]:>4} tensors")


def main(argv=None):
    ap = argparse.ArgumentParser(description="N730 precision profiler")
    ap.add_argument("--model", type=str, help="Hugging Face model path or hub id")
    ap.add_argument("--synthetic", action="store_true")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--target-bits", type=float, default=None, help="average bits per weight to allocate")
    ap.add_argument("--output", type=str, default="sensitivity_map.json")
    ap.add_argument("--quiet", action="store_true")
    a = ap.parse_args(argv)
    if a.model and not a.synthetic:
        model_id, layers = a.model, load_model_layers(a.model)
    else:
        model_id, layers = f"synthetic-{a.layers}L-h{a.hidden}", generate_synthetic_layers(a.layers, a.hidden, seed=0)
    smap = run_profiler(model_id, layers, verbose=not a.quiet, target_bits=a.target_bits)
    print_summary(smap)
    Path(a.output).write_text(json.dumps(asdict(smap), indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
