"""Precision profiler (n730_b200.profiler): the reference's sensitivity score, pinned to the
reference profiler's own outputs (tests/golden/ref_profiler.npz, written by
tests/golden/make_golden.py from src-code/profiler.py), and the group-wise assignment."""
import importlib.util
import math
from pathlib import Path

import numpy as np
import pytest

from n730_b200 import profiler as P
from n730_b200 import synthetic
from n730_b200.formats import read_header

GOLDEN = Path(__file__).resolve().parent / "golden"
_spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


def test_sensitivity_matches_reference_profiler():
    g = np.load(GOLDEN / "ref_profiler.npz")
    for case, score, kurt, outl in zip(make_golden.profiler_cases(), g["scores"], g["kurtosis"], g["outlier_ratio"]):
        w = make_golden.profiler_tensor(*case[:5])
        assert P.compute_sensitivity(w, case[5], case[6]) == pytest.approx(score, abs=1e-12), case
        p = P.profile_weight_tensor(w, case[5], "t", case[6], measure=False)
        assert p.weight_kurtosis == pytest.approx(kurt, abs=1e-4) and p.outlier_ratio == pytest.approx(outl, abs=1e-6)


def test_quant_error_orders_candidates():
    w = np.random.default_rng(0).normal(0, 0.02, (300, 512)).astype(np.float32)
    e = [P.quant_error(w, c) for c in P.CANDIDATES]
    assert e == sorted(e, reverse=True)          # more bits, smaller error
    assert 0.4 < e[0] < 0.55 and 0.08 < e[1] < 0.13 and e[2] < 0.01 and e[3] < 1e-3
    assert math.isinf(P.quant_error(np.ones((4, 96), np.float32), "INT4G128"))  # 96 columns: no g128 tiling
    assert P.quant_error(np.zeros((4, 128), np.float32), "INT2G64") == 0.0


def test_assignment_is_monotone_in_sensitivity():
    errs = {"INT2G64": 0.47, "INT4G128": 0.11, "INT8PC": 0.007, "FP16": 0.0002}
    order = {c: i for i, c in enumerate(P.CANDIDATES)}
    picks = [P.assign_precision(s, "model.layers.3.mlp.up_proj.weight", errs) for s in np.linspace(0, 1, 21)]
    assert [order[p] for p in picks] == sorted(order[p] for p in picks)
    assert picks[0] == "INT2G64" and picks[-1] == "FP16"
    assert P.assign_precision(0.0, "lm_head.weight", errs) == "INT4G128"  # embeddings / lm_head floor


def test_budget_allocation_and_convert(tmp_path):
    shape = synthetic.SHAPES["tiny"]
    tensors = [(n, w) for n, w in synthetic.host_tensors(shape, seed=4) if w.ndim == 2]
    for target in (3.5, 4.25, 6.0):  # below ~3.03 the floors (embedding, lm_head at INT4) decide
        smap = P.run_profiler("tiny", tensors, verbose=False, target_bits=target)
        bits = sum(p["bits_per_weight"] * p["param_count"] for p in smap.profiles) / smap.total_params
        assert bits <= target + 1e-9
        assert target - bits < 8.0  # the budget is used up to one upgrade
    # the map's precision strings are the converter's: the file holds what was assigned
    from dataclasses import asdict
    from n730_b200.converter import convert
    smap = asdict(P.run_profiler("tiny", tensors, verbose=False, target_bits=4.25))
    convert(iter(tensors), smap, tmp_path / "m.n730", verbose=False)
    ids = {"INT2G64": 0x42, "INT4G128": 0x44, "INT8PC": 0x48, "FP16": 16}
    want = {p["layer_name"]: ids[p["assigned_precision"]] for p in smap["profiles"]}
    got = {e["layer_name"]: e["precision"] for e in read_header(tmp_path / "m.n730")["seek_table"]}
    names = {"INT2G": 0x42, "INT4G": 0x44, "INT8G": 0x48, "FP16": 16}
    assert {k: names.get(v, v) for k, v in got.items()} == want


def test_synthetic_layers_follow_the_reference_pattern():
    layers = P.generate_synthetic_layers(20, 256, seed=0)
    smap = P.run_profiler("s", layers, verbose=False)
    s = [p["sensitivity_score"] for p in smap.profiles]
    assert s[-1] > 0.7 and s[10] < 0.2       # outlier-heavy last layers score high, middle ones low
    assert smap.profiles[-1]["assigned_precision"] in ("INT8PC", "FP16")
