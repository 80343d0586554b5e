"""The benchmark's reference arm (``bench.py --impl reference``) on the host CPU.

The arm times the reference's own CPU decode path (its ``n730_read_layer``
core, built from its sources into ``oracle/_ref``, plus numpy GEMVs) for whole
tokens; here it runs on a one-layer cut of the 7B shape at a short context, so
the check of its output line takes seconds.  A rank other than 0 under a
multi-process launch prints nothing and exits 0.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

REF_CORE = REPO / "oracle" / "_ref" / "n730core.so"


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", *args],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(not REF_CORE.exists(), reason="oracle/_ref/n730core.so is built by __graft_entry__.build()")
def test_reference_arm_line():
    p = _run({}, "--layers", "1", "--ctx", "64", "--steps", "2", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    import bench
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and 1 <= d["steps"] <= 2
    # one token per step at batch 1: the rate and the step time describe the same run
    assert abs(d["value"] * d["ms_per_step"] / 1000.0 - 1.0) < 0.01
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["unit"] == "tok/s"
    assert cb["cores"] == len(os.sched_getaffinity(0)) and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["ctx"] == 64 and "1 layers" in d["config"]["workload"]


def test_reference_arm_other_rank_is_silent():
    p = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, "--steps", "2", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
