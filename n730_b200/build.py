"""Build the native libraries in-tree.

    python -m n730_b200.build [--clean] [-j N]

Outputs (git-ignored, shipped with the source tree):
  n730_b200/lib/n730_cuda.so  - sm_100a kernels + the C ABI (include/n730_cuda.h)
  n730_b200/lib/n730core.so   - the .n730 file reader / CPU dequant core (include/n730core.h)

nvcc compiles every ``csrc/*.cu`` for ``-gencode arch=compute_100a,code=sm_100a``
only (B200); objects are cached under ``_build/`` keyed by source and header
mtimes.  NCCL comes from the wheel that PyTorch uses, linked by rpath, so the
process holds a single NCCL.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
BUILD = REPO / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I", str(CSRC), "-I", str(REPO / "include")]


def _nccl_dirs():
    try:
        import nvidia.nccl as m  # the NCCL wheel PyTorch loads
        base = Path(list(m.__path__)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    except Exception:
        pass
    return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")


def _stale(obj: Path, src: Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in [src, *deps])


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"command failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(jobs: int = 0, verbose: bool = False, ptxas_info: bool = False) -> dict:
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    nccl_inc, nccl_lib = _nccl_dirs()
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))
    srcs = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    logs = {}

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        if not ptxas_info and not _stale(obj, src, headers):
            return obj, ""
        cmd = [NVCC, *ARCH, *NVCC_FLAGS, *extra, "-I", str(nccl_inc), "-c", str(src), "-o", str(obj)]
        return obj, _run(cmd)

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        results = list(ex.map(compile_one, srcs))
    objs = [o for o, _ in results]
    for (o, log), s in zip(results, srcs):
        if log:
            logs[s.name] = log
    so = LIB / "n730_cuda.so"
    _run([NVCC, *ARCH, "-shared", "-o", str(so), *map(str, objs), "-cudart", "static",
          "-L", str(nccl_lib), "-l:libnccl.so.2", f"-Xlinker=-rpath,{nccl_lib}", "-lpthread", "-ldl"])
    core = LIB / "n730core.so"
    core_src = CSRC / "core_io.cpp"
    if core_src.exists() and _stale(core, core_src, headers):
        _run(["g++", "-O3", "-march=x86-64-v3", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", "-fvisibility=hidden",
              "-I", str(REPO / "include"), "-o", str(core), str(core_src), "-lpthread"])
    if verbose:
        for k, v in logs.items():
            print(f"== {k}\n{v}")
    return logs


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args(argv)
    if a.clean and BUILD.exists():
        shutil.rmtree(BUILD)
    build(a.j, a.v, a.ptxas_info)
    print("built", sorted(p.name for p in LIB.glob("*.so")))
    return 0


if __name__ == "__main__":
    sys.exit(main())
