"""Build libmpo_b200.so (the sm_100a kernels behind mps_pointops) in place.

    python mps-pointops_b200/build.py            # incremental
    python mps-pointops_b200/build.py --clean    # from scratch

Every .cu under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo, -O3 and
-fmad=false (no floating-point contraction: the kernels must reproduce the
reference's separately rounded arithmetic), and linked into
mps_pointops/_lib/libmpo_b200.so next to the Python package, which loads it
with ctypes.  Objects go to mps-pointops_b200/_build/.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OBJ = HERE / "_build"
LIB_DIR = HERE / "mps_pointops" / "_lib"
LIB = LIB_DIR / "libmpo_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _deps(src: Path) -> list[Path]:
    return [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def build(clean: bool = False, verbose: bool = False) -> Path:
    if clean and OBJ.exists():
        shutil.rmtree(OBJ)
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    compiler = nvcc()
    sources = sorted(CSRC.glob("*.cu"))
    objects = []
    jobs = []
    for src in sources:
        obj = OBJ / (src.stem + ".o")
        objects.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(p.stat().st_mtime for p in _deps(src)):
            continue
        jobs.append([compiler, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{res.stdout}{res.stderr}")
        return res

    with ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        list(pool.map(run, jobs))
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        tmp = LIB.with_suffix(".so.tmp")
        run([compiler, *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(clean="--clean" in sys.argv, verbose="-v" in sys.argv))
