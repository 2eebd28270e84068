"""Build libdsalt_b200.so (sm_100a) in-tree: dsalt/_lib/libdsalt_b200.so.

    python dsalt-library_b200/build.py [--jobs N] [--verbose]

Every ``csrc/*.cu`` is compiled with ``-gencode arch=compute_100a,code=sm_100a``
and linked into one shared library with the C ABI of ``include/dsalt_b200.h``.
nvcc cross-compiles, so no GPU is needed to build.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
OUT_DIR = HERE / "dsalt" / "_lib"
OBJ_DIR = HERE / "_build"
LIB = OUT_DIR / "libdsalt_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: Path, extra: list[str], verbose: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    deps = [src] + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "dsalt_b200.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, flush=True)
    return obj


def build(jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra or [], verbose), srcs))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose or a.ptxas_v, ["-Xptxas", "-v"] if a.ptxas_v else None))
