"""Build recipe of the in-tree CUDA library ``recant_b200/_lib/librecant_b200.so``.

Plain nvcc, sm_100a only:  python -m recant_b200.build  [--force]
Each ``csrc/*.cu`` compiles to ``_build/<name>.o`` (in parallel), then links into one
shared library with a static CUDA runtime, so the library has no dependency on torch.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(OUT_DIR, "librecant_b200.so")
BUILD = os.path.join(ROOT, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, extra):
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr[-4000:]}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    jobs = []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if force or _stale(obj, [s, *hdrs]):
            jobs.append((s, obj))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for msg in ex.map(lambda j: _compile(j[0], j[1], list(extra)), jobs):
            if verbose and msg:
                print(msg)
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    return LIB


if __name__ == "__main__":
    extra = [a for a in sys.argv[1:] if a.startswith("-X") or a.startswith("-D")]
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, extra=extra))
