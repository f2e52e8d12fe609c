"""Build ``ancha_b200/lib/libancha_b200.so`` from ``ancha_b200/csrc`` for sm_100a.

Every ``.cu`` / ``.cpp`` source is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into ``_build/`` (object files are
reused while they are newer than every source and header), then linked as one shared
library with the CUDA runtime linked statically. The library exports exactly the C ABI of
``include/ancha_b200.h``. Run ``python -m ancha_b200.build`` (``--force`` rebuilds all).
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
OBJ = os.path.join(ROOT, "_build", "obj")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libancha_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-I" + os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(p) for p in [src] + _headers() + [__file__])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-x", "cu", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}\n{' '.join(cmd)}")
    if "warning" in r.stderr.lower():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile every source and link the shared library; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = list(extra or [])
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, extra), _sources()))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl",
               "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
