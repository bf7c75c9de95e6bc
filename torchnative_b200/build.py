"""Build libtorchnative_b200.so in-tree from csrc/*.cu for sm_100a.

    python -m torchnative_b200.build [--force]

nvcc compiles each translation unit for `-gencode arch=compute_100a,code=sm_100a`
(cross-compiles without a GPU) with the CUDA runtime linked statically, so the
library loads on a machine without a driver and exports only the C ABI
declared in include/torchnative_b200.h.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libtorchnative_b200.so")
HEADER = os.path.join(ROOT, "include", "torchnative_b200.h")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", "-DTN_BUILD"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [HEADER]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def _compile(src: str, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources()))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="--ptxas-v" in sys.argv)
    print(LIB)
