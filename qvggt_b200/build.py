"""Build the sm_100a CUDA library ``libqvggt_b200.so`` in-tree.

    python -m qvggt_b200.build [-j N] [-v] [--ptxas-v]

Each ``csrc/*.cu`` is compiled with nvcc for ``compute_100a``/``sm_100a``
(``-lineinfo -O3``) into ``_build/`` and linked into
``qvggt_b200/libqvggt_b200.so``.  Only the CUDA runtime is linked; the driver
entry point used for TMA descriptors is fetched at run time through
``cudaGetDriverEntryPoint``.  Every call compiles every source from scratch
(the object directory is emptied first; a full build takes well under a
minute), so a stale object or library can never stand in for the sources.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libqvggt_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: str, extra: list[str], verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, file=sys.stderr)
    return obj


def build(jobs: int = 8, verbose: bool = False, ptxas_v: bool = False) -> str:
    if os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD)
    extra = ["-Xptxas", "-v"] if ptxas_v else []
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.v, a.ptxas_v))
