"""Build libaeth_galore.so (sm_100a) in-tree with nvcc.

    python aethelstream_b200/build.py [--force] [--verbose]

Run it as a script (or load it by file path): importing the package itself
requires the built library.

The library is a single translation unit (csrc/aeth_galore.cu) linked against
the static CUDA runtime, so it only needs the driver on the machine that loads
it.  No fast-math: the NF4/INT8 codes and the REF-mode arithmetic must round
exactly like the CPU definition.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libaeth_galore.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-ffp-contract=off",
    "-shared", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  [os.path.join(ROOT, "include", "aeth_galore.h")])


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-I", os.path.join(ROOT, "include"),
           os.path.join(CSRC, "aeth_galore.cu"), "-o", LIB + ".tmp"]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libaeth_galore.so")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print per-kernel register/smem usage")
    a = ap.parse_args()
    build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=["-Xptxas", "-v"] if a.ptxas_v else None)
    print(LIB)
