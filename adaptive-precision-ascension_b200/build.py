"""Build libapa_kernels.so in-tree for sm_100a.

    python adaptive-precision-ascension_b200/build.py [--force] [--checks]

Compiles csrc/apa_kernels.cu (which includes the cast, GEMM and ladder
kernels) with nvcc for ``compute_100a``/``sm_100a`` into
``apa/libapa_kernels.so`` next to the Python package. Rebuilds only when a
source or header is newer than the library (or with --force).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "apa", "libapa_kernels.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if not force and not needs_build():
        return OUT
    cmd = [NVCC, *FLAGS, *extra, os.path.join(CSRC, "apa_kernels.cu"), "-o", OUT + ".tmp"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libapa_kernels.so")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else []
    print(build(force="--force" in sys.argv, verbose=True, extra=extra))
