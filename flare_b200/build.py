"""Builds libflare_b200.so in-tree (flare_b200/) for sm_100a with nvcc.

    python -m flare_b200.build          # incremental
    python -m flare_b200.build --force  # rebuild everything
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libflare_b200.so")
SOURCES = ["api.cu", "bvh.cu", "bvh4.cu", "ploc.cu", "trace.cu", "shade.cu", "viewer.cu", "optim.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "renderer.cuh", "umma.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr"]


def _mtime(p):
    return os.path.getmtime(p) if os.path.exists(p) else 0.0


def build(force: bool = False, verbose: bool = False, extra=None) -> str:
    os.makedirs(OBJ, exist_ok=True)
    hdr_t = max(_mtime(os.path.join(CSRC, h)) for h in HEADERS)
    hdr_t = max(hdr_t, _mtime(os.path.join(HERE, "..", "include", "flare_b200.h")))
    objs = []
    changed = force
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _mtime(o) < max(_mtime(s), hdr_t):
            cmd = [NVCC, *FLAGS, *(extra or []), "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
            changed = True
    if changed or not os.path.exists(LIB):
        # export only the C ABI: api.cu marks nothing hidden-visible except via the version script below
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", *objs, "-o", LIB,
               "-Xlinker", f"--version-script={os.path.join(CSRC, 'exports.map')}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
    print(LIB)
