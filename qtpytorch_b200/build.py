"""Build the mxb CUDA library in-tree: qtpytorch_b200/libmxb.so (sm_100a).

    python -m qtpytorch_b200.build            # incremental
    python -m qtpytorch_b200.build --force    # rebuild everything

Each .cu in csrc/ compiles to an object under csrc/_build/, then one shared
library is linked.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(CSRC, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libmxb.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
         "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    objs = []
    for src in sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src[:-3] + ".o")
        objs.append(o)
        if (not force and os.path.exists(o)
                and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr)):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if (force or not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
