"""Build libtrixium_b200.so (sm_100a) in-tree with nvcc.

    python -m trixium_b200.build [--force] [--verbose]

The library links only the CUDA runtime: it takes raw device pointers and a cudaStream_t, so
it has no dependency on torch.  The .so is written next to this file and is what
trixium_b200/_lib.py loads.
"""

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtrixium_b200.so")
BUILD = os.path.join(ROOT, "_build", "trixium_b200")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "trixium_b200.h")]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found")
    return exe


def stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, ptxas_v=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    hdrs = headers()
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or stale(o, [s] + hdrs):
            cmd = [nvcc()] + ARCH + FLAGS + ["-I", os.path.join(ROOT, "include"), "-c", s, "-o", o]
            if ptxas_v:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))


if __name__ == "__main__":
    sys.exit(main())
