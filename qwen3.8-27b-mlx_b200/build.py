"""Build recipe of the GDN CUDA library (sm_100a), used by
``__graft_entry__.build()`` and runnable by hand:

    python qwen3.8-27b-mlx_b200/build.py [--force] [-D NAME=VALUE ...]

Compiles every ``csrc/*.cu`` and ``csrc/*.cpp`` with nvcc into object files
under ``_build/`` and links them into ``libgdn_b200.so`` next to this file, so
the library lives in-tree and travels with the repository snapshot.
Recompiles only sources (or headers) newer than their object file.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgdn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def build(force: bool = False, defines=(), out: str = LIB, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    tag = "_".join(d.replace("=", "-") for d in defines)
    objdir = os.path.join(BUILD, tag) if tag else BUILD
    os.makedirs(objdir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    hdr = _newest_header()
    common = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC]
    common += [f"-D{d}" for d in defines]
    objs, changed = [], force
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            cmd = [nvcc(), *common, *ARCH, "-c", s, "-o", o]
            if s.endswith(".cu"):
                cmd[1:1] = ["-Xptxas", "-v"] if verbose else []
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
            changed = True
    if changed or not os.path.exists(out):
        cmd = [nvcc(), "-shared", *ARCH, "-o", out, *objs, "-lcuda"]
        subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-D", dest="defines", action="append", default=[])
    ap.add_argument("--out", default=LIB)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.defines, a.out, a.verbose))
    sys.exit(0)
