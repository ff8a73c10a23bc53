"""Builds libtritier_b200.so (sm_100a) in-tree with nvcc.

    python -m tritiercache_b200.csrc.build        # or build() from Python

Flags: -gencode arch=compute_100a,code=sm_100a, -O3, -lineinfo, no fast-math
(IEEE division and correctly rounded conversions are part of the bit-exact
quantize contract).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
SOURCES = ["tt_api.cu", "tt_attn.cu", "tt_engine.cu", "tt_noalloc.cu"]
# every header in this directory (and the C ABI header) is a dependency of
# every object: editing any of them rebuilds all sources
HEADERS = sorted(os.path.basename(h) for h in glob.glob(os.path.join(HERE, "*.cuh"))) + \
    [os.path.join("..", "..", "include", "tritier_b200.h")]
LIB = os.path.join(PKG, "libtritier_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    hdrs = [os.path.join(HERE, h) for h in HEADERS]
    objs = []
    procs = []
    for src in SOURCES:
        sp = os.path.join(HERE, src)
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [sp] + hdrs):
            cmd = [NVCC] + FLAGS + ["-c", sp, "-o", obj]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + out.decode(errors="replace"))
        if verbose and out:
            print(out.decode(errors="replace"), file=sys.stderr)
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs + ["-lcudart"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
