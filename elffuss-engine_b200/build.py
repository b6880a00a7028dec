"""Build libelffuss_cuda.so (sm_100a) in-tree with nvcc.

    python elffuss-engine_b200/build.py [--verbose] [--ptxas-info] [--trace]

Steps: generate csrc/gen/iq_grids.h from gguf-py (the IQ2_XXS / IQ1_S
codebooks), then compile every csrc/*.cu for sm_100a and link one shared
library next to this file. Rebuilds only when a source is newer than the .so.
--trace also links libelffuss_cuda_trace.so: the same library with the GEMV
kernel's launch-phase timestamps compiled in (-DEF_GEMV_TRACE), for
`bench.py --gemv-trace` only.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
GEN = os.path.join(CSRC, "gen", "iq_grids.h")
LIB = os.path.join(HERE, "libelffuss_cuda.so")
TRACE_LIB = os.path.join(HERE, "libelffuss_cuda_trace.so")
OBJ = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False, trace: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    gen_script = os.path.join(CSRC, "gen_grids.py")
    if force or _newer(GEN, [gen_script]):
        subprocess.run([sys.executable, gen_script, GEN], check=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [GEN] + \
        glob.glob(os.path.join(HERE, "..", "include", "*.h"))
    objs = []
    for src in sources():
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    if force or _newer(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if trace:
        src = os.path.join(CSRC, "gemv.cu")
        tobj = os.path.join(OBJ, "gemv_trace.o")
        if force or _newer(tobj, [src] + headers):
            subprocess.run([NVCC, *ARCH, *FLAGS, "-DEF_GEMV_TRACE", "-c", src, "-o", tobj], check=True)
        tobjs = [tobj if o.endswith(os.sep + "gemv.o") else o for o in objs]
        if force or _newer(TRACE_LIB, tobjs):
            subprocess.run([NVCC, *ARCH, "-shared", "-o", TRACE_LIB, *tobjs, "-lcudart_static"], check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--trace", action="store_true", help="also link the launch-phase trace library")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info, a.force, a.trace))
