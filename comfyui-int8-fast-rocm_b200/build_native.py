"""Build libqlinear_b200.so in-tree with nvcc for sm_100a.

    python build_native.py [-j N] [--verbose] [--ptxas-v]

The CUDA sources under csrc/ are compiled in parallel into objects under
_build/ and linked into ./libqlinear_b200.so next to this file.  The CUDA
runtime is linked statically; the driver API (cuTensorMapEncodeTiled) is
reached through cudaGetDriverEntryPointByVersion, so no -lcuda is needed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqlinear_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DNDEBUG",
         # no implicit multiply-add contraction: the quantisers and epilogues
         # reproduce two-rounding float32 sequences bit for bit (explicit
         # fma / __fmaf_rn / fma.rn.f32x2 still issue fused operations)
         "-fmad=false"]
SOURCES = ["abi.cu", "rowquant.cu", "gemm.cu", "weights.cu", "dit.cu", "noalloc.cu"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(jobs: int = 8, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "qlinear_b200.h"))
    headers.append(os.path.abspath(__file__))  # a flag change rebuilds everything
    cc = nvcc()
    cmds, objs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if ptxas_v or _stale(o, [s] + headers):
            extra = ["-Xptxas", "-v"] if ptxas_v else []
            cmds.append([cc, *ARCH, *FLAGS, *extra, "-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for err in ex.map(run, cmds):
            if err and (verbose or ptxas_v):
                print(err)
    if cmds or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        run([cc, *ARCH, "-shared", "-o", tmp, *objs])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.verbose, a.ptxas_v))
    sys.exit(0)
