"""Build recipe for libvfr_retrieval.so (sm_100a only).

Compiles every csrc/*.cu and csrc/*.cpp with nvcc for
`-gencode arch=compute_100a,code=sm_100a` and links one shared library next to
this file, so it travels with the source tree.  Incremental: an object is
rebuilt when its source or any csrc header is newer.  Usage:
    python vocal-fast-rs_b200/build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvfr_retrieval.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", CSRC,
          "-I", os.path.join(HERE, "..", "include")]
CUFLAGS = ["--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    hs.append(os.path.join(HERE, "..", "include", "vfr_retrieval.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src: str, force: bool, verbose: bool, ptxas_v: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()):
        return obj
    cmd = [NVCC, *ARCH, *COMMON]
    if src.endswith(".cu"):
        cmd += CUFLAGS
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
    cmd += ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if (verbose or ptxas_v) and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose, ptxas_v), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        # No -lcuda: driver entry points (cuTensorMapEncodeTiled) are resolved at
        # run time through cudaGetDriverEntryPoint, so the library also loads on
        # a host without a GPU driver (the CPU test suite checks its exports).
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xlinker", "--no-undefined"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_v))
