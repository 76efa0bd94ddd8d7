"""Builds libpp_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python pop2-bezier_b200/build_native.py [--force] [--verbose]

Objects go to pop2-bezier_b200/_build/ and the library to
pop2-bezier_b200/libpp_b200.so, so the built file travels with the working
tree.  quant.cu is compiled with -fmad=false / -prec-div=true: its divisions
and products must round exactly as the reference's quantizer does.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpp_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "-I", os.path.join(ROOT, "include")]

SOURCES = [
    ("csrc/kernels/quant.cu", ["-fmad=false", "-prec-div=true", "-prec-sqrt=true"]),
    ("csrc/kernels/attention.cu", []),
    ("csrc/kernels/attention_static.cu", []),
    ("csrc/kernels/decoder.cu", ["-fmad=false", "-prec-div=true", "-prec-sqrt=true"]),
    ("csrc/kernels/sampling.cu", ["-fmad=false", "-prec-div=true", "-prec-sqrt=true"]),
    ("csrc/kernels/lanes.cu", []),
    ("csrc/host/abi.cpp", []),
    ("csrc/host/sched.cpp", []),
    ("csrc/host/selfcheck.cpp", []),
]
HEADERS = ["csrc/kernels/common.cuh", "csrc/kernels/quant_row.cuh", "csrc/kernels/lanes.cuh", "csrc/host/internal.h"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _mtime(path: str) -> float:
    return os.path.getmtime(path) if os.path.exists(path) else 0.0


def _newest_dep() -> float:
    deps = [os.path.join(HERE, h) for h in HEADERS] + [os.path.join(ROOT, "include", "pp_b200.h")]
    return max(_mtime(p) for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    dep_time = _newest_dep()
    jobs = []
    objs = []
    for src, extra in SOURCES:
        src_path = os.path.join(HERE, src)
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _mtime(obj) < max(_mtime(src_path), dep_time, _mtime(__file__)):
            cmd = [nv, *ARCH, *COMMON, *extra, "-c", src_path, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [nv, *COMMON, *extra, "-x", "cu", *ARCH, "-c", src_path, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if jobs or force or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        link = [nv, *ARCH, "-shared", "-cudart", "shared", "-o", tmp, *objs]
        run(link)
        os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
