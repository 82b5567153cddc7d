"""Build libib_cuda.so in-tree for sm_100a.

Each CUDA/C++ source is compiled to an object under _build/ (skipped when up to
date), then linked into inference.cpp_b200/libib_cuda.so.  The CUDA runtime is
linked statically so the library does not depend on which libcudart another
component of the process loaded.

    python inference.cpp_b200/build.py [-j N] [--force]
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
LIB = os.path.join(HERE, "libib_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-ffp-contract=off", "-I" + CSRC, "-I" + INCLUDE,
          "--expt-relaxed-constexpr"]
# per-source extra flags
EXTRA = {
    "synth.cu": ["-fmad=false"],
}


def sources() -> list[str]:
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime() -> float:
    m = 0.0
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return p


def compile_one(src: str, force: bool, hdr_m: float) -> tuple[str, str]:
    obj = os.path.join(BUILD, src + ".o")
    s = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(s), hdr_m)):
        return obj, ""
    cmd = [nvcc()] + ARCH + COMMON + EXTRA.get(src, []) + ["-c", s, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), "-x", "cu"] + ARCH + COMMON + EXTRA.get(src, []) + ["-c", s, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(jobs: int = 0, force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    hdr_m = headers_mtime()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: compile_one(s, force, hdr_m), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for o, log in results:
            if log:
                print(log, file=sys.stderr)
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.force, a.v))
