"""Builds the engine's shared library in-tree: varblockspmm_b200/libvbsr_b200.so (sm_100a).

Run `python varblockspmm_b200/build.py` or call build() (__graft_entry__.build() does both this
and the oracle). nvcc cross-compiles for sm_100a, so this
works on a machine without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvbsr_b200.so")
CXXLIB = os.path.join(HERE, "libvbsr_b200_cxx.so")

CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", CUDA + "/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [*os.environ.get("VBSR_EXTRA_FLAGS", "").split(),
          "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall",
          "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]

SOURCES = ["vbsr_host.cpp", "vbsr_device.cu", "vbsr_multi.cpp", "vbsr_io.cpp"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "vbsr_b200.h"))
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if _stale(o, [s] + headers) or ptxas_info:
            extra = ["-Xptxas", "-v"] if (ptxas_info and src.endswith(".cu")) else []
            jobs.append([NVCC, *ARCH, *COMMON, *extra, "-c", s, "-o", o])
    log = ""
    with ThreadPoolExecutor(max_workers=4) as ex:
        for out in ex.map(_run, jobs):
            log += out
    if _stale(LIB, objs):
        log += _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lpthread"])
    # C++ drop-in API (include/varblockspmm/vbsr.hpp) over the C ABI
    # (with the library comparator plans on cuSPARSE / cuBLAS)
    cxx_srcs = [os.path.join(CSRC, f) for f in ("vbsr_api.cpp", "vbsr_comparators.cpp")]
    hdr = [os.path.join(ROOT, "include", "varblockspmm", "vbsr.hpp")] + headers
    if _stale(CXXLIB, cxx_srcs + [LIB] + hdr):
        log += _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall",
                     "-I" + os.path.join(ROOT, "include"), "-I" + CUDA + "/include",
                     *cxx_srcs, "-o", CXXLIB, "-L" + HERE, "-lvbsr_b200",
                     "-L" + CUDA + "/lib64", "-lcusparse", "-lcublas", "-lcudart",
                     "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + CUDA + "/lib64"])
    if verbose and log:
        print(log)
    return log


if __name__ == "__main__":
    print(build(verbose=False, ptxas_info="-v" in sys.argv) or "ok")
