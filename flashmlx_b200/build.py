"""Builds libflashmoe.so (the C-ABI library) in-tree with nvcc for sm_100a, and the C++
host layer's driver program fm_host (flashmlx_b200/host) with g++.

    python -m flashmlx_b200.build [--force]

The library links the CUDA runtime statically, so it neither depends on nor clashes
with the runtime bundled by other frameworks in the same process.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libflashmoe.so")
SOURCES = ["route.cu", "qgemv.cu", "qgemm_tc.cu", "ep.cu", "api.cu"]
HEADERS = ["fm_common.cuh", "fm_internal.cuh", "fm_ep.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-DFM_BUILD"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "flashmoe.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static"])
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


HOST = os.path.join(PKG, "host")
HOST_SOURCES = ["checkpoint.cpp", "moe_model.cpp", "fm_host.cpp"]
HOST_HEADERS = ["checkpoint.hpp", "moe_model.hpp", "flashmoe.hpp", "json.hpp"]
HOST_EXE = os.path.join(LIB_DIR, "fm_host")


def cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def build_host(force: bool = False) -> str:
    """The C++ host layer's driver program (flashmlx_b200/host): g++, linked against
    libflashmoe.so (found next to it at run time) and the static CUDA runtime.  Rebuilt
    when a host source or the C header is newer; the CUDA library is built only if absent."""
    if not os.path.exists(LIB):
        build()
    deps = [os.path.join(HOST, f) for f in HOST_SOURCES + HOST_HEADERS] + [os.path.join(INCLUDE, "flashmoe.h")]
    if not force and os.path.exists(HOST_EXE) and all(os.path.getmtime(d) <= os.path.getmtime(HOST_EXE) for d in deps):
        return HOST_EXE
    cuda = cuda_home()
    tmp = HOST_EXE + ".tmp"
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-I", INCLUDE, "-I", HOST,
           "-I", os.path.join(cuda, "include"), *[os.path.join(HOST, f) for f in HOST_SOURCES],
           "-L", LIB_DIR, "-lflashmoe", "-Wl,-rpath,$ORIGIN", "-L", os.path.join(cuda, "lib64"), "-lcudart_static",
           "-ldl", "-lpthread", "-lrt", "-o", tmp]
    subprocess.check_call(cmd)
    os.replace(tmp, HOST_EXE)
    return HOST_EXE


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_host(force="--force" in sys.argv))
