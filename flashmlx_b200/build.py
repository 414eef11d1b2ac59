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
SOURCES = ["route.cu", "qgemv.cu", "qgemv_tma.cu", "qgemm_tc.cu", "ep.cu", "decoder.cu", "api.cu"]
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
HOST_LIB_SOURCES = ["checkpoint.cpp", "moe_model.cpp", "decoder.cpp"]
HOST_HEADERS = ["checkpoint.hpp", "moe_model.hpp", "decoder.hpp", "device_store.hpp", "flashmoe.hpp", "json.hpp",
                "fmh.h"]
HOST_LIB = os.path.join(LIB_DIR, "libflashmoe_host.so")
HOST_EXE = os.path.join(LIB_DIR, "fm_host")


def cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc())))


def build_host(force: bool = False) -> str:
    """The C++ host layer (flashmlx_b200/host) with g++: libflashmoe_host.so (loader,
    MoEModel, Decoder and its C interface fmh.h) and the fm_host driver program, linked
    against libflashmoe.so (found next to them at run time) and the static CUDA runtime
    (its symbols kept private).  Rebuilt when a host source or a C header is newer; the
    CUDA library is built only if absent."""
    if not os.path.exists(LIB):
        build()
    deps = [os.path.join(HOST, f) for f in HOST_LIB_SOURCES + HOST_HEADERS + ["fm_host.cpp"]]
    deps.append(os.path.join(INCLUDE, "flashmoe.h"))
    outs = (HOST_LIB, HOST_EXE)
    if not force and all(os.path.exists(o) for o in outs) and \
            max(os.path.getmtime(d) for d in deps) <= min(os.path.getmtime(o) for o in outs):
        return HOST_EXE
    cuda = cuda_home()
    cxx = shutil.which("g++") or "g++"
    common = ["-std=c++17", "-O2", "-Wall", "-Wextra", "-I", INCLUDE, "-I", HOST, "-I", os.path.join(cuda, "include")]
    cudart = ["-L", os.path.join(cuda, "lib64"), "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    tmp = HOST_LIB + ".tmp"
    subprocess.check_call([cxx, *common, "-fPIC", "-shared", *[os.path.join(HOST, f) for f in HOST_LIB_SOURCES],
                           "-L", LIB_DIR, "-lflashmoe", "-Wl,-rpath,$ORIGIN", "-Wl,--exclude-libs,ALL", *cudart,
                           "-o", tmp])
    os.replace(tmp, HOST_LIB)
    tmp = HOST_EXE + ".tmp"
    subprocess.check_call([cxx, *common, os.path.join(HOST, "fm_host.cpp"), "-L", LIB_DIR, "-lflashmoe_host",
                           "-lflashmoe", "-Wl,-rpath,$ORIGIN", *cudart, "-o", tmp])
    os.replace(tmp, HOST_EXE)
    return HOST_EXE


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_host(force="--force" in sys.argv))
