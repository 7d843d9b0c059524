"""Builds libmsb.so (the CUDA kernels and the C ABI) in-tree with nvcc.

Usage: python moestream_b200/csrc/build.py [--force]
Output: moestream_b200/libmsb.so, compiled for sm_100a only.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
OUT = os.path.join(PKG, "libmsb.so")
BUILD = os.path.join(PKG, "_build")

SOURCES = ["host_api.cpp", "expert_cache.cpp", "pool.cu", "route.cu", "mmid.cu", "mmid_tc.cu", "mmid_f16.cu", "ep.cu", "ep_peers.cu", "gguf.cpp", "arena.cpp", "router.cu", "dstreamer.cu"]
HEADERS = ["msb_internal.h", "dcache.cuh", "expert_cache.hpp", "pool.cuh", "quant.cuh", "sm100.cuh",
           os.path.join("..", "..", "include", "msb.h")]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "-Wno-deprecated-gpu-targets"]
CU_FLAGS = ARCH + ["-lineinfo", "--expt-relaxed-constexpr"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(HERE, h) for h in HEADERS]
    objs = []
    for src in SOURCES:
        path = os.path.join(HERE, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [path] + headers):
            continue
        cmd = [NVCC] + COMMON + ["-c", path, "-o", obj]
        if src.endswith(".cu"):
            cmd += CU_FLAGS
            if verbose:
                cmd += ["-Xptxas", "-v"]
        else:
            cmd += ["-x", "c++"]
        subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        tmp = OUT + ".tmp"
        subprocess.run([NVCC] + ARCH + ["-shared", "-o", tmp] + objs, check=True)
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
