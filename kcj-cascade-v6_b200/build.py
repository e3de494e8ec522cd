"""Build of the sm_100a C-ABI library ``cascade_cpp/libcascade_b200.so``.

Plain nvcc, in-tree: objects go to ``_build/`` beside this file and the
shared library next to the Python package that loads it, so the library
travels with the source tree. Rebuilds only what changed.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "cascade_cpp", "libcascade_b200.so")

SOURCES = ["sha256.cu", "copy.cu", "kvquant.cu", "index.cu", "store.cu", "pipeline.cu", "dht.cu", "policy.cpp",
           "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def nccl_paths() -> tuple[str, str]:
    """Include and lib dirs of the NCCL that torch itself loads."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    if spec and spec.submodule_search_locations:
        for base in spec.submodule_search_locations:
            inc = os.path.join(base, "nccl", "include")
            lib = os.path.join(base, "nccl", "lib")
            if os.path.exists(os.path.join(inc, "nccl.h")):
                return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".hpp", ".h"))]
    hs.append(os.path.join(INCLUDE, "cascade_b200.h"))
    return hs


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    nccl_inc, nccl_lib = nccl_paths()
    hdr_mtime = max(os.path.getmtime(h) for h in _headers())
    common = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              f"-I{INCLUDE}", f"-I{CSRC}", f"-I{nccl_inc}"]
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), hdr_mtime):
            continue
        cmd = [nvcc, *ARCH, *common, "-c", path, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [nvcc, *ARCH, *common, "-x", "c++", "-c", path, "-o", obj]
        elif ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose or ptxas_info)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, f"-L{nccl_lib}", "-l:libnccl.so.2",
               f"-Xlinker=-rpath,{nccl_lib}"]
        _run(cmd, verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv))
