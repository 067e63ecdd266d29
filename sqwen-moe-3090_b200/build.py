"""Build libsqmix.so (CUDA kernels + C ABI) for sm_100a with nvcc, in-tree.

    python sqwen-moe-3090_b200/build.py [--ptxas-verbose]

Objects go to ``_build/`` beside this file; the shared library is written to
``sqmix/libsqmix.so`` so that the host package loads it from the source tree.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "sqmix", "libsqmix.so")
INCLUDE = os.path.join(REPO, "include")

SOURCES = ["host.cpp", "abi.cpp", "ggml_bridge.cpp", "kv_append.cu", "fa_decode.cu", "fa_prefill.cu", "gdn.cu", "gdn_chunk.cu", "gdn_front.cu",
           "gdn_layer.cu", "peer_merge.cu", "mul_mat.cu", "mul_mat_gemm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "sqmix.h"))
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        if not force and not verbose_ptxas and not _stale(obj, [path] + headers):
            continue
        cmd = [nvcc()] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else [])
        if src.endswith(".cpp"):
            cmd += ["-x", "cu"]
        cmd += ["-c", path, "-o", obj]
        print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", OUT] + objs + ["-cudart", "static"]
        print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(args.ptxas_verbose, args.force))
    sys.exit(0)
