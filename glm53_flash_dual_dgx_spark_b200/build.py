"""Build the C-ABI library ``libnvfp4kv.so`` (sm_100a) in-tree with nvcc.

    python -m glm53_flash_dual_dgx_spark_b200.build [--verbose]

Objects go to ``_build/`` next to this file; the shared library is written beside the
package's Python files so it travels with the source tree.  Only sources newer than their
object are recompiled.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libnvfp4kv.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

SOURCES = ["abi_common.cu", "nvfp4_append.cu", "nvfp4_gather.cu", "nvfp4_rope.cu", "nvfp4_indexer.cu", "nvfp4_mla_decode.cu",
           "nvfp4_mla_decode_fp4.cu", "nvfp4_mla_decode_static.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", INCLUDE]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnvfp4kv.so")
    return exe


def _deps_mtime() -> float:
    newest = os.path.getmtime(os.path.join(INCLUDE, "nvfp4kv.h"))
    for f in os.listdir(CSRC):
        if f.endswith((".cuh", ".h")):
            newest = max(newest, os.path.getmtime(os.path.join(CSRC, f)))
    return newest


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    dep_t = _deps_mtime()
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), dep_t) and not ptxas_info:
            continue
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", s, "-o", o]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="rebuild everything with -Xptxas -v")
    a = ap.parse_args(argv)
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main(sys.argv[1:])
