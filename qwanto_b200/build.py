"""Build qwn_cuda.so in-tree for sm_100a (B200).

The library is the drop-in boundary: the reference's qwnrun dlopen()s a file
named qwn_cuda.so from its own directory, so the product is built under that
name.  nvcc cross-compiles here without a GPU; the .so travels with the tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "qwn_cuda.so")

SOURCES = ["kv_pool.cu", "kv_attention.cu", "kv_evict.cu", "abi_v1.cu", "linear_attention.cu", "ref_api.cu"]
HEADERS = [os.path.join(CSRC, "kv_internal.cuh"), os.path.join(CSRC, "kv_store.cuh")] + [
    os.path.join(INCLUDE, h) for h in ("qwn_cuda_abi.h", "qwn_kv_b200.h", "qwn_paged_kv.h", "qwanto_turboquant.h",
                                       "qwanto_attention.h", "qwanto_pagedeviction.h")]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: the codecs depend on IEEE division and rounding.
FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                "-I", INCLUDE, "-I", CSRC, "-DQWN_CUDA_BUILDING_DLL"]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, ptxas_v: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if _stale(obj, [path] + HEADERS) or ptxas_v:
        cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + ["-c", path, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if ptxas_v:
            sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_v), SOURCES))
    if _stale(LIB, objs):
        # -Bsymbolic: calls inside the library bind to its own definitions even
        # when the host program defines the same reference-named symbols
        cmd = [NVCC] + ARCH + ["-shared", "-Xlinker", "-Bsymbolic", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_v="-v" in sys.argv)
    print(LIB)
