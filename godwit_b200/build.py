"""Builds the in-tree shared libraries.

  godwit_b200/libgodwit_cuda.so   the product: sm_100a kernels + the C-ABI of
                                  include/godwit_cuda.h (static cudart, no torch)
  oracle/liboracle.so             the CPU restatement used only by tests, the
                                  smoke check and bench.py's CPU-baseline leg

Both are rebuilt only when a source is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "godwit_b200")
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libgodwit_cuda.so")
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_LIB = os.path.join(ORACLE_DIR, "liboracle.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr"]
CU_SOURCES = ["gw_kernels.cu", "gw_gemv.cu", "gw_grouped.cu", "gw_int8.cu", "gw_ep.cu", "gw_api.cu"]
HEADERS = ["gw_device.cuh", "gw_internal.h", "gw_async.cuh"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES + HEADERS]
    srcs.append(os.path.join(ROOT, "include", "godwit_cuda.h"))
    if not force and not _stale(LIB, srcs):
        return LIB
    nvcc = _nvcc()
    objdir = os.path.join(ROOT, "_build")
    os.makedirs(objdir, exist_ok=True)
    from concurrent.futures import ThreadPoolExecutor

    def compile_one(s: str) -> str:
        obj = os.path.join(objdir, s.replace(".cu", ".o"))
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", os.path.join(CSRC, s), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as pool:  # one nvcc per source file
        objs = list(pool.map(compile_one, CU_SOURCES))
    tmp = LIB + ".tmp"
    subprocess.run([nvcc, *ARCH, "-shared", *objs, "-o", tmp], check=True)
    os.replace(tmp, LIB)
    return LIB


def build_oracle(force: bool = False) -> str:
    src = os.path.join(ORACLE_DIR, "mxfp4_oracle.c")
    if not force and not _stale(ORACLE_LIB, [src]):
        return ORACLE_LIB
    tmp = ORACLE_LIB + ".tmp"
    # -O2 without -ffast-math keeps IEEE fp32 semantics; -fno-tree-vectorize
    # keeps the reference's sequential accumulation order.
    subprocess.run(["gcc", "-O2", "-fno-tree-vectorize", "-fPIC", "-shared", "-pthread",
                    src, "-o", tmp, "-lm"], check=True)
    os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_cuda(force=force, verbose="-v" in sys.argv))
    print(build_oracle(force=force))
