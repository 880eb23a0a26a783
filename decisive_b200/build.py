"""Builds libdecisive_b200.so in-tree with nvcc for sm_100a (the only target).

Usage: python -m decisive_b200.build [--force] [--verbose]
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
LIB = os.path.join(HERE, "libdecisive_b200.so")
SOURCES = ["gemm_i8_q4.cu", "gemm_i8_q8.cu", "gemm_i8_swiglu.cu", "gemm_i8.cu", "quant.cu", "gemm_tc.cu", "gemv.cu", "layer_ops.cu", "attention_tc.cu", "capi.cu", "model.cu", "noalloc.cu",
           "tuner.cu", "packed_io.cu", "bert.cu", "decima_w8a32.cu", "gemm_dq.cu"]
HEADERS = ["gemm_i8.cuh", "common.cuh", "kernels.h", "layer_ops.h", "capi_internal.h", "packed_io.h"]
PUBLIC_HEADER = os.path.join(os.path.dirname(HERE), "include", "decisive_b200.h")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def host_compiler() -> list[str]:
    # /usr/bin/g++ is the system compiler the CUDA toolkit supports in this image
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths if os.path.exists(p))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    cmd = [nvcc(), *host_compiler(), *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [PUBLIC_HEADER]
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest(deps):
        return LIB
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    cmd = [nvcc(), *host_compiler(), *ARCH, "-shared", "-o", LIB, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
