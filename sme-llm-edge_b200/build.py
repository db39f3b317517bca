"""Builds libspecdec_sm100.so (sm_100a) in-tree with nvcc.

    python sme-llm-edge_b200/build.py            # incremental
    python sme-llm-edge_b200/build.py --clean

Objects go to sme-llm-edge_b200/_build/, the library to
sme-llm-edge_b200/specdec/libspecdec_sm100.so (both git-ignored; the .so
travels with the source tree to the GPU host).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "specdec", "libspecdec_sm100.so")
SOURCES = ["runtime.cu", "sampling.cu", "kvcache.cu", "attention.cu", "gemm_w4a16.cu", "gemv_w4a16.cu", "engine.cu", "compat.cu", "sme_loader.cu", "radix_cache.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-extended-lambda",
    "-Xcompiler", "-fPIC", "-ccbin", "/usr/bin/g++",
    "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
]


def _compile(src: str) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    srcp = os.path.join(CSRC, src)
    deps = [srcp, os.path.join(CSRC, "common.cuh"), os.path.join(CSRC, "internal.h"), os.path.join(CSRC, "ptx.cuh"), os.path.join(CSRC, "tcgen05.cuh"), os.path.join(ROOT, "include", "specdec.h")]
    if os.path.exists(obj) and all(os.path.getmtime(obj) >= os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *FLAGS, "-c", srcp, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(clean: bool = False, verbose: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(_compile, SOURCES))
    if not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
               "-ccbin", "/usr/bin/g++", "-Xlinker", "-soname=libspecdec_sm100.so", "-o", OUT, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args()
    try:
        build(clean=a.clean, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
