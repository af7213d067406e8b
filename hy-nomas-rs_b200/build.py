"""Build libnomas_kv.so (C ABI + sm_100a kernels) in-tree.

    python hy-nomas-rs_b200/build.py          # incremental
    python hy-nomas-rs_b200/build.py --clean  # from scratch

Objects go to hy-nomas-rs_b200/_build/, the library to
hy-nomas-rs_b200/nomas_kv/libnomas_kv.so (both git-ignored; the .so travels
with the source tree to the GPU host).  nvcc cross-compiles for sm_100a, so
this runs on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "nomas_kv", "libnomas_kv.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

SOURCES = ["kernels_commit.cu", "kernels_gather.cu", "kernels_qvg.cu", "kernels_qvg_fit.cu", "kernels_project.cu",
           "kernels_attn.cu",
           "bank.cpp", "abi.cpp",
           "noalloc.cu"]
HEADERS = ["nkv_kernels.h", "nkv_device.cuh", "nkv_quant.cuh", "nkv_policy.h", "bank.h"]

# -fmad=false / -ffp-contract=off: the reference rounds every multiply and
# add separately; the kernels ask for fused operations explicitly where the
# result is provably identical.
COMMON = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-fmad=false",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math,-Wall,-Wno-unused-function",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    deps = [path] + [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "nomas_kv.h")]
    if _newer(obj, deps):
        cmd = [NVCC, *COMMON, "-c", path, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(clean: bool = False, verbose: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(_compile, SOURCES))
    if _newer(LIB, objs):
        cmd = [NVCC, "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs,
               "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args()
    try:
        build(clean=a.clean, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
