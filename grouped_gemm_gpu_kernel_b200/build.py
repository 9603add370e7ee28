"""Build libgrouped_gemm_b200.so in place (sm_100a only).

    python -m grouped_gemm_gpu_kernel_b200.build [--verbose]

Compiles every CUDA / C++ source under csrc/ with nvcc for ``arch=compute_100a,code=sm_100a``
and links one shared library next to this file. The static CUDA runtime is linked in, so the
library needs only the driver at run time; it is loaded with ctypes (Python) or linked directly
(C/C++ callers of include/grouped_gemm_b200.h or include/grouped_gemm/grouped_gemm.cuh).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libgrouped_gemm_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)
BUILD_DIR = os.path.join(PKG, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]
SOURCES = ["gg_kernels.cu", "gg_host.cu", "gg_copy.cu", "gg_simt.cu", "gg_ipc.cu", "grouped_gemm_api.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd[:3])} ...")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    return res


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _deps():
    out = []
    for root in (CSRC, INCLUDE):
        for dirpath, _, files in os.walk(root):
            out += [os.path.join(dirpath, f) for f in files if f.endswith((".cu", ".cuh", ".h", ".cpp"))]
    return out


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    deps = _deps()
    if not force and not ptxas_info and _newer(LIB_PATH, deps + [__file__]):
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    cc = nvcc()
    objs = []
    for src in SOURCES:
        obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
        extra = ["-Xptxas", "-v"] if (ptxas_info and src.endswith(".cu")) else []
        lang = ["-x", "cu"] if src.endswith(".cu") else []
        res = _run([cc, *ARCH, *NVCC_FLAGS, *extra, *lang, "-c", os.path.join(CSRC, src), "-o", obj], verbose)
        if ptxas_info:
            sys.stdout.write(res.stderr)
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    _run([cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"], verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
