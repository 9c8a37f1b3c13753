"""Builds libkvasir_b200.so in-tree with nvcc for sm_100a (B200).

    python -m kvasir_b200.build          # incremental
    python -m kvasir_b200.build --force  # rebuild everything

The library lands in kvasir_b200/_lib/ so that it travels with the source tree
(no JIT cache, no site-packages install).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libkvasir_b200.so")
SOURCES = ["kvb_api.cu", "kvb_blas.cpp", "kvb_decoder.cpp", "kvb_checkpoint.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _cuda_home(nvcc: str) -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*")) +
            [os.path.join(ROOT, "include", "kvasir_b200.h"), os.path.abspath(__file__)])


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    deps = _deps()
    common = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "-I", os.path.join(ROOT, "include"), "-I", CSRC]
    objs = []
    for src in SOURCES:
        obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, deps):
            cmd = [nvcc, *ARCH, *common, "-c", os.path.join(CSRC, src), "-o", obj]
            if ptxas_verbose and src.endswith(".cu"):
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        libdir = os.path.join(_cuda_home(nvcc), "lib64")
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcublas", "-lcublasLt",
               "-Xlinker", f"-rpath,{libdir}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas" in sys.argv))
