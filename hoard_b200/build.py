"""Builds hoard_b200/libhoard_moe.so in-tree with nvcc for sm_100a (no JIT cache, no torch
extension machinery): every .cu is compiled for `-gencode arch=compute_100a,code=sm_100a`, the
host C++ with g++, and the objects are linked into one shared library with a static CUDA runtime.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libhoard_moe.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v,-warn-spills"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter"]


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    cpp = sorted(f for f in os.listdir(CSRC) if f.endswith(".cpp"))
    return cu, cpp


def _newer(src_paths, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _run(cmd, log):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + r.stdout)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError(f"build step failed: {' '.join(cmd)}")
    return r.stdout


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles and links libhoard_moe.so if any source is newer than it; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    cu, cpp = _sources()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "hoard_moe.h"))
    objs, jobs = [], []
    cxx = shutil.which("g++") or "g++"
    for f in cu:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + headers, obj):
            jobs.append(([NVCC, *GENCODE, *NVCC_FLAGS, "-I", CSRC, "-c", src, "-o", obj], obj + ".log"))
    for f in cpp:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + headers, obj):
            jobs.append(([cxx, *CXX_FLAGS, "-I", os.path.join(CUDA_HOME, "include"), "-I", CSRC, "-c", src, "-o", obj],
                         obj + ".log"))
    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        outs = list(ex.map(lambda j: _run(*j), jobs))
    if verbose:
        for o in outs:
            print(o)
    if force or jobs or _newer(objs, LIB):
        tmp = LIB + ".tmp"
        _run([NVCC, *GENCODE, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread", "-ldl", "-lrt"],
             os.path.join(BUILD, "link.log"))
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
