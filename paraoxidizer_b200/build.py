"""Builds libpox_cuda.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

The shared library is the product: the C ABI of include/pox_cuda.h over the hand-written
kernels in csrc/. It is compiled for sm_100a only.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libpox_cuda.so")
BUILD_DIR = os.path.join(PKG, "_build")

SOURCES = ["pox_api.cu", "gemv.cu", "gemm_tc05.cu", "gemm_tcq.cu", "engine.cu", "comm.cu", "quantize.cu", "noalloc.cu", "persist.cu", "pox_file.cpp"]
HEADERS = ["common.cuh", "gemv.cuh", "api_internal.h", "model.h", "comm.cuh", "tc05.cuh", "attn.cuh", "persist.h"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _nccl_dirs():
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    if spec is None or not spec.submodule_search_locations:
        return None, None
    base = os.path.join(list(spec.submodule_search_locations)[0], "nccl")
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return None, None


ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-ffp-contract=off", "-Xptxas", "-O3"]


def _stale(objs) -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "pox_cuda.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu under csrc/ for sm_100a and link libpox_cuda.so (in-tree)."""
    if not force and not _stale(None):
        return LIB
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    nccl_inc, nccl_lib = _nccl_dirs()
    inc = ["-I", os.path.join(ROOT, "include"), "-I", CSRC]
    if nccl_inc:
        inc += ["-I", nccl_inc, "-DPOX_HAVE_NCCL"]
    objs = []
    procs = []
    for s in SOURCES:
        o = os.path.join(BUILD_DIR, os.path.splitext(s)[0] + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, *inc, "-c", os.path.join(CSRC, s), "-o", o]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(o)
    errs = []
    for s, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            errs.append(f"--- {s}\n{out}")
        elif verbose and out.strip():
            print(out, file=sys.stderr)
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    link = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
    if nccl_lib:
        link += ["-L", nccl_lib, "-lnccl", "-Xlinker", "-rpath", "-Xlinker", nccl_lib]
    subprocess.run(link, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
