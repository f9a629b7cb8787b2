"""Builds the two native libraries of the package, in place:

* ``libpc2d_sm100.so``  -- the CUDA kernels and the C ABI of
  ``include/paraconv2d.h`` (nvcc, sm_100a only, links cudart only);
* ``libptparaconv2d.so`` -- the ``torch.ops.ptparaconv2d`` registration
  (g++ against the installed torch, links libpc2d_sm100.so).

Both are rebuilt only when a source or header is newer than the library.
Usage: ``python paraconv2d_b200/build.py [--force] [--verbose]`` (run as a file: importing
the package loads the libraries this builds).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc") if os.path.exists(os.path.join(CUDA_HOME, "bin", "nvcc")) else "nvcc"

KERNEL_LIB = os.path.join(PKG, "libpc2d_sm100.so")
OP_LIB = os.path.join(PKG, "libptparaconv2d.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I" + INCLUDE, "-I" + CSRC]


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    return res


def kernel_sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def build_kernel_lib(force=False, verbose=False, ptxas_verbose=False):
    srcs = kernel_sources()
    if not force and os.path.exists(KERNEL_LIB) and os.path.getmtime(KERNEL_LIB) >= _newest(srcs + headers() + [__file__]):
        return KERNEL_LIB
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        _run([NVCC, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-c", src, "-o", obj], verbose or ptxas_verbose)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = KERNEL_LIB + f".tmp{os.getpid()}"
    _run([NVCC, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcudart"], verbose)
    os.replace(tmp, KERNEL_LIB)
    return KERNEL_LIB


def build_op_lib(force=False, verbose=False):
    src = os.path.join(CSRC, "pc2d_op.cpp")
    if (not force and os.path.exists(OP_LIB)
            and os.path.getmtime(OP_LIB) >= _newest([src, os.path.join(INCLUDE, "paraconv2d.h"), KERNEL_LIB, __file__])):
        return OP_LIB
    import sysconfig

    import torch

    tdir = os.path.dirname(torch.__file__)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = shutil.which("g++") or "c++"
    tmp = OP_LIB + f".tmp{os.getpid()}"
    _run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          "-isystem", os.path.join(tdir, "include"),
          "-isystem", os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
          "-isystem", sysconfig.get_path("include"), "-I" + os.path.join(CUDA_HOME, "include"), "-I" + INCLUDE,
          src, "-o", tmp,
          "-L" + PKG, "-l:libpc2d_sm100.so", "-Wl,-rpath,$ORIGIN",
          "-L" + os.path.join(tdir, "lib"), "-Wl,-rpath," + os.path.join(tdir, "lib"),
          "-ltorch", "-ltorch_cpu", "-lc10", "-lc10_cuda", "-ltorch_cuda",
          "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart"], verbose)
    os.replace(tmp, OP_LIB)
    return OP_LIB


def build_all(force=False, verbose=False, ptxas_verbose=False):
    build_kernel_lib(force, verbose, ptxas_verbose)
    build_op_lib(force, verbose)
    return KERNEL_LIB, OP_LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args(argv)
    build_all(a.force, a.verbose, a.ptxas_verbose)
    print(KERNEL_LIB)
    print(OP_LIB)


if __name__ == "__main__":
    sys.exit(main())
