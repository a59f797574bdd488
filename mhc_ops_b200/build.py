"""Build the in-tree libraries.

    python -m mhc_ops_b200.build        (or mhc_ops_b200.build.build())

* mhc_ops_b200/lib/libmhc_ops.so -- the kernels and the C ABI, nvcc for sm_100a;
* mhc_ops_b200/lib/libmhc_torch.so -- the TORCH_LIBRARY(mhc, ...) operators
  over that C ABI (csrc/torch_ops.cpp), g++ against the installed torch;
* mhc_ops_b200/lib/libmhc_ops_dbg.so (``--debug-bounds``) -- the same
  sources with -DMHC_DEBUG_BOUNDS: every checked global access must fall in
  the buffers of its call, or it is skipped and recorded (mhc_debug_bounds).
  Load it by setting MHC_OPS_LIBRARY to its path before importing the package.

A build is skipped when its .so is newer than every source it depends on,
unless force=True.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libmhc_ops.so")
DBG_LIB = os.path.join(LIBDIR, "libmhc_ops_dbg.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-O3",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


TORCH_LIB = os.path.join(LIBDIR, "libmhc_torch.so")
TORCH_SRC = os.path.join(CSRC, "torch_ops.cpp")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date(lib: str = LIB, sources: list[str] | None = None) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(s) <= t for s in (sources if sources is not None else _sources()))


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/torch_ops.cpp into lib/libmhc_torch.so (links libmhc_ops.so
    next to it and the installed torch); returns the library path."""
    deps = [TORCH_SRC, LIB] + glob.glob(os.path.join(ROOT, "include", "*.h"))
    if not force and up_to_date(TORCH_LIB, deps):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension as ce
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + ["-I", os.path.join(ROOT, "include")]
    libdirs = ce.library_paths(device_type="cuda")
    torch_lib = libdirs[0]
    tmp = TORCH_LIB + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *inc, TORCH_SRC,
           "-o", tmp, "-L", LIBDIR, "-lmhc_ops", *[f"-L{p}" for p in libdirs],
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building the torch operators failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          debug_bounds: bool = False) -> str:
    """Compile csrc/mhc_ops.cu into lib/libmhc_ops.so (lib/libmhc_ops_dbg.so
    with debug_bounds); returns the library path."""
    lib = DBG_LIB if debug_bounds else LIB
    if not force and up_to_date(lib):
        return lib
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = lib + ".tmp"
    flags = (["-DMHC_DEBUG_BOUNDS"] if debug_bounds else []) + list(extra_flags or [])
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *flags,
           "-I", os.path.join(ROOT, "include"), os.path.join(CSRC, "mhc_ops.cu"), "-o", tmp, "-lcuda"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    force = "--force" in sys.argv
    if "--debug-bounds" in sys.argv:
        print(build(force=force, verbose=True, debug_bounds=True))
    else:
        print(build(force=force, verbose=True))
        print(build_torch_ops(force=force, verbose=True))
