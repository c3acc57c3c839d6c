"""Build libnpub200.so (the sm_100a kernels and their C ABI) in-tree with nvcc, and the torch operators over it.

    python -m npu_ai_b200.build            # incremental
    python -m npu_ai_b200.build --force    # full rebuild

The libraries land next to this file so they travel with the source tree; no JIT cache, no site-packages install:
  * ``npu_ai_b200/libnpub200.so``: every ``csrc/*.cu`` (kernels + C ABI), objects in ``npu_ai_b200/_build/``;
  * ``npu_ai_b200/libnpub200_torch.so``: ``csrc/torch_ops.cpp``, the TORCH_LIBRARY(npub200) operators
    (torch.ops.npub200.gemm / .attention), linked against libnpub200.so and torch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libnpub200.so")
TORCH_LIB = os.path.join(HERE, "libnpub200_torch.so")
TORCH_SRC = os.path.join(CSRC, "torch_ops.cpp")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    nv = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nv):
        raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")
    return nv


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if force or _stale(obj, [src] + _headers()):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every kernel for sm_100a and link libnpub200.so; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-Xlinker", "-soname=libnpub200.so", "-lcudart_static",
               "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of libnpub200.so failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_torch_ops(force, verbose)
    return LIB


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/torch_ops.cpp with the host compiler against torch's headers into libnpub200_torch.so."""
    if not (force or _stale(TORCH_LIB, [TORCH_SRC, LIB, os.path.join(INCLUDE, "npu_b200.h")])):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension as ce
    inc = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    cxx = shutil.which("g++") or "c++"
    tmp = TORCH_LIB + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in inc], f"-I{INCLUDE}", TORCH_SRC, "-o", tmp, f"-L{HERE}", "-l:libnpub200.so",
           "-Wl,-rpath,$ORIGIN", *[f"-L{p}" for p in libdirs], *[f"-Wl,-rpath,{p}" for p in libdirs[:1]],
           "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build of libnpub200_torch.so failed:\n{r.stdout}\n{r.stderr[-4000:]}")
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
