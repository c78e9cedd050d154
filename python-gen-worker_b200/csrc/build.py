#!/usr/bin/env python3
"""Build libgwb200.so (the C-ABI hot-path library) for sm_100a only.

Counterpart of the reference's ``csrc/build.py`` (which builds a
TORCH_LIBRARY extension for sm_100a + sm_120a). Here the kernels live in a
plain C-ABI library (``include/gwb200.h``, bound by ctypes), and a thin
TORCH_LIBRARY(cozy_kernels) extension, ``libgwb200_torch.so``, puts the
reference loader's ops (``build_info``, ``probe_add_one``) and the
quantized-linear ops on top of it. Architecture
coverage is verified at run time by a probe launch (``gwb_probe_add_one``) and
``gwb_device_check``, not by inspecting the binary.

Usage: python csrc/build.py [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent / "gen_worker_b200"
OUT = PKG / "_lib" / "libgwb200.so"
TORCH_OUT = PKG / "_lib" / "libgwb200_torch.so"
SOURCES = ["capi.cu", "act_quant.cu", "gemm.cu", "codec.cu", "awq.cu", "noalloc.cu", "gwb.h", "ptx.cuh"]
HEADER = HERE.parent.parent / "include" / "gwb200.h"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    '-DGWB_ARCH_STRING="sm_100a"',
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = [HERE / s for s in SOURCES] + [HEADER, Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or stale():
        OUT.parent.mkdir(parents=True, exist_ok=True)
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *NVCC_FLAGS, str(HERE / "capi.cu"), "-o", str(tmp)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True, cwd=str(HERE))
        os.replace(tmp, OUT)
    build_torch_ext(force=force, verbose=verbose)
    return OUT


def torch_ext_stale() -> bool:
    if not TORCH_OUT.exists():
        return True
    t = TORCH_OUT.stat().st_mtime
    deps = [HERE / "torch_ext.cpp", HEADER, Path(__file__), OUT]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """libgwb200_torch.so: the TORCH_LIBRARY(cozy_kernels) face of the C ABI,
    compiled with g++ against this interpreter's torch and linked to
    libgwb200.so beside it (rpath $ORIGIN)."""
    if not force and not torch_ext_stale():
        return TORCH_OUT
    import torch
    from torch.utils import cpp_extension as ce
    cuda_inc = str(Path(nvcc()).resolve().parent.parent / "include")
    abi = int(torch.compiled_with_cxx11_abi())
    tmp = TORCH_OUT.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{cuda_inc}",
           str(HERE / "torch_ext.cpp"), "-o", str(tmp),
           *[f"-L{p}" for p in ce.library_paths()], "-lc10", "-lc10_cuda", "-ltorch_cpu",
           "-ltorch", f"-L{OUT.parent}", "-l:libgwb200.so", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=str(HERE))
    os.replace(tmp, TORCH_OUT)
    return TORCH_OUT


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(f"[build] {p}")
