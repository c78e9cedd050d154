#!/usr/bin/env python3
"""Build libgwb200.so (the C-ABI hot-path library) for sm_100a only.

Counterpart of the reference's ``csrc/build.py`` (which builds a
TORCH_LIBRARY extension for sm_100a + sm_120a). Here the library exposes a
plain C ABI (``include/gwb200.h``); Python binds it with ctypes. Architecture
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
    if not force and not stale():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, str(HERE / "capi.cu"), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=str(HERE))
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(f"[build] {p}")
