"""Loader for the C-ABI library ``libgwb200.so``.

Mirrors the reference's native-kernel loader
(``src/gen_worker/models/native_kernels.py:86-143``): the library path comes
from ``GEN_WORKER_B200_LIB`` or the in-tree build, loading is probed with the
``probe_add_one`` numerics check on the GPU, and ``build_info`` identifies the
build. Unlike the reference there is no silent fallback: the quantized-linear
ops raise :class:`NativeKernelError` when the library is missing or the GPU
is not sm_100.
"""

from __future__ import annotations

import ctypes
import functools
import os
from pathlib import Path
from typing import Optional

LIB_ENV = "GEN_WORKER_B200_LIB"
_DEFAULT = Path(__file__).resolve().parent / "_lib" / "libgwb200.so"

c_void_p = ctypes.c_void_p
c_i64 = ctypes.c_int64
c_int = ctypes.c_int

# (name, argtypes); every entry point returns int status.
_SIGNATURES = {
    "gwb_build_info": [ctypes.c_char_p, ctypes.c_size_t],
    "gwb_probe_add_one": [c_void_p, c_void_p, c_i64, c_void_p],
    "gwb_svdq_w4a4_quant": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_int,
                            c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_svdq_w4a4_quant_mma": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_int,
                                c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_svdq_w4a4_scale_k8": [c_void_p, c_i64, c_i64, c_void_p, c_void_p],
    "gwb_svdq_w4a4_weight_expand": [c_void_p, c_i64, c_i64, c_void_p, c_void_p],
    "gwb_svdq_w4a4_gemm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_i64, c_i64, c_i64, c_int, c_int, c_void_p, c_void_p],
    "gwb_svdq_w4a4_gemm_packed": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_i64, c_i64, c_i64, c_int, c_int, c_void_p,
                                  c_void_p],
    "gwb_svdq_w4a4_gemm_stored": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_i64, c_i64, c_i64, c_int, c_int, c_void_p,
                                  c_void_p],
    "gwb_svdq_w4a4_gemm_packed_stored": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int, c_int,
                                         c_void_p, c_void_p],
    "gwb_svdq_w4a4_linear_stored": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_i64, c_i64, c_i64, c_int, c_int, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_svdq_w4a4_group_partials": [c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p,
                                     c_void_p],
    "gwb_svdq_w4a4_linear": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_i64, c_i64, c_i64, c_int, c_int, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p],
    "gwb_svdq_w4a4_linear_noalloc": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int, c_int,
                                     c_void_p, c_void_p],
    "gwb_w8a8_quant": [c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_void_p],
    "gwb_fp8_quant": [c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_void_p],
    "gwb_nvfp4_quant": [c_void_p, c_void_p, c_i64, c_i64, c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_nvfp4_quant_lowrank": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_int, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_nvfp4_gemm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                       c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int, c_void_p,
                       c_void_p],
    "gwb_nunchaku_qweight_to_e2m1": [c_void_p, c_i64, c_i64, c_void_p],
    "gwb_nunchaku_wscales_to_blocked": [c_void_p, c_i64, c_i64, c_void_p],
    "gwb_nunchaku_vector_unpack": [c_void_p, c_i64, c_int, c_void_p],
    "gwb_nunchaku_lowrank_unpack": [c_void_p, c_i64, c_i64, c_int, c_void_p],
    "gwb_lowrank_dequant": [c_void_p, c_void_p, c_i64, c_i64, c_int, c_int, c_void_p],
    "gwb_awq_qweight_unpack": [c_void_p, c_i64, c_i64, c_void_p],
    "gwb_awq_w4a16_mm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64,
                         c_void_p, c_void_p],
    "gwb_fp8_gemm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64,
                     c_int, c_void_p, c_void_p],
    "gwb_fp8_linear": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int,
                       c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_w8a8_gemm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64,
                      c_int, c_void_p, c_void_p],
    "gwb_w8a8_linear": [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_int,
                        c_void_p, c_void_p, c_void_p, c_void_p],
    "gwb_device_error": [ctypes.POINTER(c_int)],
    "gwb_set_wait_limit": [ctypes.c_longlong],
    "gwb_test_stalled_wait": [c_int, c_void_p],
    "gwb_device_check": [],
    "gwb_status_string": [c_int],
}

EXPORTED = tuple(_SIGNATURES)


class NativeKernelError(RuntimeError):
    """The native library is missing, refused the call or reported an error."""


def library_path() -> Path:
    override = os.environ.get(LIB_ENV, "").strip()
    return Path(override) if override else _DEFAULT


@functools.lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    """Load (never build) the library; raise when it is absent."""
    path = library_path()
    if not path.exists():
        raise NativeKernelError(
            f"native library {path} does not exist; build it with "
            f"`python python-gen-worker_b200/csrc/build.py`")
    try:
        handle = ctypes.CDLL(str(path))
    except OSError as exc:
        raise NativeKernelError(f"native library {path} failed to load: {exc}") from exc
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_char_p if name == "gwb_status_string" else c_int
    return handle


TORCH_LIB = _DEFAULT.parent / "libgwb200_torch.so"


@functools.lru_cache(maxsize=1)
def torch_ops():
    """Load the TORCH_LIBRARY(cozy_kernels) extension (``libgwb200_torch.so``,
    beside the C-ABI library; the file the reference's loader takes from
    ``GEN_WORKER_NATIVE_KERNELS_LIB``) and return ``torch.ops.cozy_kernels``."""
    import torch

    if not TORCH_LIB.exists():
        raise NativeKernelError(f"torch extension {TORCH_LIB} does not exist; build it with "
                                f"`python python-gen-worker_b200/csrc/build.py`")
    lib()   # the C-ABI library it links against, from the same folder
    torch.ops.load_library(str(TORCH_LIB))
    return torch.ops.cozy_kernels


def status_string(code: int) -> str:
    return lib().gwb_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise NativeKernelError(f"{what}: status {code} ({status_string(code)})")


def build_info() -> str:
    buf = ctypes.create_string_buffer(256)
    lib().gwb_build_info(buf, 256)
    return buf.value.decode()


def device_error() -> int:
    """Read and clear the device-side error flag (synchronises)."""
    code = c_int(0)
    check(lib().gwb_device_error(ctypes.byref(code)), "gwb_device_error")
    return int(code.value)


def extension_reason() -> Optional[str]:
    """Why the native path cannot run HERE, or None when it can (load +
    sm_100 check + probe numerics; ``native_kernels.py:120-143``)."""
    try:
        import torch

        handle = lib()
        if not torch.cuda.is_available():
            return "no CUDA device"
        if handle.gwb_device_check() != 0:
            major, minor = torch.cuda.get_device_capability()
            return f"device is sm_{major}{minor}, the library targets sm_100a"
        x = torch.arange(8, device="cuda", dtype=torch.float32)
        y = torch.empty_like(x)
        stream = torch.cuda.current_stream().cuda_stream
        check(handle.gwb_probe_add_one(x.data_ptr(), y.data_ptr(), 8, stream), "probe")
        if not torch.equal(y, x + 1):
            return "probe op numerics failed"
    except NativeKernelError as exc:
        return str(exc)
    return None


def extension_available() -> bool:
    return extension_reason() is None


_READY: dict = {}


def require() -> ctypes.CDLL:
    """The loaded library, or a loud error (no CPU fallback). The probe runs
    once per device per process (lane decisions are cached per process in
    the reference too, ``native_kernels.py:19-20``)."""
    import torch

    dev = torch.cuda.current_device() if torch.cuda.is_available() else -1
    if dev not in _READY:
        _READY[dev] = extension_reason()
    reason = _READY[dev]
    if reason is not None:
        raise NativeKernelError(f"gwb200 native path unavailable: {reason}")
    return lib()
