"""gen_worker_b200 — B200-native (sm_100a) SVDQuant W4A4 / W8A8 quantized
linear: the hot path of gen-worker's quantized diffusion-transformer serving,
behind the reference's module surface (``SvdqLinear`` / ``Fp8ScaledLinear``
buffers, ``swap_svdq_linears``-style seam) and a C-ABI library
(``include/gwb200.h``) bound with ctypes.
"""

from .native import (NativeKernelError, build_info, device_error, extension_available,
                     extension_reason, library_path)
from .modules import (LAYOUT_INT4, LAYOUT_NVFP4, Fp8RowwiseLinear, SvdqInt4Linear,
                      SvdqNvfp4Linear, W8A8Int8Linear, build_fp8_rowwise_linear,
                      build_svdq_int4_linear, build_svdq_nvfp4_linear, build_w8a8_int8_linear,
                      fp8_rowwise_from_linear, quantize_fp8_rows, quantize_int4_rows,
                      quantize_int8_rows, svdq_int4_from_linear, swap_linears)
from . import awq, codec, ops

__all__ = [
    "LAYOUT_INT4", "LAYOUT_NVFP4", "NativeKernelError", "Fp8RowwiseLinear", "SvdqInt4Linear",
    "SvdqNvfp4Linear", "W8A8Int8Linear", "build_fp8_rowwise_linear", "build_info",
    "build_svdq_int4_linear", "build_svdq_nvfp4_linear", "build_w8a8_int8_linear",
    "device_error", "fp8_rowwise_from_linear", "quantize_fp8_rows",
    "extension_available", "extension_reason", "library_path", "ops", "awq", "codec",
    "quantize_int4_rows", "quantize_int8_rows", "svdq_int4_from_linear", "swap_linears",
]
