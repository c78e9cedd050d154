"""Torch-facing ops over the C ABI (``torch.ops.gwb200.*``).

Counterparts of the reference's custom ops
``cozy_gen_worker::svdq_quant`` / ``svdq_gemm_w4a4_lora`` /
``svdq_epilogue_lora`` (``src/gen_worker/models/svdq_fused.py:293-391``):
outputs are allocated with ``torch.empty`` on the input device, inputs are
never copied (they must already be contiguous CUDA tensors of the stated
dtype), work is enqueued on the current stream, and every op has a fake
(meta) implementation so ``torch.compile`` can trace through it. There is no
CPU implementation: a CPU tensor raises.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import native

GROUP = 64


class SvdqB200Error(RuntimeError):
    """Typed failure of a gwb200 op (``SvdqFusedError`` counterpart,
    ``svdq_fused.py:34``)."""


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need(t: Optional[torch.Tensor], name: str, dtype: torch.dtype, ndim: int) -> None:
    if t is None:
        return
    if not t.is_cuda:
        raise SvdqB200Error(f"{name} must be a CUDA tensor (no CPU path), got {t.device}")
    if t.dtype != dtype:
        raise SvdqB200Error(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != ndim:
        raise SvdqB200Error(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise SvdqB200Error(f"{name} must be contiguous")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def rank_pad_of(rank: int) -> int:
    return 0 if rank <= 0 else ((rank + 15) // 16) * 16


# ---------------------------------------------------------------- W4A4
@torch.library.custom_op("gwb200::svdq_w4a4_quant", mutates_args=())
def svdq_w4a4_quant(x2: torch.Tensor, smooth: Optional[torch.Tensor],
                    proj_down_t: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """x2 bf16 [M, K] -> packed interchange form (codes u8 [M, K/2],
    ascale f16 [M, K/64]) and la bf16 [M, rank_pad] = x2 · L1 (raw x)."""
    _need(x2, "x2", torch.bfloat16, 2)
    _need(smooth, "smooth", torch.bfloat16, 1)
    _need(proj_down_t, "proj_down_t", torch.bfloat16, 2)
    m, k = x2.shape
    rp = 0 if proj_down_t is None else int(proj_down_t.shape[0])
    codes = torch.empty(m, k // 2, dtype=torch.uint8, device=x2.device)
    ascale = torch.empty(m, k // GROUP, dtype=torch.float16, device=x2.device)
    la = torch.empty(m, rp, dtype=torch.bfloat16, device=x2.device)
    lib = native.require()
    native.check(lib.gwb_svdq_w4a4_quant(x2.data_ptr(), _ptr(smooth), _ptr(proj_down_t), m, k, rp,
                                         codes.data_ptr(), ascale.data_ptr(),
                                         la.data_ptr() if rp else None, _stream()),
                 "svdq_w4a4_quant")
    return codes, ascale, la


@svdq_w4a4_quant.register_fake
def _(x2, smooth, proj_down_t):
    m, k = x2.shape
    rp = 0 if proj_down_t is None else int(proj_down_t.shape[0])
    return (x2.new_empty(m, k // 2, dtype=torch.uint8),
            x2.new_empty(m, k // GROUP, dtype=torch.float16),
            x2.new_empty(m, rp, dtype=torch.bfloat16))


@torch.library.custom_op("gwb200::svdq_w4a4_quant_mma", mutates_args=())
def svdq_w4a4_quant_mma(x2: torch.Tensor, smooth: Optional[torch.Tensor],
                        proj_down_t: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The same quantiser (identical codes and scales) writing the GEMM
    operand form: a_q8 u8 [M, K] (e4m3 bytes of q * 2^-9, within-8 operand
    order), a_scale_k8 f16 [K/64, M, 8], la bf16 [M, rank_pad]."""
    _need(x2, "x2", torch.bfloat16, 2)
    _need(smooth, "smooth", torch.bfloat16, 1)
    _need(proj_down_t, "proj_down_t", torch.bfloat16, 2)
    m, k = x2.shape
    rp = 0 if proj_down_t is None else int(proj_down_t.shape[0])
    codes = torch.empty(m, k, dtype=torch.uint8, device=x2.device)
    sk8 = torch.empty(k // GROUP, m, 8, dtype=torch.float16, device=x2.device)
    la = torch.empty(m, rp, dtype=torch.bfloat16, device=x2.device)
    lib = native.require()
    native.check(lib.gwb_svdq_w4a4_quant_mma(x2.data_ptr(), _ptr(smooth), _ptr(proj_down_t), m, k,
                                             rp, codes.data_ptr(), sk8.data_ptr(),
                                             la.data_ptr() if rp else None, _stream()),
                 "svdq_w4a4_quant_mma")
    return codes, sk8, la


@svdq_w4a4_quant_mma.register_fake
def _(x2, smooth, proj_down_t):
    m, k = x2.shape
    rp = 0 if proj_down_t is None else int(proj_down_t.shape[0])
    return (x2.new_empty(m, k, dtype=torch.uint8),
            x2.new_empty(k // GROUP, m, 8, dtype=torch.float16),
            x2.new_empty(m, rp, dtype=torch.bfloat16))


@torch.library.custom_op("gwb200::svdq_w4a4_scale_k8", mutates_args=())
def svdq_w4a4_scale_k8(scale: torch.Tensor) -> torch.Tensor:
    """Group scales f16 [R, K/64] -> GEMM scale-operand rows f16 [K/64, R, 8]
    (weights at load time, or activation scales from ``svdq_w4a4_quant``)."""
    _need(scale, "scale", torch.float16, 2)
    r, g = scale.shape
    out = torch.empty(g, r, 8, dtype=torch.float16, device=scale.device)
    lib = native.require()
    native.check(lib.gwb_svdq_w4a4_scale_k8(scale.data_ptr(), r, g * GROUP, out.data_ptr(),
                                            _stream()), "svdq_w4a4_scale_k8")
    return out


@svdq_w4a4_scale_k8.register_fake
def _(scale):
    return scale.new_empty(scale.shape[1], scale.shape[0], 8, dtype=torch.float16)


def expand_w4a4_weight(w_codes: torch.Tensor) -> torch.Tensor:
    """Load-time repack of the packed INT4 weight u8 [N, K/2] into the GEMM
    operand form u8 [N, K] (e4m3 bytes of q * 2^-9, within-8 operand order),
    on the weight's CUDA device."""
    _need(w_codes, "w_codes", torch.uint8, 2)
    n, k = w_codes.shape[0], w_codes.shape[1] * 2
    out = torch.empty(n, k, dtype=torch.uint8, device=w_codes.device)
    lib = native.require()
    native.check(lib.gwb_svdq_w4a4_weight_expand(w_codes.data_ptr(), n, k, out.data_ptr(),
                                                 _stream()), "svdq_w4a4_weight_expand")
    return out


def _w4a4_gemm(fn: str, a: torch.Tensor, k: int, a_scale_k8, w_q8, w_scale_k8, la, proj_up,
               bias, gelu) -> torch.Tensor:
    _need(a_scale_k8, "a_scale_k8", torch.float16, 3)
    _need(w_q8, "w_q8", torch.uint8, 2)
    _need(w_scale_k8, "w_scale_k8", torch.float16, 3)
    _need(bias, "bias", torch.bfloat16, 1)
    m = a.shape[0]
    n = w_q8.shape[0]
    if int(w_q8.shape[1]) != k:
        raise SvdqB200Error(f"w_q8 K {w_q8.shape[1]} != activation K {k}")
    rp = 0
    if la is not None and proj_up is not None and la.shape[1] > 0:
        _need(la, "la", torch.bfloat16, 2)
        _need(proj_up, "proj_up", torch.bfloat16, 2)
        rp = int(la.shape[1])
        if int(proj_up.shape[1]) != rp:
            raise SvdqB200Error(f"la rank {rp} != proj_up rank {proj_up.shape[1]}")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    lib = native.require()
    native.check(getattr(lib, fn)(a.data_ptr(), a_scale_k8.data_ptr(), w_q8.data_ptr(),
                                  w_scale_k8.data_ptr(), _ptr(la) if rp else None,
                                  _ptr(proj_up) if rp else None, _ptr(bias), m, n, k, rp,
                                  int(bool(gelu)), out.data_ptr(), _stream()), fn)
    return out


@torch.library.custom_op("gwb200::svdq_w4a4_gemm", mutates_args=())
def svdq_w4a4_gemm(a_q8: torch.Tensor, a_scale_k8: torch.Tensor, w_q8: torch.Tensor,
                   w_scale_k8: torch.Tensor, la: Optional[torch.Tensor],
                   proj_up: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                   gelu: bool) -> torch.Tensor:
    """INT4 group-64 GEMM on operand-form activations (``svdq_w4a4_quant_mma``)
    + promotion + low-rank up-projection + bias (+ GELU) -> bf16 [M, N]."""
    _need(a_q8, "a_q8", torch.uint8, 2)
    return _w4a4_gemm("gwb_svdq_w4a4_gemm", a_q8, int(a_q8.shape[1]), a_scale_k8, w_q8,
                      w_scale_k8, la, proj_up, bias, gelu)


@svdq_w4a4_gemm.register_fake
def _(a_q8, a_scale_k8, w_q8, w_scale_k8, la, proj_up, bias, gelu):
    return a_q8.new_empty(a_q8.shape[0], w_q8.shape[0], dtype=torch.bfloat16)


@torch.library.custom_op("gwb200::svdq_w4a4_gemm_packed", mutates_args=())
def svdq_w4a4_gemm_packed(codes: torch.Tensor, a_scale_k8: torch.Tensor, w_q8: torch.Tensor,
                          w_scale_k8: torch.Tensor, la: Optional[torch.Tensor],
                          proj_up: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                          gelu: bool) -> torch.Tensor:
    """The same GEMM on packed activation codes u8 [M, K/2] (unpacked to the
    operand layout in shared memory)."""
    _need(codes, "codes", torch.uint8, 2)
    return _w4a4_gemm("gwb_svdq_w4a4_gemm_packed", codes, int(codes.shape[1]) * 2, a_scale_k8,
                      w_q8, w_scale_k8, la, proj_up, bias, gelu)


@svdq_w4a4_gemm_packed.register_fake
def _(codes, a_scale_k8, w_q8, w_scale_k8, la, proj_up, bias, gelu):
    return codes.new_empty(codes.shape[0], w_q8.shape[0], dtype=torch.bfloat16)


def _w4a4_gemm_stored(fn: str, a: torch.Tensor, k: int, a_scale_k8, weight, weight_scale, la,
                      proj_up, bias, gelu) -> torch.Tensor:
    _need(a_scale_k8, "a_scale_k8", torch.float16, 3)
    _need(weight, "weight", torch.uint8, 2)
    _need(weight_scale, "weight_scale", torch.float16, 2)
    _need(bias, "bias", torch.bfloat16, 1)
    m = a.shape[0]
    n = weight.shape[0]
    if int(weight.shape[1]) * 2 != k or tuple(weight_scale.shape) != (n, k // GROUP):
        raise SvdqB200Error(f"stored weight {tuple(weight.shape)} / weight_scale "
                            f"{tuple(weight_scale.shape)} do not match activation K {k}")
    rp = 0
    if la is not None and proj_up is not None and la.shape[1] > 0:
        _need(la, "la", torch.bfloat16, 2)
        _need(proj_up, "proj_up", torch.bfloat16, 2)
        rp = int(la.shape[1])
        if int(proj_up.shape[1]) != rp:
            raise SvdqB200Error(f"la rank {rp} != proj_up rank {proj_up.shape[1]}")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    lib = native.require()
    native.check(getattr(lib, fn)(a.data_ptr(), a_scale_k8.data_ptr(), weight.data_ptr(),
                                  weight_scale.data_ptr(), _ptr(la) if rp else None,
                                  _ptr(proj_up) if rp else None, _ptr(bias), m, n, k, rp,
                                  int(bool(gelu)), out.data_ptr(), _stream()), fn)
    return out


def stored_weights_supported(in_features: int) -> bool:
    """The stored-weight GEMM reads 8 groups of scales per 16-byte row:
    in_features must be a multiple of 512."""
    return in_features % (8 * GROUP) == 0


@torch.library.custom_op("gwb200::svdq_w4a4_gemm_stored", mutates_args=())
def svdq_w4a4_gemm_stored(a_q8: torch.Tensor, a_scale_k8: torch.Tensor, weight: torch.Tensor,
                          weight_scale: torch.Tensor, la: Optional[torch.Tensor],
                          proj_up: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                          gelu: bool) -> torch.Tensor:
    """INT4 group-64 GEMM on the weight AS STORED (``weight`` u8 [N, K/2],
    ``weight_scale`` f16 [N, K/64]; expanded in shared memory) and
    operand-form activations (``svdq_w4a4_quant_mma``) + promotion +
    low-rank up-projection + bias (+ GELU) -> bf16 [M, N]
    (``svdq_gemm_w4a4_lora``, ``svdq_fused.py:379-383``)."""
    _need(a_q8, "a_q8", torch.uint8, 2)
    return _w4a4_gemm_stored("gwb_svdq_w4a4_gemm_stored", a_q8, int(a_q8.shape[1]), a_scale_k8,
                             weight, weight_scale, la, proj_up, bias, gelu)


@svdq_w4a4_gemm_stored.register_fake
def _(a_q8, a_scale_k8, weight, weight_scale, la, proj_up, bias, gelu):
    return a_q8.new_empty(a_q8.shape[0], weight.shape[0], dtype=torch.bfloat16)


@torch.library.custom_op("gwb200::svdq_w4a4_gemm_packed_stored", mutates_args=())
def svdq_w4a4_gemm_packed_stored(codes: torch.Tensor, a_scale_k8: torch.Tensor,
                                 weight: torch.Tensor, weight_scale: torch.Tensor,
                                 la: Optional[torch.Tensor], proj_up: Optional[torch.Tensor],
                                 bias: Optional[torch.Tensor], gelu: bool) -> torch.Tensor:
    """The stored-weight GEMM on packed activation codes u8 [M, K/2] (both
    operands expanded in shared memory)."""
    _need(codes, "codes", torch.uint8, 2)
    return _w4a4_gemm_stored("gwb_svdq_w4a4_gemm_packed_stored", codes, int(codes.shape[1]) * 2,
                             a_scale_k8, weight, weight_scale, la, proj_up, bias, gelu)


@svdq_w4a4_gemm_packed_stored.register_fake
def _(codes, a_scale_k8, weight, weight_scale, la, proj_up, bias, gelu):
    return codes.new_empty(codes.shape[0], weight.shape[0], dtype=torch.bfloat16)


@torch.library.custom_op("gwb200::svdq_w4a4_group_partials", mutates_args=())
def svdq_w4a4_group_partials(codes: torch.Tensor, w_q8: torch.Tensor) -> torch.Tensor:
    """Debug: every 64-group integer partial sum of the tcgen05 GEMM,
    s32 [K/64, M, N] (packed activation codes, expanded weight)."""
    _need(codes, "codes", torch.uint8, 2)
    _need(w_q8, "w_q8", torch.uint8, 2)
    m, k = codes.shape[0], codes.shape[1] * 2
    n = w_q8.shape[0]
    out = torch.empty(k // GROUP, m, n, dtype=torch.int32, device=codes.device)
    lib = native.require()
    native.check(lib.gwb_svdq_w4a4_group_partials(codes.data_ptr(), w_q8.data_ptr(), m, n, k,
                                                  out.data_ptr(), _stream()),
                 "svdq_w4a4_group_partials")
    return out


@svdq_w4a4_group_partials.register_fake
def _(codes, w_q8):
    return codes.new_empty(codes.shape[1] * 2 // GROUP, codes.shape[0], w_q8.shape[0],
                           dtype=torch.int32)


# ---------------------------------------------------------------- W8A8
@torch.library.custom_op("gwb200::w8a8_quant", mutates_args=())
def w8a8_quant(x2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token INT8: x2 bf16 [M, K] -> (q s8 [M, K], scale f32 [M])."""
    _need(x2, "x2", torch.bfloat16, 2)
    m, k = x2.shape
    q = torch.empty(m, k, dtype=torch.int8, device=x2.device)
    s = torch.empty(m, dtype=torch.float32, device=x2.device)
    lib = native.require()
    native.check(lib.gwb_w8a8_quant(x2.data_ptr(), m, k, q.data_ptr(), s.data_ptr(), _stream()),
                 "w8a8_quant")
    return q, s


@w8a8_quant.register_fake
def _(x2):
    return x2.new_empty(x2.shape, dtype=torch.int8), x2.new_empty(x2.shape[0], dtype=torch.float32)


@torch.library.custom_op("gwb200::w8a8_gemm", mutates_args=())
def w8a8_gemm(q: torch.Tensor, scale: torch.Tensor, w_q: torch.Tensor, w_scale: torch.Tensor,
              bias: Optional[torch.Tensor], gelu: bool) -> torch.Tensor:
    _need(q, "q", torch.int8, 2)
    _need(scale, "scale", torch.float32, 1)
    _need(w_q, "w_q", torch.int8, 2)
    _need(w_scale, "w_scale", torch.float32, 1)
    _need(bias, "bias", torch.bfloat16, 1)
    m, k = q.shape
    n = w_q.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=q.device)
    lib = native.require()
    native.check(lib.gwb_w8a8_gemm(q.data_ptr(), scale.data_ptr(), w_q.data_ptr(),
                                   w_scale.data_ptr(), _ptr(bias), m, n, k, int(bool(gelu)),
                                   out.data_ptr(), _stream()), "w8a8_gemm")
    return out


@w8a8_gemm.register_fake
def _(q, scale, w_q, w_scale, bias, gelu):
    return q.new_empty(q.shape[0], w_q.shape[0], dtype=torch.bfloat16)


# ---------------------------------------------------------------- FP8 rowwise
def _as_fp8_bytes(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    _need(t, name, torch.uint8, 2)
    return t


@torch.library.custom_op("gwb200::fp8_quant", mutates_args=())
def fp8_quant(x2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token FP8 e4m3 (the reference's dynamic rowwise ``_quant_src``,
    ``w8a8.py:261-273``): x2 bf16 [M, K] -> (q e4m3 bytes u8 [M, K],
    scale f32 [M])."""
    _need(x2, "x2", torch.bfloat16, 2)
    m, k = x2.shape
    q = torch.empty(m, k, dtype=torch.uint8, device=x2.device)
    s = torch.empty(m, dtype=torch.float32, device=x2.device)
    lib = native.require()
    native.check(lib.gwb_fp8_quant(x2.data_ptr(), m, k, q.data_ptr(), s.data_ptr(), _stream()),
                 "fp8_quant")
    return q, s


@fp8_quant.register_fake
def _(x2):
    return x2.new_empty(x2.shape, dtype=torch.uint8), x2.new_empty(x2.shape[0], dtype=torch.float32)


@torch.library.custom_op("gwb200::fp8_gemm", mutates_args=())
def fp8_gemm(q: torch.Tensor, scale: torch.Tensor, w_q: torch.Tensor, w_scale: torch.Tensor,
             bias: Optional[torch.Tensor], gelu: bool) -> torch.Tensor:
    """``_scaled_mm`` rowwise on e4m3 operands (``Fp8ScaledLinear.forward``,
    ``w8a8.py:374-378``): q / w_q e4m3 bytes (u8 or float8_e4m3fn) [M, K] /
    [N, K], scale f32 [M], w_scale f32 [N] -> bf16 [M, N] (+ GELU)."""
    q = _as_fp8_bytes(q, "q")
    w_q = _as_fp8_bytes(w_q, "w_q")
    _need(scale, "scale", torch.float32, 1)
    _need(w_scale, "w_scale", torch.float32, 1)
    _need(bias, "bias", torch.bfloat16, 1)
    m, k = q.shape
    n = w_q.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=q.device)
    lib = native.require()
    native.check(lib.gwb_fp8_gemm(q.data_ptr(), scale.data_ptr(), w_q.data_ptr(),
                                  w_scale.data_ptr(), _ptr(bias), m, n, k, int(bool(gelu)),
                                  out.data_ptr(), _stream()), "fp8_gemm")
    return out


@fp8_gemm.register_fake
def _(q, scale, w_q, w_scale, bias, gelu):
    return q.new_empty(q.shape[0], w_q.shape[0], dtype=torch.bfloat16)


# ---------------------------------------------------------------- NVFP4
def nvfp4_blocked_numel(rows: int, k: int) -> int:
    """Bytes of the cuBLAS blocked e4m3 scale layout for [rows, k/16] scales
    (``blocked_scale_numel``, ``nvfp4_quant.py:87-89``)."""
    return ((rows + 127) // 128) * 128 * ((k // 16 + 3) // 4) * 4


@torch.library.custom_op("gwb200::nvfp4_quant", mutates_args=())
def nvfp4_quant(x2: torch.Tensor, smooth: Optional[torch.Tensor]
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The reference's NVFP4 activation chain (smoothing divide, per-tensor
    ``s2``, ``quantize_activation``): x2 bf16 [M, K] -> (codes u8 [M, K/2],
    blocked e4m3 scale bytes u8, work f32 [4 + K] with ``work[1] = s2``)."""
    _need(x2, "x2", torch.bfloat16, 2)
    _need(smooth, "smooth", torch.bfloat16, 1)
    m, k = x2.shape
    codes = torch.empty(m, k // 2, dtype=torch.uint8, device=x2.device)
    sblk = torch.empty(nvfp4_blocked_numel(m, k), dtype=torch.uint8, device=x2.device)
    work = torch.empty(4 + k, dtype=torch.float32, device=x2.device)
    lib = native.require()
    native.check(lib.gwb_nvfp4_quant(x2.data_ptr(), _ptr(smooth), m, k, codes.data_ptr(),
                                     sblk.data_ptr(), work.data_ptr(), _stream()), "nvfp4_quant")
    return codes, sblk, work


@nvfp4_quant.register_fake
def _(x2, smooth):
    m, k = x2.shape
    return (x2.new_empty(m, k // 2, dtype=torch.uint8),
            x2.new_empty(nvfp4_blocked_numel(m, k), dtype=torch.uint8),
            x2.new_empty(4 + k, dtype=torch.float32))


@torch.library.custom_op("gwb200::nvfp4_quant_lowrank", mutates_args=())
def nvfp4_quant_lowrank(x2: torch.Tensor, smooth: Optional[torch.Tensor], down_t: torch.Tensor
                        ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """:func:`nvfp4_quant` plus the low-rank activations from the same pass
    over x: down_t bf16 [rank_pad, K] -> (codes, blocked scales, work, la3
    bf16 [M, 3 * rank_pad]). la3 = [u_hi | u_lo | u_hi] with u = bf16(x2 ·
    proj_down) / s2 (raw x, as the reference) split into two bf16 parts
    (:func:`nvfp4_la_from_la3` recovers bf16(x2 · proj_down))."""
    _need(x2, "x2", torch.bfloat16, 2)
    _need(smooth, "smooth", torch.bfloat16, 1)
    _need(down_t, "down_t", torch.bfloat16, 2)
    m, k = x2.shape
    rp = int(down_t.shape[0])
    if int(down_t.shape[1]) != k:
        raise SvdqB200Error(f"down_t K {down_t.shape[1]} != activation K {k}")
    codes = torch.empty(m, k // 2, dtype=torch.uint8, device=x2.device)
    sblk = torch.empty(nvfp4_blocked_numel(m, k), dtype=torch.uint8, device=x2.device)
    work = torch.empty(4 + k, dtype=torch.float32, device=x2.device)
    la = torch.empty(m, 3 * rp, dtype=torch.bfloat16, device=x2.device)
    native.check(native.require().gwb_nvfp4_quant_lowrank(
        x2.data_ptr(), _ptr(smooth), down_t.data_ptr(), m, k, rp, codes.data_ptr(),
        sblk.data_ptr(), work.data_ptr(), la.data_ptr(), _stream()), "nvfp4_quant_lowrank")
    return codes, sblk, work, la


@nvfp4_quant_lowrank.register_fake
def _(x2, smooth, down_t):
    m, k = x2.shape
    return (x2.new_empty(m, k // 2, dtype=torch.uint8),
            x2.new_empty(nvfp4_blocked_numel(m, k), dtype=torch.uint8),
            x2.new_empty(4 + k, dtype=torch.float32),
            x2.new_empty(m, 3 * down_t.shape[0], dtype=torch.bfloat16))


def nvfp4_la_from_la3(la3: torch.Tensor, work: torch.Tensor) -> torch.Tensor:
    """(u_hi + u_lo) · s2: the low-rank activation bf16(x · proj_down) the
    three-part form was built from (to ~2^-17), f32 [M, rank_pad]."""
    rp = la3.shape[1] // 3
    return (la3[:, :rp].float() + la3[:, rp:2 * rp].float()) * work[1]


@torch.library.custom_op("gwb200::nvfp4_gemm", mutates_args=())
def nvfp4_gemm(codes: torch.Tensor, sblk: torch.Tensor, work: torch.Tensor, w_codes: torch.Tensor,
               w_sblk: torch.Tensor, w_scale_2: torch.Tensor, la: Optional[torch.Tensor],
               proj_up: Optional[torch.Tensor], bias: Optional[torch.Tensor]) -> torch.Tensor:
    """Block-scaled NVFP4 GEMM + ``s2 · weight_scale_2`` + low-rank + bias
    -> bf16 [M, N] (``_gemm_w4a4`` and the rest of the NVFP4
    ``SvdqLinear.forward``, ``svdq_native.py:148-155``). The low-rank operands
    are three-part: la3 [M, 3 * rank_pad] from :func:`nvfp4_quant_lowrank` and
    up3 [N, 3 * rank_pad] from :func:`nvfp4_lowrank_prepare`; la3 · up3ᵀ is
    the low-rank product divided by ``s2 · weight_scale_2``."""
    _need(codes, "codes", torch.uint8, 2)
    _need(w_codes, "w_codes", torch.uint8, 2)
    _need(work, "work", torch.float32, 1)
    _need(bias, "bias", torch.bfloat16, 1)
    if sblk.dtype == torch.float8_e4m3fn:
        sblk = sblk.view(torch.uint8)
    if w_sblk.dtype == torch.float8_e4m3fn:
        w_sblk = w_sblk.view(torch.uint8)
    m, k = codes.shape[0], codes.shape[1] * 2
    n = w_codes.shape[0]
    if int(w_codes.shape[1]) * 2 != k:
        raise SvdqB200Error(f"w_codes K {w_codes.shape[1] * 2} != activation K {k}")
    if w_sblk.numel() != nvfp4_blocked_numel(n, k) or sblk.numel() != nvfp4_blocked_numel(m, k):
        raise SvdqB200Error("blocked scale buffers do not match the operand shapes")
    ws2 = w_scale_2.float().reshape(-1).contiguous()
    if ws2.numel() not in (1, n):
        raise SvdqB200Error(f"weight_scale_2 has {ws2.numel()} entries (want 1 or {n})")
    rp = 0
    if la is not None and proj_up is not None and la.shape[1] > 0:
        _need(la, "la", torch.bfloat16, 2)
        _need(proj_up, "proj_up", torch.bfloat16, 2)
        if la.shape[1] % 3 or tuple(proj_up.shape) != (n, la.shape[1]):
            raise SvdqB200Error(f"three-part la {tuple(la.shape)} / up {tuple(proj_up.shape)} "
                                f"do not match (want [M, 3r] and [{n}, 3r])")
        rp = int(la.shape[1]) // 3
    out = torch.empty(m, n, dtype=torch.bfloat16, device=codes.device)
    lib = native.require()
    native.check(lib.gwb_nvfp4_gemm(codes.data_ptr(), sblk.data_ptr(), work.data_ptr(),
                                    w_codes.data_ptr(), w_sblk.data_ptr(), ws2.data_ptr(),
                                    int(ws2.numel() == n and n > 1), _ptr(la) if rp else None,
                                    _ptr(proj_up) if rp else None, _ptr(bias), m, n, k, rp,
                                    out.data_ptr(), _stream()), "nvfp4_gemm")
    return out


def nvfp4_lowrank_prepare(proj_down: torch.Tensor, proj_up: torch.Tensor,
                          w_scale_2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Load time: ``proj_down`` bf16 padded to [K, rank_pad], and the
    three-part up-projection up3 bf16 [N, 3 * rank_pad] = [w_hi | w_hi |
    w_lo] with w = proj_up / weight_scale_2[n] (f32) split into two bf16
    parts, so that la3 · up3ᵀ = u_hi w_hi + u_lo w_hi + u_hi w_lo."""
    k, r = proj_down.shape
    n = proj_up.shape[0]
    rp = rank_pad_of(r)
    down = torch.zeros(k, rp, dtype=torch.bfloat16, device=proj_down.device)
    down[:, :r] = proj_down.to(torch.bfloat16)
    w = torch.zeros(n, rp, dtype=torch.float32, device=proj_up.device)
    w[:, :r] = proj_up.float() / w_scale_2.float().reshape(-1, 1)
    hi = w.to(torch.bfloat16)
    lo = (w - hi.float()).to(torch.bfloat16)
    return down, torch.cat([hi, hi, lo], dim=1).contiguous()


@nvfp4_gemm.register_fake
def _(codes, sblk, work, w_codes, w_sblk, w_scale_2, la, proj_up, bias):
    return codes.new_empty(codes.shape[0], w_codes.shape[0], dtype=torch.bfloat16)


# ---------------------------------------------------------------- load-time repacks
def prepare_w4a4_weights(w_scale: Optional[torch.Tensor], proj_down: Optional[torch.Tensor],
                         proj_up: Optional[torch.Tensor],
                         weight: Optional[torch.Tensor] = None,
                         operand_form: bool = True) -> dict:
    """Load-time repack of the module buffers into the kernel operand layouts
    (the reference repacks at load too: ``to_buffers``,
    ``svdq_layout.py:473-483``):
      weight u8 [N, K/2]         -> w_q8 u8 [N, K] (CUDA only; else None)
      weight_scale f16 [N, K/64] -> w_scale_k8 f16 [K/64, N, 8] (CUDA only;
                                    None when w_scale is None or on the CPU)
      proj_down bf16 [K, r]      -> proj_down_t bf16 [rank_pad, K] (zero rows)
      proj_up bf16 [N, r]        -> proj_up_pad bf16 [N, rank_pad] (zero cols)
    With ``operand_form=False`` the weight and its scales stay as stored
    (the stored-weight GEMM reads them directly) and only the low-rank
    factors are repacked."""
    out: dict = {"w_scale_k8": None, "w_q8": None}
    if operand_form and weight is not None and weight.is_cuda:
        out["w_q8"] = expand_w4a4_weight(weight.contiguous())
    if operand_form and w_scale is not None and w_scale.is_cuda:
        out["w_scale_k8"] = svdq_w4a4_scale_k8(w_scale.to(torch.float16).contiguous())
    if proj_down is not None and proj_up is not None and proj_down.shape[1] > 0:
        k, r = proj_down.shape
        n = proj_up.shape[0]
        rp = rank_pad_of(r)
        if rp > 128:
            raise SvdqB200Error(f"low-rank rank {r} > 128 is not supported")
        dt = torch.zeros(rp, k, dtype=torch.bfloat16, device=proj_down.device)
        dt[:r] = proj_down.to(torch.bfloat16).t()
        up = torch.zeros(n, rp, dtype=torch.bfloat16, device=proj_up.device)
        up[:, :r] = proj_up.to(torch.bfloat16)
        out["proj_down_t"] = dt
        out["proj_up_pad"] = up
    else:
        out["proj_down_t"] = None
        out["proj_up_pad"] = None
    return out
