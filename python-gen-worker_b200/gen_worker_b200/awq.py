"""AWQ W4A16 modulation layers (the timestep-embedding consumers ``img_mod`` /
``txt_mod`` of an SVDQuant checkpoint), packed-resident.

Counterpart of the reference's packed lane
(``src/gen_worker/models/svdq_awq_packed.py``): the same module buffers
(``weight`` u8 [N, K/2] unsigned 4-bit codes with even k in the low nibble,
``wscales`` / ``wzeros`` [N, K/64] in the compute dtype, ``bias``), the same
op (``awq_w4a16_mm(x2, weight, wscales, wzeros, bias)``, here
``torch.ops.gwb200.awq_w4a16_mm`` over ``gwb_awq_w4a16_mm``), the same
load-time decode of the on-disk tensors (TinyChat ``qweight`` I32 [N/4, K/2],
``wscales`` / ``wzeros`` [ceil_num_groups, N], the adaLN split interleave and
its ``+1`` bias fold undone, ``build_awq_packed_linear``,
``svdq_awq_packed.py:204-249``) and the same refusals (``AwqPackedError``).
The GEMV is a native sm_100a kernel; the TinyChat unpack is native host code.
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from . import native
from .ops import SvdqB200Error, _need, _ptr, _stream

GROUP_SIZE = 64
_PACK_SIZE = 8
_NUM_PACKS_FACTOR = {32: 4, 64: 2}


class AwqPackedError(RuntimeError):
    """Typed packed-AWQ failure (``AwqPackedError``, ``svdq_awq_packed.py:20``)."""


def awq_packed_supported(out_features: int, in_features: int) -> bool:
    return out_features % 16 == 0 and in_features % 128 == 0


def num_scale_rows(in_features: int, group_size: int) -> int:
    """The exporter's padded scale-row count (``ceil_num_groups``,
    ``svdq_awq.py:18-28``): groups rounded up to packs of 8, packs to a
    multiple of 2 (group 64) or 4 (group 32)."""
    if in_features % group_size:
        raise AwqPackedError(f"in_features {in_features} not divisible by group size {group_size}")
    packs = -(-(in_features // group_size) // _PACK_SIZE)
    factor = _NUM_PACKS_FACTOR.get(group_size, 1)
    return -(-packs // factor) * factor * _PACK_SIZE


# ---------------------------------------------------------------- op
@torch.library.custom_op("gwb200::awq_w4a16_mm", mutates_args=())
def awq_w4a16_mm(x2: torch.Tensor, weight: torch.Tensor, wscales: torch.Tensor,
                 wzeros: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    """x2 bf16 [M, K] · bf16(q · wscales + wzeros)ᵀ + bias -> bf16 [M, N]."""
    _need(x2, "x2", torch.bfloat16, 2)
    _need(weight, "weight", torch.uint8, 2)
    _need(wscales, "wscales", torch.bfloat16, 2)
    _need(wzeros, "wzeros", torch.bfloat16, 2)
    _need(bias, "bias", torch.bfloat16, 1)
    m, k = x2.shape
    n = int(weight.shape[0])
    if int(weight.shape[1]) * 2 != k or tuple(wscales.shape) != (n, k // GROUP_SIZE) \
            or wzeros.shape != wscales.shape:
        raise SvdqB200Error(f"awq operands do not match: x2 {tuple(x2.shape)}, weight "
                            f"{tuple(weight.shape)}, wscales {tuple(wscales.shape)}")
    out = torch.empty(m, n, dtype=torch.bfloat16, device=x2.device)
    native.check(native.require().gwb_awq_w4a16_mm(
        x2.data_ptr(), weight.data_ptr(), wscales.data_ptr(), wzeros.data_ptr(), _ptr(bias),
        m, n, k, out.data_ptr(), _stream()), "awq_w4a16_mm")
    return out


@awq_w4a16_mm.register_fake
def _(x2, weight, wscales, wzeros, bias):
    return x2.new_empty(x2.shape[0], weight.shape[0], dtype=torch.bfloat16)


# ---------------------------------------------------------------- load time
def unpack_qweight(qweight: torch.Tensor, out_features: int, in_features: int) -> torch.Tensor:
    """TinyChat ``qweight`` I32 [N/4, K/2] -> ``weight`` u8 [N, K/2] (native
    host code, ``gwb_awq_qweight_unpack``)."""
    n, k = int(out_features), int(in_features)
    if n % 4 or k % 64:
        raise AwqPackedError(f"AWQ W4A16 [{n}, {k}] needs oc%4==0 and ic%64==0")
    if tuple(qweight.shape) != (n // 4, k // 2):
        raise AwqPackedError(f"AWQ qweight shape {tuple(qweight.shape)} != expected "
                             f"{(n // 4, k // 2)} for [{n}, {k}]")
    src = qweight.detach().to("cpu").contiguous()
    out = torch.empty(n, k // 2, dtype=torch.uint8)
    native.check(native.lib().gwb_awq_qweight_unpack(ctypes.c_void_p(src.data_ptr()), n, k,
                                                    ctypes.c_void_p(out.data_ptr())),
                 "awq_qweight_unpack")
    return out


def scales_and_zeros(wscales: torch.Tensor, wzeros: torch.Tensor, out_features: int,
                     in_features: int) -> tuple[torch.Tensor, torch.Tensor, int]:
    """[rows, N] grids -> ([N, ng], [N, ng], group size), the live rows only;
    the same checks as the reference (``_scales_and_zeros``, ``svdq_awq.py:50-73``)."""
    n, k = int(out_features), int(in_features)
    if wscales.shape[1] != n or wzeros.shape != wscales.shape:
        raise AwqPackedError(f"AWQ scale/zero grids {tuple(wscales.shape)}/{tuple(wzeros.shape)} "
                             f"do not match out_features {n}")
    s = wscales.detach().to("cpu").float()
    live = (s != 0).any(dim=1)
    ng = int(torch.count_nonzero(live))
    if ng == 0 or not bool(live[:ng].all()):
        raise AwqPackedError("AWQ wscales has zero rows before its last live row — not the "
                             "ceil_num_groups padding this decoder understands")
    if k % ng:
        raise AwqPackedError(f"in_features {k} not divisible by {ng} live scale groups")
    gs = k // ng
    if num_scale_rows(k, gs) != int(wscales.shape[0]):
        raise AwqPackedError(f"AWQ scale rows {int(wscales.shape[0])} != ceil_num_groups("
                             f"{k}, {gs}) = {num_scale_rows(k, gs)}")
    z = wzeros.detach().to("cpu").float()
    return s[:ng].t().contiguous(), z[:ng].t().contiguous(), gs


class AwqPackedLinear(nn.Module):
    """Packed-resident AWQ W4A16 linear (``_AwqPackedLinear``,
    ``svdq_awq_packed.py:133-176``)."""

    _cozy_awq_packed = True

    def __init__(self, in_features: int, out_features: int, *, bias: bool,
                 compute_dtype: Any = torch.bfloat16, device: Any = None) -> None:
        super().__init__()
        if not awq_packed_supported(out_features, in_features):
            raise AwqPackedError(f"AwqPackedLinear [{out_features}, {in_features}] breaks the "
                                 f"packed contract (out%16, in%128)")
        if compute_dtype != torch.bfloat16:
            raise AwqPackedError(f"compute dtype {compute_dtype} is not supported (bf16 only)")
        self.compute_dtype = compute_dtype
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        ng = in_features // GROUP_SIZE
        dev = device or torch.device("meta")
        self.register_buffer("weight", torch.empty(out_features, in_features // 2,
                                                   dtype=torch.uint8, device=dev))
        self.register_buffer("wscales", torch.empty(out_features, ng, dtype=compute_dtype,
                                                    device=dev))
        self.register_buffer("wzeros", torch.empty(out_features, ng, dtype=compute_dtype,
                                                   device=dev))
        if bias:
            self.bias: Optional[nn.Parameter] = nn.Parameter(
                torch.empty(out_features, dtype=compute_dtype, device=dev), requires_grad=False)
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features).contiguous()
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        y = awq_w4a16_mm(x2, self.weight, self.wscales, self.wzeros,
                         None if self.bias is None else self.bias.detach())
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, lane=awq-packed")


def build_awq_packed_linear(tensors: Dict[str, torch.Tensor], out_features: int,
                            in_features: int, *, adanorm_splits: int = 1,
                            compute_dtype: Any = None, device: Any = None) -> AwqPackedLinear:
    """Packed-resident module from the on-disk AWQ tensors
    (``build_awq_packed_linear``, ``svdq_awq_packed.py:204-249``). For
    ``adanorm_splits`` > 1 the exporter's row interleave (stored row
    ``j * splits + s`` is row ``s * (N / splits) + j``) is undone and 1 is taken
    off the bias of splits 1 and ``splits - 2``."""
    missing = [k for k in ("qweight", "wscales", "wzeros") if k not in tensors]
    if missing:
        raise AwqPackedError(f"not an AWQ W4A16 linear (missing {missing})")
    compute = compute_dtype or torch.bfloat16
    n, k = int(out_features), int(in_features)
    codes = unpack_qweight(tensors["qweight"], n, k)
    scale, zero, gs = scales_and_zeros(tensors["wscales"], tensors["wzeros"], n, k)
    if gs != GROUP_SIZE:
        raise AwqPackedError(f"AWQ group size {gs} != {GROUP_SIZE} — the packed lane only ships "
                             f"the g{GROUP_SIZE} contract")
    bias = tensors.get("bias")
    splits = int(adanorm_splits)
    if splits > 1:
        if n % splits:
            raise AwqPackedError(f"out_features {n} not divisible by adanorm_splits {splits}")
        per = n // splits
        idx = torch.arange(n)
        perm = (idx % per) * splits + idx // per
        codes, scale, zero = codes[perm], scale[perm], zero[perm]
        if bias is not None:
            b = bias.detach().to("cpu").float().view(per, splits).t().contiguous()
            delta = torch.zeros(splits)
            delta[1] = 1.0
            delta[splits - 2] = 1.0
            bias = (b - delta.reshape(splits, 1)).reshape(n)
    mod = AwqPackedLinear(k, n, bias=bias is not None, compute_dtype=compute,
                          device=torch.device("cpu"))
    dev = device or "cpu"
    mod.weight = codes.contiguous().to(dev)
    mod.wscales = scale.to(compute).contiguous().to(dev)
    mod.wzeros = zero.to(compute).contiguous().to(dev)
    if bias is not None:
        mod.bias = nn.Parameter(bias.detach().to(compute).reshape(-1).to(dev), requires_grad=False)
    return mod


__all__ = ["AwqPackedError", "AwqPackedLinear", "GROUP_SIZE", "awq_packed_supported",
           "awq_w4a16_mm", "build_awq_packed_linear", "num_scale_rows", "scales_and_zeros",
           "unpack_qweight"]
