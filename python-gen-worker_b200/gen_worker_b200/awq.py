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
# The exporter pads the [rows, N] scale / zero grids to a whole number of
# row quanta: 8 groups per pack, and packs in pairs (group 64) or fours
# (group 32), i.e. 16 or 32 rows; other group sizes pad to packs of 8.
_ROW_QUANTUM = {64: 16, 32: 32}


class AwqPackedError(RuntimeError):
    """Typed packed-AWQ failure (``AwqPackedError``, ``svdq_awq_packed.py:20``)."""


def awq_packed_supported(out_features: int, in_features: int) -> bool:
    return out_features % 16 == 0 and in_features % 128 == 0


def num_scale_rows(in_features: int, group_size: int) -> int:
    """Rows of the exporter's padded scale grid for ``in_features`` split in
    groups of ``group_size`` (the count ``ceil_num_groups`` gives,
    ``svdq_awq.py:18-28``): the group count rounded up to the row quantum."""
    if in_features % group_size:
        raise AwqPackedError(f"{in_features} input features do not split into groups of "
                             f"{group_size}")
    quantum = _ROW_QUANTUM.get(group_size, 8)
    return -(-(in_features // group_size) // quantum) * quantum


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
        raise AwqPackedError(f"TinyChat unpack of a [{n}, {k}] linear needs out % 4 == 0 and "
                             f"in % 64 == 0")
    if tuple(qweight.shape) != (n // 4, k // 2):
        raise AwqPackedError(f"qweight shape {tuple(qweight.shape)}: a [{n}, {k}] linear "
                             f"stores {(n // 4, k // 2)}")
    src = qweight.detach().to("cpu").contiguous()
    out = torch.empty(n, k // 2, dtype=torch.uint8)
    native.check(native.lib().gwb_awq_qweight_unpack(ctypes.c_void_p(src.data_ptr()), n, k,
                                                    ctypes.c_void_p(out.data_ptr())),
                 "awq_qweight_unpack")
    return out


def scales_and_zeros(wscales: torch.Tensor, wzeros: torch.Tensor, out_features: int,
                     in_features: int) -> tuple[torch.Tensor, torch.Tensor, int]:
    """[rows, N] scale / zero grids -> ([N, ng], [N, ng], group size).

    The live groups are the rows above the exporter's all-zero padding,
    found by scanning up from the last row. The grid is accepted when no
    all-zero row sits among the live ones, the live count divides
    ``in_features`` and the padded height is the exporter's for that group
    size (the grids ``_scales_and_zeros`` accepts, ``svdq_awq.py:50-73``)."""
    n, k = int(out_features), int(in_features)
    if wscales.dim() != 2 or int(wscales.shape[1]) != n or wzeros.shape != wscales.shape:
        raise AwqPackedError(f"scale grid {tuple(wscales.shape)} / zero grid "
                             f"{tuple(wzeros.shape)}: want matching [rows, {n}] grids")
    s = wscales.detach().to("cpu").float()
    row_used = (s != 0).any(dim=1)
    rows = int(s.shape[0])
    live = rows
    while live > 0 and not bool(row_used[live - 1]):
        live -= 1
    if live == 0 or not bool(row_used[:live].all()):
        raise AwqPackedError("scale grid has an all-zero row among its groups (not trailing "
                             "padding)")
    if k % live:
        raise AwqPackedError(f"{live} scale groups do not divide {k} input features")
    gs = k // live
    if num_scale_rows(k, gs) != rows:
        raise AwqPackedError(f"scale grid has {rows} rows; group size {gs} pads to "
                             f"{num_scale_rows(k, gs)}")
    z = wzeros.detach().to("cpu").float()
    return s[:live].t().contiguous(), z[:live].t().contiguous(), gs


class AwqPackedLinear(nn.Module):
    """Packed-resident AWQ W4A16 linear (``_AwqPackedLinear``,
    ``svdq_awq_packed.py:133-176``)."""

    _cozy_awq_packed = True

    def __init__(self, in_features: int, out_features: int, *, bias: bool,
                 compute_dtype: Any = torch.bfloat16, device: Any = None) -> None:
        super().__init__()
        if not awq_packed_supported(out_features, in_features):
            raise AwqPackedError(f"AwqPackedLinear [{out_features}, {in_features}]: the GEMV "
                                 f"needs out % 16 == 0 and in % 128 == 0")
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
    absent = [k for k in ("qweight", "wscales", "wzeros") if k not in tensors]
    if absent:
        raise AwqPackedError(f"AWQ W4A16 linear lacks required tensor(s) {absent}")
    compute = compute_dtype or torch.bfloat16
    n, k = int(out_features), int(in_features)
    codes = unpack_qweight(tensors["qweight"], n, k)
    scale, zero, gs = scales_and_zeros(tensors["wscales"], tensors["wzeros"], n, k)
    if gs != GROUP_SIZE:
        raise AwqPackedError(f"group size {gs}: this lane runs group {GROUP_SIZE} only")
    bias = tensors.get("bias")
    splits = int(adanorm_splits)
    if splits > 1:
        if n % splits:
            raise AwqPackedError(f"{n} output rows do not split into adanorm_splits={splits}")
        per = n // splits
        # stored row j * splits + s holds logical row s * per + j
        logical = torch.arange(n)
        stored = (logical % per) * splits + logical // per
        codes, scale, zero = codes[stored], scale[stored], zero[stored]
        if bias is not None:
            b = bias.detach().to("cpu").float()[stored].view(splits, per)
            # the exporter folded +1 into the two scale chunks (split 1 and
            # split splits - 2); take it back off
            for chunk in {1, splits - 2}:
                b[chunk] -= 1.0
            bias = b.reshape(n)
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
