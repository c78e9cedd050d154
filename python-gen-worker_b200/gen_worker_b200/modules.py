"""Drop-in quantized linear modules and the module-swap seam.

``SvdqInt4Linear`` keeps the buffer names of the reference's ``SvdqLinear``
(``src/gen_worker/models/svdq_native.py:94-138``): ``weight`` (packed nibbles,
u8 [N, K/2]), ``weight_scale``, ``smooth_factor`` [K], ``proj_down`` [K, r],
``proj_up`` [N, r], ``bias`` [N]; its layout tag ``int4-g64-lownib`` names the
INT4 group-64 format (fp16 scale per 64-group, ``weight_scale`` f16
[N, K/64], even k in the low nibble, sign-magnitude nibbles). ``W8A8Int8Linear`` keeps
``Fp8ScaledLinear``'s (``src/gen_worker/models/w8a8.py:313-354``): ``weight``
s8 [N, K], ``weight_scale`` f32 [N, 1], ``bias``.

The forward is the reference's dataflow (smooth -> quantise -> GEMM -> scale
-> + (x·L1)·L2ᵀ -> + bias) executed by two native kernels; an optional
fused GELU(tanh) covers the FF projection that diffusers follows with GELU.
"""

from __future__ import annotations

from typing import Any, Dict, Optional

import torch
import torch.nn as nn

from . import ops

LAYOUT_INT4 = "int4-g64-lownib"
GROUP = 64
_K_ALIGN = 128
_N_ALIGN = 128


class SvdqB200LayoutError(ValueError):
    """A buffer set this module does not understand (``SvdqLayoutError``
    counterpart, ``svdq_layout.py:41``)."""


# ---------------------------------------------------------------- producer
def quantize_int4_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric INT4 group-64 quantisation of a [R, K] matrix (fp32 math):
    s = fp16(clamp(amax/7, 2^-24, 65504)); q = clamp(rint(w/s), -7, 7);
    packed two per byte, even k in the low nibble, sign-magnitude nibbles
    (bit 3 = sign, bits 0-2 = |q|)."""
    r, k = w.shape
    if k % GROUP:
        raise SvdqB200LayoutError(f"K={k} is not a multiple of {GROUP}")
    g = w.float().reshape(r, k // GROUP, GROUP)
    s = (g.abs().amax(dim=-1) / 7.0).clamp(min=2.0 ** -24, max=65504.0).to(torch.float16)
    q = torch.round(g / s.float().unsqueeze(-1)).clamp(-7, 7).reshape(r, k).to(torch.int16)
    q = torch.where(q < 0, 8 | (-q), q)
    packed = ((q[:, 1::2] << 4) | q[:, 0::2]).to(torch.uint8).contiguous()
    return packed, s


def quantize_int8_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric INT8 (``quantize_tree_w8a8``'s per-out-channel
    producer, ``w8a8.py:774-779``, with qmax 127)."""
    wf = w.float()
    s = (wf.abs().amax(dim=-1) / 127.0).clamp(min=1e-12)
    q = torch.round(wf / s.unsqueeze(-1)).clamp(-127, 127).to(torch.int8)
    return q, s


# ---------------------------------------------------------------- modules
class SvdqInt4Linear(nn.Module):
    _cozy_svdq_linear = True
    layout = LAYOUT_INT4

    def __init__(self, in_features: int, out_features: int, *, rank: int, bias: bool,
                 compute_dtype: Any = torch.bfloat16, smooth: bool = True,
                 gelu: bool = False, device: Any = None, weight_form: str = "stored") -> None:
        super().__init__()
        if weight_form not in ("stored", "operand"):
            raise SvdqB200LayoutError(f"weight_form {weight_form!r} is not 'stored' or 'operand'")
        self.weight_form = weight_form
        if in_features % _K_ALIGN or out_features % _N_ALIGN:
            raise SvdqB200LayoutError(
                f"SvdqInt4Linear dims [{out_features}, {in_features}] break the "
                f"tile alignment (in%{_K_ALIGN}, out%{_N_ALIGN})")
        if compute_dtype != torch.bfloat16:
            raise SvdqB200LayoutError("compute dtype must be bf16")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.rank = int(rank)
        self.gelu = bool(gelu)
        self.compute_dtype = compute_dtype
        dev = device or torch.device("meta")
        self.register_buffer("weight", torch.empty(out_features, in_features // 2,
                                                   dtype=torch.uint8, device=dev))
        self.register_buffer("weight_scale", torch.empty(out_features, in_features // GROUP,
                                                         dtype=torch.float16, device=dev))
        if smooth:
            self.register_buffer("smooth_factor", torch.empty(in_features, dtype=compute_dtype,
                                                              device=dev))
        else:
            self.smooth_factor = None
        if self.rank:
            self.register_buffer("proj_down", torch.empty(in_features, self.rank,
                                                          dtype=compute_dtype, device=dev))
            self.register_buffer("proj_up", torch.empty(out_features, self.rank,
                                                        dtype=compute_dtype, device=dev))
        else:
            self.proj_down = None
            self.proj_up = None
        if bias:
            self.bias: Optional[nn.Parameter] = nn.Parameter(
                torch.empty(out_features, dtype=compute_dtype, device=dev), requires_grad=False)
        else:
            self.bias = None
        self._packed: Optional[Dict[str, Any]] = None

    @property
    def stored(self) -> bool:
        """True when the GEMM reads ``weight`` / ``weight_scale`` as stored
        (``weight_form="stored"``, the default, and in_features % 512 == 0);
        otherwise the weight is expanded once into the e4m3 operand form at
        load time (2.4x the device memory, ~5 % faster GEMMs)."""
        return self.weight_form == "stored" and ops.stored_weights_supported(self.in_features)

    def prepare(self) -> Dict[str, Any]:
        """Kernel-layout copies of the low-rank buffers (and, when the stored
        weights cannot be read directly, of the weight and its scales), built
        once on the buffers' device."""
        dev = self.weight.device
        if self._packed is None or self._packed["device"] != dev:
            p = ops.prepare_w4a4_weights(self.weight_scale, self.proj_down, self.proj_up,
                                         weight=self.weight, operand_form=not self.stored)
            p["device"] = dev
            self._packed = p
        return self._packed

    def quantize(self, x2: torch.Tensor) -> tuple:
        """First launch of the forward: smoothing, INT4 codes and scales in
        operand form, and la = x2 · proj_down on raw x."""
        p = self.prepare()
        codes, a_sk8, la = ops.svdq_w4a4_quant_mma(x2, self.smooth_factor, p["proj_down_t"])
        return codes, a_sk8, (la if p["proj_down_t"] is not None else None)

    def gemm(self, a_q8: torch.Tensor, a_scale_k8: torch.Tensor,
             la: Optional[torch.Tensor]) -> torch.Tensor:
        """Second launch of the forward: the GEMM with the fused promotion,
        low-rank, bias and GELU epilogue."""
        p = self.prepare()
        bias = self.bias.detach() if self.bias is not None else None
        if self.stored:
            return ops.svdq_w4a4_gemm_stored(a_q8, a_scale_k8, self.weight, self.weight_scale, la,
                                             p["proj_up_pad"], bias, self.gelu)
        return ops.svdq_w4a4_gemm(a_q8, a_scale_k8, p["w_q8"], p["w_scale_k8"], la,
                                  p["proj_up_pad"], bias, self.gelu)

    def _apply(self, fn, recurse=True):  # noqa: ANN001 — drop stale repacks on .to()
        self._packed = None
        return super()._apply(fn, recurse)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = self.gemm(*self.quantize(x2))
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rank={self.rank}, bias={self.bias is not None}, "
                f"smooth={self.smooth_factor is not None}, gelu={self.gelu}, "
                f"layout={self.layout}")


class W8A8Int8Linear(nn.Module):
    _cozy_w8a8_linear = True

    def __init__(self, in_features: int, out_features: int, *, bias: bool,
                 compute_dtype: Any = torch.bfloat16, gelu: bool = False,
                 device: Any = None) -> None:
        super().__init__()
        if in_features % 128 or out_features % 256:
            raise SvdqB200LayoutError(
                f"W8A8Int8Linear dims [{out_features}, {in_features}] break the tile "
                f"alignment (in%128, out%256)")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.gelu = bool(gelu)
        self.compute_dtype = compute_dtype
        dev = device or torch.device("meta")
        self.register_buffer("weight", torch.empty(out_features, in_features, dtype=torch.int8,
                                                   device=dev))
        self.register_buffer("weight_scale", torch.empty(out_features, 1, dtype=torch.float32,
                                                         device=dev))
        if bias:
            self.bias: Optional[nn.Parameter] = nn.Parameter(
                torch.empty(out_features, dtype=compute_dtype, device=dev), requires_grad=False)
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        q, s = ops.w8a8_quant(x2)
        y = ops.w8a8_gemm(q, s, self.weight, self.weight_scale.reshape(-1),
                          self.bias.detach() if self.bias is not None else None, self.gelu)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, gelu={self.gelu}, mode=int8-rowwise")


LAYOUT_NVFP4 = "nvfp4-blocked"


class SvdqNvfp4Linear(nn.Module):
    """Drop-in for the reference's NVFP4 ``SvdqLinear`` (``src/gen_worker/
    models/svdq_native.py:94-156``) with its buffer set as stored: ``weight``
    u8 [N, K/2] (packed e2m1), ``weight_scale`` e4m3 [blocked numel] (cuBLAS
    blocked layout), ``weight_scale_2`` f32 [1, N] or [1, 1], optional
    ``smooth_factor`` [K], ``proj_down`` [K, r], ``proj_up`` [N, r], ``bias``.
    Forward: the smoothing divide, per-tensor ``s2`` with ``la = x ·
    proj_down`` (bf16 on raw x, as the reference) in the same pass, the NVFP4
    activation codes in a second pass, then one block-scaled tcgen05 GEMM whose accumulator
    starts from the low-rank product (divided by ``weight_scale_2 · s2``: the
    quantiser writes la / s2 and the load-time up-projection is proj_up /
    weight_scale_2, each as two bf16 parts, exact to ~2^-17) and ends with
    ``· s2 · weight_scale_2 + bias``. No torch op runs per call."""
    _cozy_svdq_linear = True
    layout = LAYOUT_NVFP4

    def __init__(self, in_features: int, out_features: int, *, rank: int, bias: bool,
                 per_channel_scale: bool = False, smooth: bool = True,
                 compute_dtype: Any = torch.bfloat16, device: Any = None) -> None:
        super().__init__()
        if in_features % 256 or out_features % 128:
            raise SvdqB200LayoutError(
                f"SvdqNvfp4Linear dims [{out_features}, {in_features}] break the tile "
                f"alignment (in%256, out%128)")
        if rank > 128:
            raise SvdqB200LayoutError(f"low-rank rank {rank} > 128 is not supported")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.rank = int(rank)
        self.compute_dtype = compute_dtype
        dev = device or torch.device("meta")
        self.register_buffer("weight", torch.empty(out_features, in_features // 2,
                                                   dtype=torch.uint8, device=dev))
        self.register_buffer("weight_scale", torch.empty(
            ops.nvfp4_blocked_numel(out_features, in_features), dtype=torch.float8_e4m3fn,
            device=dev))
        self.register_buffer("weight_scale_2", torch.empty(
            1, out_features if per_channel_scale else 1, dtype=torch.float32, device=dev))
        if smooth:
            self.register_buffer("smooth_factor", torch.empty(in_features, dtype=compute_dtype,
                                                              device=dev))
        else:
            self.smooth_factor = None
        if self.rank:
            self.register_buffer("proj_down", torch.empty(in_features, self.rank,
                                                          dtype=compute_dtype, device=dev))
            self.register_buffer("proj_up", torch.empty(out_features, self.rank,
                                                        dtype=compute_dtype, device=dev))
        else:
            self.proj_down = None
            self.proj_up = None
        if bias:
            self.bias: Optional[nn.Parameter] = nn.Parameter(
                torch.empty(out_features, dtype=compute_dtype, device=dev), requires_grad=False)
        else:
            self.bias = None
        self._up_pad: Optional[tuple] = None

    def _apply(self, fn, recurse=True):
        self._up_pad = None
        return super()._apply(fn, recurse)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        la = up = None
        if self.rank:
            if self._up_pad is None:
                down_pad, up_over_ws2 = ops.nvfp4_lowrank_prepare(self.proj_down, self.proj_up,
                                                                  self.weight_scale_2)
                self._up_pad = (down_pad.t().contiguous(), up_over_ws2)
            # la from the amax pass (x is read twice per call, not three times);
            # the GEMM applies s2 to the load-time proj_up / weight_scale_2
            codes, sblk, work, la = ops.nvfp4_quant_lowrank(x2, self.smooth_factor,
                                                            self._up_pad[0])
            up = self._up_pad[1]
        else:
            codes, sblk, work = ops.nvfp4_quant(x2, self.smooth_factor)
        y = ops.nvfp4_gemm(codes, sblk, work, self.weight, self.weight_scale,
                           self.weight_scale_2, la, up,
                           self.bias.detach() if self.bias is not None else None)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rank={self.rank}, bias={self.bias is not None}, "
                f"smooth={self.smooth_factor is not None}, layout={self.layout}")


def build_svdq_nvfp4_linear(buf: Dict[str, Any], *, device: Any = None) -> SvdqNvfp4Linear:
    """From the reference's NVFP4 ``SvdqBuffers`` (``svdq_layout.py:66-84``)."""
    w = buf["weight"]
    n, k2 = w.shape
    down = buf.get("proj_down")
    rank = 0 if down is None else int(down.shape[1])
    ws2 = buf["weight_scale_2"].float().reshape(1, -1)
    mod = SvdqNvfp4Linear(k2 * 2, n, rank=rank, bias=buf.get("bias") is not None,
                          per_channel_scale=ws2.shape[1] > 1,
                          smooth=buf.get("smooth_factor") is not None,
                          device=torch.device("cpu"))
    dev = device or w.device
    mod.weight = w.contiguous().to(dev)
    wsc = buf["weight_scale"]
    if wsc.dtype == torch.uint8:
        wsc = wsc.view(torch.float8_e4m3fn)
    mod.weight_scale = wsc.reshape(-1).contiguous().to(dev)
    mod.weight_scale_2 = ws2.contiguous().to(dev)
    if mod.smooth_factor is not None:
        mod.smooth_factor = buf["smooth_factor"].to(torch.bfloat16).reshape(-1).contiguous().to(dev)
    if rank:
        mod.proj_down = down.to(torch.bfloat16).contiguous().to(dev)
        mod.proj_up = buf["proj_up"].to(torch.bfloat16).contiguous().to(dev)
    if mod.bias is not None:
        mod.bias = nn.Parameter(buf["bias"].detach().to(torch.bfloat16).reshape(-1).to(dev),
                                requires_grad=False)
    return mod


class Fp8RowwiseLinear(nn.Module):
    """Drop-in for the reference's ``Fp8ScaledLinear`` in rowwise mode
    (``src/gen_worker/models/w8a8.py:359-381``): buffers ``weight``
    float8_e4m3fn [N, K], ``weight_scale`` f32 [N, 1], ``bias``; per-token
    dynamic FP8 activations; one tcgen05 kind::f8f6f4 GEMM with the scales,
    bias and (optionally) GELU(tanh) fused."""
    _cozy_w8a8_linear = True

    def __init__(self, in_features: int, out_features: int, *, bias: bool,
                 compute_dtype: Any = torch.bfloat16, gelu: bool = False,
                 device: Any = None) -> None:
        super().__init__()
        if in_features % 128 or out_features % 256:
            raise SvdqB200LayoutError(
                f"Fp8RowwiseLinear dims [{out_features}, {in_features}] break the tile "
                f"alignment (in%128, out%256)")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.gelu = bool(gelu)
        self.compute_dtype = compute_dtype
        dev = device or torch.device("meta")
        self.register_buffer("weight", torch.empty(out_features, in_features,
                                                   dtype=torch.float8_e4m3fn, device=dev))
        self.register_buffer("weight_scale", torch.empty(out_features, 1, dtype=torch.float32,
                                                         device=dev))
        if bias:
            self.bias: Optional[nn.Parameter] = nn.Parameter(
                torch.empty(out_features, dtype=compute_dtype, device=dev), requires_grad=False)
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        q, s = ops.fp8_quant(x2)
        y = ops.fp8_gemm(q, s, self.weight, self.weight_scale.reshape(-1),
                         self.bias.detach() if self.bias is not None else None, self.gelu)
        return y.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, gelu={self.gelu}, mode=fp8-rowwise")


# ---------------------------------------------------------------- builders / swap
def build_svdq_int4_linear(buf: Dict[str, Any], *, gelu: bool = False,
                           device: Any = None,
                           weight_form: str = "stored") -> SvdqInt4Linear:
    """A device-resident module from a buffer dict with the ``SvdqBuffers``
    field names (``svdq_layout.py:66-78``; ``build_svdq_linear``,
    ``svdq_native.py:173-197``)."""
    w = buf["weight"]
    n, k2 = w.shape
    down = buf.get("proj_down")
    rank = 0 if down is None else int(down.shape[1])
    mod = SvdqInt4Linear(k2 * 2, n, rank=rank, bias=buf.get("bias") is not None,
                         smooth=buf.get("smooth_factor") is not None, gelu=gelu,
                         device=torch.device("cpu"), weight_form=weight_form)
    dev = device or w.device
    ws = buf["weight_scale"]
    if tuple(ws.shape) != (n, k2 * 2 // GROUP):
        raise SvdqB200LayoutError(f"weight_scale shape {tuple(ws.shape)} != {(n, k2 * 2 // GROUP)}")
    mod.weight = w.contiguous().to(dev)
    mod.weight_scale = ws.to(torch.float16).contiguous().to(dev)
    if mod.smooth_factor is not None:
        mod.smooth_factor = buf["smooth_factor"].to(torch.bfloat16).reshape(-1).contiguous().to(dev)
    if rank:
        mod.proj_down = down.to(torch.bfloat16).contiguous().to(dev)
        mod.proj_up = buf["proj_up"].to(torch.bfloat16).contiguous().to(dev)
    if mod.bias is not None:
        mod.bias = nn.Parameter(buf["bias"].detach().to(torch.bfloat16).reshape(-1).to(dev),
                                requires_grad=False)
    return mod


def build_w8a8_int8_linear(buf: Dict[str, Any], *, gelu: bool = False,
                           device: Any = None) -> W8A8Int8Linear:
    w = buf["weight"]
    n, k = w.shape
    mod = W8A8Int8Linear(k, n, bias=buf.get("bias") is not None, gelu=gelu,
                         device=torch.device("cpu"))
    dev = device or w.device
    mod.weight = w.to(torch.int8).contiguous().to(dev)
    mod.weight_scale = buf["weight_scale"].float().reshape(n, 1).contiguous().to(dev)
    if mod.bias is not None:
        mod.bias = nn.Parameter(buf["bias"].detach().to(torch.bfloat16).reshape(-1).to(dev),
                                requires_grad=False)
    return mod


def build_fp8_rowwise_linear(buf: Dict[str, Any], *, gelu: bool = False,
                             device: Any = None) -> Fp8RowwiseLinear:
    """From the reference's W8A8 checkpoint tensors: ``weight``
    float8_e4m3fn (or its bytes) [N, K], ``weight_scale`` f32 [N] or [N, 1],
    optional ``bias``."""
    w = buf["weight"]
    n, k = w.shape
    mod = Fp8RowwiseLinear(k, n, bias=buf.get("bias") is not None, gelu=gelu,
                           device=torch.device("cpu"))
    dev = device or w.device
    if w.dtype == torch.uint8:
        w = w.view(torch.float8_e4m3fn)
    if w.dtype != torch.float8_e4m3fn:
        raise SvdqB200LayoutError(f"Fp8RowwiseLinear weight dtype {w.dtype} is not e4m3")
    mod.weight = w.contiguous().to(dev)
    mod.weight_scale = buf["weight_scale"].float().reshape(n, 1).contiguous().to(dev)
    if mod.bias is not None:
        mod.bias = nn.Parameter(buf["bias"].detach().to(torch.bfloat16).reshape(-1).to(dev),
                                requires_grad=False)
    return mod


def quantize_fp8_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's data-free W8A8 producer (``quantize_tree_w8a8``,
    ``w8a8.py:774-779``): per output row ``scale = max(amax/448, 1e-12)``,
    ``e4m3(clamp(w/scale, ±448))`` -> (float8_e4m3fn [N, K], f32 [N])."""
    wf = w.float()
    scale = (wf.abs().amax(dim=1, keepdim=True) / 448.0).clamp(min=1e-12)
    return (wf / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), scale.reshape(-1)


def fp8_rowwise_from_linear(lin: nn.Linear, gelu: bool = False) -> Fp8RowwiseLinear:
    q, s = quantize_fp8_rows(lin.weight.detach())
    buf = {"weight": q, "weight_scale": s,
           "bias": lin.bias.detach() if lin.bias is not None else None}
    return build_fp8_rowwise_linear(buf, gelu=gelu, device=lin.weight.device)


def svdq_int4_from_linear(lin: nn.Linear, smooth: Optional[torch.Tensor] = None,
                          proj_down: Optional[torch.Tensor] = None,
                          proj_up: Optional[torch.Tensor] = None,
                          gelu: bool = False) -> SvdqInt4Linear:
    """Data-free producer: quantise a dense linear's W·diag(smooth) to INT4
    group-64 (the stored weight that ``fold_to_dense`` divides back by smooth,
    ``svdq_native.py:207-208``)."""
    w = lin.weight.detach().float()
    if smooth is not None:
        w = w * smooth.to(torch.bfloat16).float().reshape(1, -1).to(w.device)
    packed, scale = quantize_int4_rows(w)
    buf = {"weight": packed, "weight_scale": scale, "smooth_factor": smooth,
           "proj_down": proj_down, "proj_up": proj_up,
           "bias": lin.bias.detach() if lin.bias is not None else None}
    return build_svdq_int4_linear(buf, gelu=gelu, device=lin.weight.device)


def swap_linears(model: nn.Module, replacements: Dict[str, nn.Module]) -> int:
    """Install modules by dotted path with ``setattr`` — the seam of
    ``swap_svdq_linears`` (``svdq_native.py:266-321``). Returns the count."""
    n = 0
    for path, mod in replacements.items():
        parent_path, _, leaf = path.rpartition(".")
        parent = model.get_submodule(parent_path) if parent_path else model
        if not hasattr(parent, leaf):
            raise SvdqB200LayoutError(f"no module at {path!r}")
        setattr(parent, leaf, mod)
        n += 1
    return n
