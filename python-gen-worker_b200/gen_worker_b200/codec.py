"""Load-time codec: nunchaku "v1 single-file" SVDQuant linears -> the buffers
of :class:`SvdqNvfp4Linear` as stored.

Counterpart of the reference's ``decode_linear`` + ``to_buffers``
(``src/gen_worker/models/svdq_layout.py:363-438``, ``:473-483``) and
``split_decoded`` (``:441-470``). The reference decodes into a row-major
"logical" domain and then re-packs into its module buffers; here each
tensor goes from nunchaku's storage order straight to the buffer layout in
one native host pass (``gwb_nunchaku_*`` in ``include/gwb200.h``):

* ``qweight`` I8 [N, K/2] -> ``weight`` u8 [N, K/2] packed e2m1, even k in
  the low nibble;
* ``wscales`` E4M3 [K/16, N] -> ``weight_scale`` in the cuBLAS blocked
  layout;
* ``wcscales`` -> ``weight_scale_2`` f32 [1, N] (or ``wtscale`` -> [1, 1]);
* ``smooth_factor`` / ``bias`` pack_scale vectors -> row-major;
* ``proj_down`` / ``proj_up`` pack_lowrank 16-bit factors -> [K, r] / [N, r],
  or int8 / e4m3 factors with per-32-block scales -> bf16.

The same refusals as the reference: missing ``qweight`` / ``wscales``, no
second-level scale, half a low-rank pair, shapes the pack forbids, mixed or
undeclared low-rank schemes -> :class:`SvdqB200LayoutError`. No CPU fallback
is involved: the codec is host code by design (it runs once, at load).
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, Optional, Sequence

import torch

from . import native
from .modules import SvdqB200LayoutError, SvdqNvfp4Linear, build_svdq_nvfp4_linear

LOWRANK_SCHEMES = ("int8", "fp8_e4m3")
_WARP_N = 128


def _host(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu").contiguous()


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _call(fn: str, *args: Any) -> None:
    code = getattr(native.lib(), fn)(*args)
    if code != 0:
        raise SvdqB200LayoutError(f"{fn}: status {code} ({native.status_string(code)})")


def qweight_to_e2m1(qweight: torch.Tensor, out_features: int, in_features: int) -> torch.Tensor:
    """nunchaku ``qweight`` [N, K/2] -> packed e2m1 ``weight`` u8 [N, K/2]."""
    n, k = int(out_features), int(in_features)
    if n % 128 or k % 128:
        raise SvdqB200LayoutError(
            f"svdq qweight [{n}, {k}] is not a multiple of the padded fragment tile (128x128)")
    src = _host(qweight).view(torch.uint8)
    if src.numel() != n * k // 2:
        raise SvdqB200LayoutError(f"qweight has {src.numel()} bytes, expected {n * k // 2}")
    out = torch.empty(n, k // 2, dtype=torch.uint8)
    _call("gwb_nunchaku_qweight_to_e2m1", _ptr(src), n, k, _ptr(out))
    return out


def wscales_to_blocked(wscales: torch.Tensor, out_features: int, in_features: int) -> torch.Tensor:
    """nunchaku ``wscales`` E4M3 [K/16, N] -> blocked ``weight_scale`` e4m3."""
    n, k = int(out_features), int(in_features)
    if n % _WARP_N or (k // 16) % 4 or k % 16:
        raise SvdqB200LayoutError(
            f"svdq wscales for [{n}, {k}] break the lane swizzle (out%{_WARP_N}, (in/16)%4)")
    src = _host(wscales).view(torch.uint8)
    if src.numel() != n * k // 16:
        raise SvdqB200LayoutError(f"wscales has {src.numel()} bytes, expected {n * k // 16}")
    out = torch.empty(n * k // 16, dtype=torch.uint8)
    _call("gwb_nunchaku_wscales_to_blocked", _ptr(src), n, k, _ptr(out))
    return out.view(torch.float8_e4m3fn)


def unpack_vector(vec: torch.Tensor, n: int) -> torch.Tensor:
    """One pack_scale(group_size=-1) vector -> row-major [n] (same dtype)."""
    n = int(n)
    if n % _WARP_N:
        raise SvdqB200LayoutError(
            f"svdq packed vector length {n} is not a multiple of warp_n={_WARP_N}")
    src = _host(vec).reshape(-1)
    if src.numel() != n:
        raise SvdqB200LayoutError(f"packed vector has {src.numel()} elements, expected {n}")
    out = torch.empty_like(src)
    _call("gwb_nunchaku_vector_unpack", _ptr(src), n, src.element_size(), _ptr(out))
    return out


def unpack_lowrank(w: torch.Tensor, *, down: bool) -> torch.Tensor:
    """pack_lowrank 16-bit factor [rows, rank] -> row-major [rows, rank]
    (``proj_down`` [K, r] when ``down``, ``proj_up`` [N, r] otherwise)."""
    src = _host(w)
    if src.dim() != 2 or src.element_size() != 2:
        raise SvdqB200LayoutError(f"low-rank factor must be a 2-D 16-bit tensor, got "
                                  f"{tuple(src.shape)} {src.dtype}")
    rows, rank = int(src.shape[0]), int(src.shape[1])
    if rows % 16 or rank % 16:
        what = "proj_down" if down else "proj_up"
        raise SvdqB200LayoutError(f"svdq {what} [{rows}, {rank}] breaks the low-rank pack "
                                  f"(rows%16, rank%16)")
    out = torch.empty_like(src)
    _call("gwb_nunchaku_lowrank_unpack", _ptr(src), rows, rank, 1 if down else 0, _ptr(out))
    return out


def _scheme_of(t: torch.Tensor) -> str:
    if t.dtype == torch.int8:
        return "int8"
    if t.dtype == torch.float8_e4m3fn:
        return "fp8_e4m3"
    return "bf16"


def dequant_lowrank(q: torch.Tensor, scale: torch.Tensor, *, block_dim: int) -> torch.Tensor:
    """int8 / e4m3 factor with fp32 per-32-block scales -> bf16."""
    scheme = _scheme_of(q)
    if scheme == "bf16":
        raise SvdqB200LayoutError(f"dequant_lowrank got a {q.dtype} tensor — not a quantized "
                                  f"low-rank factor")
    src = _host(q).view(torch.uint8)
    rows, cols = int(src.shape[0]), int(src.shape[1])
    n = rows if block_dim == 0 else cols
    if n % 32:
        raise SvdqB200LayoutError(f"low-rank factor dim {n} is not a multiple of the quant "
                                  f"block 32")
    want = (n // 32, cols) if block_dim == 0 else (rows, n // 32)
    s = _host(scale).float()
    if tuple(s.shape) != want:
        raise SvdqB200LayoutError(f"low-rank scale shape {tuple(s.shape)} != {want} for a "
                                  f"{(rows, cols)} factor blocked along dim {block_dim}")
    out = torch.empty(rows, cols, dtype=torch.bfloat16)
    _call("gwb_lowrank_dequant", _ptr(src), _ptr(s), rows, cols, int(block_dim),
          0 if scheme == "int8" else 1, _ptr(out))
    return out


def decode_nunchaku_linear(tensors: Dict[str, torch.Tensor], out_features: int,
                           in_features: int, *,
                           lowrank_quant: Optional[str] = None) -> Dict[str, Any]:
    """One nunchaku svdq linear -> the :class:`SvdqNvfp4Linear` buffer dict
    (``weight``, ``weight_scale``, ``weight_scale_2``, ``second_kind``,
    ``proj_down``, ``proj_up``, ``smooth_factor``, ``bias``, ``rank``,
    ``lowrank_quant``), host tensors."""
    n, k = int(out_features), int(in_features)
    missing = [name for name in ("qweight", "wscales") if name not in tensors]
    if missing:
        raise SvdqB200LayoutError(f"not an svdq W4A4 linear (missing {missing})")
    buf: Dict[str, Any] = {
        "weight": qweight_to_e2m1(tensors["qweight"], n, k),
        "weight_scale": wscales_to_blocked(tensors["wscales"], n, k),
    }
    if "wcscales" in tensors:
        wc = tensors["wcscales"]
        if int(wc.numel()) != n:
            raise SvdqB200LayoutError(f"wcscales numel {int(wc.numel())} != out_features {n}")
        buf["weight_scale_2"] = unpack_vector(wc.float(), n).reshape(1, n)
        buf["second_kind"] = "per_channel"
    elif "wtscale" in tensors:
        buf["weight_scale_2"] = _host(tensors["wtscale"]).float().reshape(1, 1)
        buf["second_kind"] = "per_tensor"
    else:
        raise SvdqB200LayoutError("svdq linear has neither wcscales nor wtscale")

    down, up = tensors.get("proj_down"), tensors.get("proj_up")
    if (down is None) != (up is None):
        raise SvdqB200LayoutError("svdq linear has only one half of the low-rank branch")
    if lowrank_quant is not None and lowrank_quant not in ("bf16",) + LOWRANK_SCHEMES:
        raise SvdqB200LayoutError(f"unknown lowrank_quant declaration {lowrank_quant!r} "
                                  f"(known: bf16, {', '.join(LOWRANK_SCHEMES)})")
    rank, scheme = 0, "bf16"
    if down is not None:
        scheme = _scheme_of(down)
        if _scheme_of(up) != scheme:
            raise SvdqB200LayoutError(f"low-rank pair mixes schemes: proj_down {down.dtype} vs "
                                      f"proj_up {up.dtype}")
        if scheme == "bf16" and ("proj_down_scale" in tensors or "proj_up_scale" in tensors):
            raise SvdqB200LayoutError("low-rank scale tensors present but the branch pair is "
                                      "not stored in a quantized dtype")
        if lowrank_quant is not None and scheme != lowrank_quant:
            raise SvdqB200LayoutError(f"artifact declares lowrank_quant={lowrank_quant!r} but "
                                      f"the branch is stored as {scheme!r}")
        rank = int(down.shape[1])
        if int(down.shape[0]) != k:
            raise SvdqB200LayoutError(f"proj_down {tuple(down.shape)} does not start with "
                                      f"in_features {k}")
        if tuple(up.shape) != (n, rank):
            raise SvdqB200LayoutError(f"proj_up {tuple(up.shape)} != [out_features={n}, "
                                      f"rank={rank}]")
        if scheme == "bf16":
            buf["proj_down"] = unpack_lowrank(down, down=True)
            buf["proj_up"] = unpack_lowrank(up, down=False)
        else:
            dscale, uscale = tensors.get("proj_down_scale"), tensors.get("proj_up_scale")
            if dscale is None or uscale is None:
                miss = "proj_down_scale" if dscale is None else "proj_up_scale"
                raise SvdqB200LayoutError(f"quantized ({scheme}) low-rank branch is missing "
                                          f"{miss}")
            buf["proj_down"] = dequant_lowrank(down, dscale, block_dim=0)
            buf["proj_up"] = dequant_lowrank(up, uscale, block_dim=1)
    else:
        buf["proj_down"] = buf["proj_up"] = None
    buf["rank"], buf["lowrank_quant"] = rank, scheme
    smooth = tensors.get("smooth_factor")
    buf["smooth_factor"] = None if smooth is None else unpack_vector(smooth, k)
    bias = tensors.get("bias")
    buf["bias"] = None if bias is None else unpack_vector(bias, n)
    return buf


def split_nvfp4_buffers(buf: Dict[str, Any], sections: Sequence[int]) -> tuple:
    """Split a fused projection's buffers (nunchaku's ``to_qkv``) along N, as
    ``split_decoded`` does in the logical domain (``svdq_layout.py:441-470``).
    Each section must be a multiple of 128 rows: a blocked scale tile holds
    128 rows, so a section is then a contiguous range of tiles."""
    w = buf["weight"]
    n, k2 = int(w.shape[0]), int(w.shape[1])
    total = sum(int(s) for s in sections)
    if total != n:
        raise SvdqB200LayoutError(f"split sections {tuple(sections)} sum to {total}, not "
                                  f"out_features {n}")
    if any(int(s) % 128 for s in sections):
        raise SvdqB200LayoutError(f"split sections {tuple(sections)} are not multiples of the "
                                  f"128-row scale tile")
    tile_bytes = (k2 * 2 // 16) * 128     # one 128-row band of blocked scales
    per_channel = buf["second_kind"] == "per_channel"
    parts, start = [], 0
    for size in (int(s) for s in sections):
        stop = start + size
        p = dict(buf)
        p["weight"] = w[start:stop].contiguous()
        ws = buf["weight_scale"].view(torch.uint8).reshape(-1)
        p["weight_scale"] = ws[start // 128 * tile_bytes:stop // 128 * tile_bytes].contiguous() \
            .view(torch.float8_e4m3fn)
        if per_channel:
            p["weight_scale_2"] = buf["weight_scale_2"][:, start:stop].contiguous()
        if buf.get("proj_up") is not None:
            p["proj_up"] = buf["proj_up"][start:stop].contiguous()
        if buf.get("bias") is not None:
            p["bias"] = buf["bias"][start:stop].contiguous()
        parts.append(p)
        start = stop
    return tuple(parts)


def build_svdq_nvfp4_from_nunchaku(tensors: Dict[str, torch.Tensor], out_features: int,
                                   in_features: int, *, device: Any = None,
                                   lowrank_quant: Optional[str] = None) -> SvdqNvfp4Linear:
    """``decode_nunchaku_linear`` + module construction (the un-fused case of
    the reference's ``convert_linear``, ``svdq_layout.py:486-489``)."""
    buf = decode_nunchaku_linear(tensors, out_features, in_features, lowrank_quant=lowrank_quant)
    return build_svdq_nvfp4_linear(buf, device=device)


__all__ = [
    "build_svdq_nvfp4_from_nunchaku", "decode_nunchaku_linear", "dequant_lowrank",
    "qweight_to_e2m1", "split_nvfp4_buffers", "unpack_lowrank", "unpack_vector",
    "wscales_to_blocked",
]
