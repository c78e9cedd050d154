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

Artifacts the reference refuses are refused here too (missing ``qweight`` /
``wscales``, no second-level scale, half a low-rank pair, shapes the pack
forbids, mixed or undeclared low-rank schemes), checked against one contract
table, :class:`SvdqB200LayoutError`. No CPU fallback
is involved: the codec is host code by design (it runs once, at load).
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, NamedTuple, Optional, Sequence

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
        raise SvdqB200LayoutError(f"qweight of a [{n}, {k}] linear: sizes must be multiples "
                                  f"of 128 (128 x 128 fragments)")
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
        raise SvdqB200LayoutError(f"wscales of a [{n}, {k}] linear: out_features must be a "
                                  f"multiple of {_WARP_N} and in_features of 64")
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
        raise SvdqB200LayoutError(f"packed vector of length {n}: the layout needs a "
                                  f"multiple of {_WARP_N}")
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
        raise SvdqB200LayoutError(f"{what} of shape [{rows}, {rank}]: the 16 x 16 pack needs "
                                  f"both sizes to be multiples of 16")
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
        raise SvdqB200LayoutError(f"a {q.dtype} factor has no block scales to apply")
    src = _host(q).view(torch.uint8)
    rows, cols = int(src.shape[0]), int(src.shape[1])
    n = rows if block_dim == 0 else cols
    if n % 32:
        raise SvdqB200LayoutError(f"blocked dimension {n} of a low-rank factor is not a "
                                  f"multiple of 32")
    want = (n // 32, cols) if block_dim == 0 else (rows, n // 32)
    s = _host(scale).float()
    if tuple(s.shape) != want:
        raise SvdqB200LayoutError(f"low-rank scale shape {tuple(s.shape)} != {want} for a "
                                  f"{(rows, cols)} factor blocked along dim {block_dim}")
    out = torch.empty(rows, cols, dtype=torch.bfloat16)
    _call("gwb_lowrank_dequant", _ptr(src), _ptr(s), rows, cols, int(block_dim),
          0 if scheme == "int8" else 1, _ptr(out))
    return out


class _Artifact(NamedTuple):
    """What the contract check learned about one linear's tensor set."""
    second_kind: str          # "per_channel" (wcscales) or "per_tensor" (wtscale)
    scheme: str               # storage of the low-rank factors: bf16, int8, fp8_e4m3
    rank: int                 # 0 when the linear has no low-rank branch


# The nunchaku v1 linear as a contract: tensors that must be present, the
# alternatives for the second-level weight scale (exactly one used), and the
# low-rank factors, which come as a pair with per-32-block scales when stored
# quantised. Each rule is checked in table order; the first broken rule is
# reported.
_REQUIRED = ("qweight", "wscales")
_SECOND_LEVEL = (("wcscales", "per_channel"), ("wtscale", "per_tensor"))
_LOWRANK_PAIR = ("proj_down", "proj_up")
_LOWRANK_SCALES = ("proj_down_scale", "proj_up_scale")


def _check_contract(t: Dict[str, torch.Tensor], n: int, k: int,
                    lowrank_quant: Optional[str]) -> _Artifact:
    known = ("bf16",) + LOWRANK_SCHEMES
    if lowrank_quant is not None and lowrank_quant not in known:
        raise SvdqB200LayoutError(f"lowrank_quant {lowrank_quant!r} is not one of "
                                  f"{', '.join(known)}")
    absent = [name for name in _REQUIRED if name not in t]
    if absent:
        raise SvdqB200LayoutError(f"nunchaku linear lacks required tensor(s) {absent}: "
                                  f"this is not an SVDQuant W4A4 artifact")
    if n % 128 or k % 128:
        raise SvdqB200LayoutError(f"qweight of a [{n}, {k}] linear: the 4-bit layout stores "
                                  f"128 x 128 fragments, so both sizes must be multiples of 128")
    second = next((kind for name, kind in _SECOND_LEVEL if name in t), None)
    if second is None:
        raise SvdqB200LayoutError("no second-level weight scale: expected 'wcscales' (per "
                                  "output channel) or 'wtscale' (per tensor)")
    if second == "per_channel" and int(t["wcscales"].numel()) != n:
        raise SvdqB200LayoutError(f"'wcscales' has {int(t['wcscales'].numel())} entries for "
                                  f"{n} output channels")
    present = [name for name in _LOWRANK_PAIR if name in t]
    if len(present) == 1:
        raise SvdqB200LayoutError(f"low-rank branch incomplete: only {present[0]!r} is present")
    if not present:
        return _Artifact(second, "bf16", 0)
    down, up = t["proj_down"], t["proj_up"]
    scheme, scheme_up = _scheme_of(down), _scheme_of(up)
    if scheme != scheme_up:
        raise SvdqB200LayoutError(f"proj_down ({scheme}) and proj_up ({scheme_up}) use "
                                  f"different storage schemes")
    if lowrank_quant is not None and lowrank_quant != scheme:
        raise SvdqB200LayoutError(f"lowrank_quant={lowrank_quant!r} was requested but the "
                                  f"factors are stored as {scheme!r}")
    scales = [name for name in _LOWRANK_SCALES if name in t]
    if scheme == "bf16" and scales:
        raise SvdqB200LayoutError(f"{scales} given for 16-bit low-rank factors, which carry "
                                  f"no block scales")
    if scheme != "bf16" and len(scales) < 2:
        gone = [name for name in _LOWRANK_SCALES if name not in t]
        raise SvdqB200LayoutError(f"{scheme} low-rank factors need both block-scale tensors; "
                                  f"{gone[0]!r} is absent")
    rank = int(down.shape[1])
    if int(down.shape[0]) != k:
        raise SvdqB200LayoutError(f"proj_down shape {tuple(down.shape)}: expected "
                                  f"[in_features={k}, rank]")
    if tuple(up.shape) != (n, rank):
        raise SvdqB200LayoutError(f"proj_up shape {tuple(up.shape)}: expected "
                                  f"[out_features={n}, rank={rank}]")
    return _Artifact(second, scheme, rank)


def decode_nunchaku_linear(tensors: Dict[str, torch.Tensor], out_features: int,
                           in_features: int, *,
                           lowrank_quant: Optional[str] = None) -> Dict[str, Any]:
    """One nunchaku svdq linear -> the :class:`SvdqNvfp4Linear` buffer dict
    (``weight``, ``weight_scale``, ``weight_scale_2``, ``second_kind``,
    ``proj_down``, ``proj_up``, ``smooth_factor``, ``bias``, ``rank``,
    ``lowrank_quant``), host tensors. The tensor set is validated against
    the contract table above before any tensor is decoded."""
    n, k = int(out_features), int(in_features)
    art = _check_contract(tensors, n, k, lowrank_quant)
    buf: Dict[str, Any] = {
        "weight": qweight_to_e2m1(tensors["qweight"], n, k),
        "weight_scale": wscales_to_blocked(tensors["wscales"], n, k),
        "second_kind": art.second_kind, "rank": art.rank, "lowrank_quant": art.scheme,
    }
    if art.second_kind == "per_channel":
        buf["weight_scale_2"] = unpack_vector(tensors["wcscales"].float(), n).reshape(1, n)
    else:
        buf["weight_scale_2"] = _host(tensors["wtscale"]).float().reshape(1, 1)
    buf["proj_down"] = buf["proj_up"] = None
    if art.rank and art.scheme == "bf16":
        buf["proj_down"] = unpack_lowrank(tensors["proj_down"], down=True)
        buf["proj_up"] = unpack_lowrank(tensors["proj_up"], down=False)
    elif art.rank:
        buf["proj_down"] = dequant_lowrank(tensors["proj_down"], tensors["proj_down_scale"],
                                           block_dim=0)
        buf["proj_up"] = dequant_lowrank(tensors["proj_up"], tensors["proj_up_scale"],
                                         block_dim=1)
    for name, length in (("smooth_factor", k), ("bias", n)):
        v = tensors.get(name)
        buf[name] = None if v is None else unpack_vector(v, length)
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
        raise SvdqB200LayoutError(f"sections {tuple(sections)} cover {total} rows of a "
                                  f"{n}-row projection")
    if any(int(s) % 128 for s in sections):
        raise SvdqB200LayoutError(f"sections {tuple(sections)} must each be a multiple of "
                                  f"128 rows (one blocked scale tile)")
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
