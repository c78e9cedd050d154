#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is readable (its path is the
first argument, default ``/root/reference``); the fixtures it writes
(``tests/golden/*.pt``) are committed and travel without the reference.
Everything is produced by CALLING the reference's own functions:

* ``pack_e2m1`` (``src/gen_worker/models/nvfp4_quant.py:54-56``) on random
  nibbles -> the nibble order the INT4 packer must reproduce;
* ``quantize_lowrank(scheme="int8")`` (``src/gen_worker/models/svdq_layout.py:261-275``)
  -> the int8 symmetric quantiser rule (scale = amax/127 clamped at 1e-12,
  divide, round half-even, clamp ±127), per 32-element block;
* ``fold_to_dense`` (``src/gen_worker/models/svdq_native.py:200-221``) on a
  synthetic NVFP4 ``DecodedLinear`` -> the fold algebra
  ``dequant(W)/smooth + proj_up·proj_downᵀ`` with the reference's own dequant;
* ``SvdqLinear``'s smoothing divide ``x2 / smooth_factor`` on bf16 tensors
  (``svdq_native.py:144``), reproduced with the reference module's forward
  arithmetic -> xs bf16;
* ``quantize_activation_torch`` (``nvfp4_quant.py:92-103``) -> the
  amax -> rounded-scale -> divide -> code structure the INT4 quantiser
  follows (kept for the NVFP4 follow-on lane);
* the FP8 rowwise activation quantiser ``_quant_src`` (dynamic, rowwise;
  ``src/gen_worker/models/w8a8.py:261-273``, reached through
  ``_build_quantizer(torch).eager_source``) -> e4m3 codes and f32 row scales
  over rows spanning many binades, an all-zero row and a row whose values
  fall into the e4m3 subnormal range after scaling;
* the nunchaku "v1 single-file" packers ``pack_qweight``, ``pack_wscales``,
  ``pack_vector``, ``pack_lowrank`` (``svdq_layout.py:165-221``) on seeded
  logical tensors, and the reference's decode of the packed tensors
  (``convert_linear``, ``split_decoded`` + ``to_buffers``,
  ``svdq_layout.py:441-489``), including int8 / e4m3 quantized low-rank
  factors (``quantize_lowrank``);
* the AWQ W4A16 exporter ``encode_awq_linear`` (``svdq_awq.py:175-210``), the
  packed-resident module's buffers ``build_awq_packed_linear``
  (``svdq_awq_packed.py:204-249``) and the decoded dense layer
  ``decode_awq_linear`` (``svdq_awq.py:108-132``), plain and with the adaLN
  split interleave (6 splits).
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _shim() -> None:
    """The reference's generated protobuf/grpc modules pin library versions
    newer/older than this image's; neutralise only the version checks."""
    try:
        import google.protobuf.runtime_version as rv  # type: ignore
        rv.ValidateProtobufRuntimeVersion = lambda *a, **k: None
    except Exception:  # noqa: BLE001
        pass
    try:
        import grpc  # type: ignore
        grpc.__version__ = "1.99.0"
    except Exception:  # noqa: BLE001
        sys.modules.setdefault("grpc", types.ModuleType("grpc"))


def main(ref_root: str = "/root/reference") -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    _shim()
    from gen_worker.models import nvfp4_quant as nq
    from gen_worker.models import svdq_layout as sl
    from gen_worker.models import svdq_native as sn
    from gen_worker.models import w8a8

    gen = torch.Generator().manual_seed(1234)
    out = {}

    # 1. nibble packing order
    # nibbles 0..15 except 8 (e2m1 -0), which sign-magnitude INT4 never uses
    nib = torch.randint(0, 15, (8, 64), generator=gen, dtype=torch.uint8)
    nib = nib + (nib >= 8).to(torch.uint8)
    out["pack_codes"] = nib
    out["pack_packed"] = nq.pack_e2m1(nib)

    # 2. int8 symmetric quantiser, blocks of LOWRANK_QUANT_BLOCK along dim 1
    w = torch.randn(16, 128, generator=gen) * 3.0
    w[3] = 0.0                     # all-zero block -> clamp path
    w[5, :32] *= 1e-14             # tiny amax -> clamp path
    q, s = sl.quantize_lowrank(w, scheme="int8", block_dim=1)
    out["int8_w"], out["int8_q"], out["int8_scale"] = w, q, s
    out["int8_block"] = torch.tensor(sl.LOWRANK_QUANT_BLOCK)

    # 3. fold algebra with the reference's own dequant
    n, k, r = 256, 512, 32
    codes = torch.randint(0, 16, (n, k), generator=gen, dtype=torch.uint8)
    scales = (torch.rand(n, k // nq.BLOCK, generator=gen) * 4 + 0.5).to(torch.float8_e4m3fn)
    second = torch.tensor([0.01])
    down = (torch.randn(k, r, generator=gen) * 0.05).to(torch.bfloat16)
    up = (torch.randn(n, r, generator=gen) * 0.05).to(torch.bfloat16)
    smooth = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16)
    bias = torch.randn(n, generator=gen).to(torch.bfloat16)
    dec = sl.DecodedLinear(out_features=n, in_features=k, codes=codes, scales=scales,
                           second=second, second_kind="per_tensor", rank=r, proj_down=down,
                           proj_up=up, smooth_factor=smooth, bias=bias)
    lin = sn.fold_to_dense(dec, compute_dtype=torch.float32)
    out["fold_deq"] = sl.dequantize_decoded(dec)
    out["fold_smooth"], out["fold_down"], out["fold_up"], out["fold_bias"] = smooth, down, up, bias
    out["fold_weight"] = lin.weight.detach().clone()
    out["fold_lin_bias"] = lin.bias.detach().clone()

    # 4. smoothing divide on bf16 tensors (SvdqLinear.forward arithmetic)
    x = (torch.randn(32, k, generator=gen) * 4).to(torch.bfloat16)
    out["smooth_x"] = x
    out["smooth_xs"] = x / smooth          # bf16 / bf16, exactly as svdq_native.py:144

    # 5. NVFP4 quantiser structure
    xa = (torch.randn(64, 256, generator=gen) * 2).to(torch.bfloat16)
    s2 = (xa.abs().amax().float() / (6.0 * 448.0)).clamp(min=1e-12)
    qa, sa = nq.quantize_activation_torch(xa, s2)
    out["nvfp4_x"], out["nvfp4_s2"], out["nvfp4_q"], out["nvfp4_sa"] = xa, s2, qa, sa

    # 6. FP8 rowwise activation quantiser (the reference's own eager source)
    quant_src = w8a8._build_quantizer(torch).eager_source
    xf = torch.randn(48, 512, generator=gen)
    xf = xf * torch.pow(2.0, torch.randint(-12, 10, (48, 1), generator=gen).float())
    xf[7] = 0.0                                      # all-zero row -> clamp path
    xf[11, :] *= 1e-3
    xf[11, 0] = 1000.0                               # most of the row lands in e4m3 subnormals
    xf = xf.to(torch.bfloat16)
    fq, fs = quant_src(xf, False, None)
    out["fp8_x"], out["fp8_q"], out["fp8_scale"] = xf, fq.view(torch.uint8), fs

    # 7. nunchaku "v1 single-file" codec: logical tensors packed by the
    # reference's own forward packers, and the reference's decode
    # (`convert_linear` = decode_linear + to_buffers) of the packed tensors
    n, k, r = 256, 256, 32
    codes = torch.randint(0, 16, (n, k), generator=gen, dtype=torch.uint8)
    scales = (torch.rand(n, k // nq.BLOCK, generator=gen) * 6 + 0.1).to(torch.float8_e4m3fn)
    wc = torch.rand(n, generator=gen) * 0.02 + 0.001
    smooth = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16)
    bias = torch.randn(n, generator=gen).to(torch.bfloat16)
    down = (torch.randn(k, r, generator=gen) * 0.05).to(torch.bfloat16)     # [in, rank]
    up = (torch.randn(n, r, generator=gen) * 0.05).to(torch.bfloat16)       # [out, rank]
    packed = {
        "qweight": sl.pack_qweight(codes),
        "wscales": sl.pack_wscales(scales, n, k),
        "wcscales": sl.pack_vector(wc, n),
        "smooth_factor": sl.pack_vector(smooth, k),
        "bias": sl.pack_vector(bias, n),
        "proj_down": sl.pack_lowrank(down.t().contiguous(), down=True),
        "proj_up": sl.pack_lowrank(up, down=False),
    }
    buf = sl.convert_linear(packed, n, k)
    out["nk_codes"], out["nk_scales"] = codes, scales.view(torch.uint8)
    out["nk_wc"], out["nk_smooth"], out["nk_bias"] = wc, smooth, bias
    out["nk_down"], out["nk_up"] = down, up
    for key, val in packed.items():
        out["nk_packed_" + key] = val.view(torch.uint8) if val.dtype == torch.float8_e4m3fn else val
    out["nk_buf_weight"] = buf.weight
    out["nk_buf_weight_scale"] = buf.weight_scale.view(torch.uint8)
    out["nk_buf_weight_scale_2"] = buf.weight_scale_2
    out["nk_buf_proj_down"], out["nk_buf_proj_up"] = buf.proj_down, buf.proj_up
    out["nk_buf_smooth"], out["nk_buf_bias"] = buf.smooth_factor, buf.bias
    # per-tensor second-level scale, no low-rank branch, no smoothing
    pt = {"qweight": packed["qweight"], "wscales": packed["wscales"],
          "wtscale": torch.tensor([0.0125])}
    bpt = sl.convert_linear(pt, n, k)
    out["nk_pt_weight_scale_2"] = bpt.weight_scale_2
    # quantized low-rank branch (int8 and e4m3, blocks of 32 along the
    # contraction dim of each factor)
    for scheme in ("int8", "fp8_e4m3"):
        qd, sd = sl.quantize_lowrank(down, scheme=scheme, block_dim=0)
        qu, su = sl.quantize_lowrank(up, scheme=scheme, block_dim=1)
        tq = {"qweight": packed["qweight"], "wscales": packed["wscales"],
              "wcscales": packed["wcscales"], "proj_down": qd, "proj_down_scale": sd,
              "proj_up": qu, "proj_up_scale": su}
        bq = sl.convert_linear(tq, n, k)
        tag = "nk_" + scheme + "_"
        out[tag + "qdown"] = qd.view(torch.uint8) if qd.dtype == torch.float8_e4m3fn else qd
        out[tag + "qup"] = qu.view(torch.uint8) if qu.dtype == torch.float8_e4m3fn else qu
        out[tag + "sdown"], out[tag + "sup"] = sd, su
        out[tag + "down"], out[tag + "up"] = bq.proj_down, bq.proj_up
    # fused projection split along N (split_decoded) on the decoded buffers
    parts = sl.split_decoded(sl.decode_linear(packed, n, k), (128, 128))
    for i, part in enumerate(parts):
        bp = sl.to_buffers(part)
        out[f"nk_split{i}_weight"] = bp.weight
        out[f"nk_split{i}_weight_scale"] = bp.weight_scale.view(torch.uint8)
        out[f"nk_split{i}_weight_scale_2"] = bp.weight_scale_2
        out[f"nk_split{i}_proj_up"] = bp.proj_up
        out[f"nk_split{i}_bias"] = bp.bias

    # 8. AWQ W4A16 modulation layers: the reference's exporter
    # (encode_awq_linear), its packed-resident module buffers
    # (build_awq_packed_linear) and its decoded dense weights (decode_awq_linear)
    from gen_worker.models import svdq_awq as sa
    from gen_worker.models import svdq_awq_packed as sp
    for oc, ic, splits in ((256, 256, 1), (384, 128, 6)):
        w = torch.randn(oc, ic, generator=gen) * 0.05
        b = torch.randn(oc, generator=gen)
        t = sa.encode_awq_linear(w, b, adanorm_splits=splits)
        ref = sa.decode_awq_linear(t, oc, ic, adanorm_splits=splits)
        tag = f"awq{oc}_"
        for key, val in t.items():
            out[tag + "t_" + key] = val
        out[tag + "dense_w"] = ref.weight.detach().clone()
        out[tag + "dense_b"] = ref.bias.detach().clone()
        if sp.awq_op() is not None:
            mod = sp.build_awq_packed_linear(t, oc, ic, adanorm_splits=splits)
            out[tag + "mod_weight"] = mod.weight.clone()
            out[tag + "mod_wscales"] = mod.wscales.clone()
            out[tag + "mod_wzeros"] = mod.wzeros.clone()
            out[tag + "mod_bias"] = mod.bias.detach().clone()

    path = HERE / "reference_golden.pt"
    torch.save(out, path)
    print(f"wrote {path} ({path.stat().st_size} bytes)")
    rank128(sl, nq)


def rank128(sl, nq) -> None:
    """Rank-128 nunchaku v1 linears at the reference's self-check probe
    shapes (``svdq_fused.py:25``, rank 128 at ``:430``; the rank the
    reference's own tests synthesise, ``tests/test_svdq_native_pgw685.py:224``):
    logical tensors packed by the reference's forward packers, and the
    reference's ``convert_linear`` buffers of the packed tensors. Written to
    its own file so the main fixture stays byte-identical."""
    gen = torch.Generator().manual_seed(4321)
    out = {}
    r = 128
    for k, n in ((512, 256), (3072, 384)):
        codes = torch.randint(0, 16, (n, k), generator=gen, dtype=torch.uint8)
        scales = (torch.rand(n, k // nq.BLOCK, generator=gen) * 6 + 0.1).to(torch.float8_e4m3fn)
        wc = torch.rand(n, generator=gen) * 0.02 + 0.001
        smooth = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16)
        bias = torch.randn(n, generator=gen).to(torch.bfloat16)
        down = (torch.randn(k, r, generator=gen) * 0.05).to(torch.bfloat16)
        up = (torch.randn(n, r, generator=gen) * 0.05).to(torch.bfloat16)
        packed = {
            "qweight": sl.pack_qweight(codes),
            "wscales": sl.pack_wscales(scales, n, k),
            "wcscales": sl.pack_vector(wc, n),
            "smooth_factor": sl.pack_vector(smooth, k),
            "bias": sl.pack_vector(bias, n),
            "proj_down": sl.pack_lowrank(down.t().contiguous(), down=True),
            "proj_up": sl.pack_lowrank(up, down=False),
        }
        buf = sl.convert_linear(packed, n, k)
        tag = f"r128_{k}x{n}_"
        for key, val in packed.items():
            out[tag + "packed_" + key] = (val.view(torch.uint8) if val.dtype == torch.float8_e4m3fn
                                          else val)
        out[tag + "buf_weight"] = buf.weight
        out[tag + "buf_weight_scale"] = buf.weight_scale.view(torch.uint8)
        out[tag + "buf_weight_scale_2"] = buf.weight_scale_2
        out[tag + "buf_proj_down"], out[tag + "buf_proj_up"] = buf.proj_down, buf.proj_up
        out[tag + "buf_smooth"], out[tag + "buf_bias"] = buf.smooth_factor, buf.bias
    path = HERE / "reference_rank128.pt"
    torch.save(out, path)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main(*sys.argv[1:])
