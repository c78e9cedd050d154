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
  fall into the e4m3 subnormal range after scaling.
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

    path = HERE / "reference_golden.pt"
    torch.save(out, path)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main(*sys.argv[1:])
