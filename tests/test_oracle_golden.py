"""The CPU oracle against fixtures produced by the reference's own functions
(tests/golden/make_golden.py)."""
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O

GOLD = torch.load(Path(__file__).parent / "golden" / "reference_golden.pt")


def test_nibble_packing_matches_reference_pack_e2m1():
    # pack_e2m1 (nvfp4_quant.py:54-56) packs raw nibble codes whose bit 3 is
    # the sign (e2m1); the INT4 packer uses the same order and the same
    # sign bit (sign-magnitude nibbles). Nibble 8 (-0) never occurs in INT4.
    nib, packed = GOLD["pack_codes"], GOLD["pack_packed"]
    assert not (nib == 8).any()
    n16 = nib.to(torch.int16)
    signed = torch.where(n16 >= 8, -(n16 & 7), n16).to(torch.int8)
    assert torch.equal(O.pack_int4(signed), packed)
    assert torch.equal(O.unpack_int4(packed), signed)


def test_int8_rule_matches_reference_quantize_lowrank():
    blk = int(GOLD["int8_block"])
    w = GOLD["int8_w"]
    r, k = w.shape
    q, s = O.quant_int8_rows(w.reshape(r * k // blk, blk))
    assert torch.equal(q.reshape(r, k), GOLD["int8_q"])
    assert torch.equal(s.reshape(r, k // blk), GOLD["int8_scale"].reshape(r, k // blk))


def test_fold_algebra_matches_reference_fold_to_dense():
    w = O.fold_dense(GOLD["fold_deq"], GOLD["fold_smooth"], GOLD["fold_down"], GOLD["fold_up"])
    assert torch.equal(w, GOLD["fold_weight"])
    assert torch.equal(GOLD["fold_bias"].float(), GOLD["fold_lin_bias"])


def test_smoothing_divide_matches_reference_bf16_semantics():
    xs = O.smooth_bf16(GOLD["smooth_x"], GOLD["fold_smooth"])
    assert torch.equal(xs.view(torch.int16), GOLD["smooth_xs"].view(torch.int16))


def test_fp8_rowwise_quantiser_matches_reference_quant_src():
    """quant_fp8_rows restates the reference's dynamic rowwise _quant_src
    (w8a8.py:261-273): e4m3 codes and f32 row scales bit for bit, including
    an all-zero row (scale clamp) and a row mostly in e4m3 subnormals."""
    q, s = O.quant_fp8_rows(GOLD["fp8_x"])
    assert torch.equal(q, GOLD["fp8_q"])
    assert torch.equal(s, GOLD["fp8_scale"].reshape(-1))
    assert int((GOLD["fp8_q"][11] & 0x78 == 0).sum()) > 100   # subnormal codes exercised


def test_nvfp4_quantiser_matches_reference_quantize_activation_torch():
    """quant_nvfp4 restates quantize_activation_torch (nvfp4_quant.py:92-103)
    with cast_e2m1's tie rule and the cuBLAS blocked scale layout: packed
    codes and blocked scales bit for bit."""
    x, s2 = GOLD["nvfp4_x"], GOLD["nvfp4_s2"]
    packed, blocked = O.quant_nvfp4(x, s2)
    assert torch.equal(packed, GOLD["nvfp4_q"])
    assert torch.equal(blocked, GOLD["nvfp4_sa"].view(torch.uint8))
    m, k = x.shape
    flat = O.from_blocked_scales(blocked, m, k // 16)
    assert torch.equal(O.to_blocked_scales(flat), blocked)


@pytest.mark.parametrize("m,k", [(1, 64), (7, 128), (33, 3072)])
def test_int4_round_trip_and_bounds(m, k):
    x = O.synth_activation(m, k, seed=m)
    packed, s = O.quant_int4(x)
    codes = O.unpack_int4(packed)
    assert codes.min() >= -7 and codes.max() <= 7
    deq = O.dequant_int4(packed, s)
    # error per element <= half a quantisation step (scale rounding adds a hair)
    err = (deq - x.float()).abs().reshape(m, k // 64, 64).amax(-1)
    assert torch.all(err <= s.float() * 0.5 * 1.001 + 1e-30)


def test_int4_zero_group_and_huge_values():
    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    x[1, 64:] = 3.0e38
    packed, s = O.quant_int4(x)
    assert s[0, 0].item() == 2.0 ** -24 and s[1, 1].item() == 65504.0
    assert torch.equal(O.unpack_int4(packed)[0], torch.zeros(128, dtype=torch.int8))
    assert torch.all(O.unpack_int4(packed)[1, 64:] == 7)


def test_group_partials_are_exact_integer_products():
    x = O.synth_activation(5, 192, seed=3)
    w = O.synth_activation(6, 192, seed=4)
    ap, _ = O.quant_int4(x)
    wp, _ = O.quant_int4(w)
    p = O.int4_group_partials(ap, wp)
    a = O.unpack_int4(ap).long()
    b = O.unpack_int4(wp).long()
    for g in range(3):
        want = a[:, 64 * g:64 * (g + 1)] @ b[:, 64 * g:64 * (g + 1)].t()
        assert torch.equal(p[g].long(), want)


def test_lora_fold_concatenates_rank():
    x = O.synth_activation(4, 256, seed=1)
    L = O.synth_svdq_layer(256, 128, 32, seed=2, x_calib=x, lora_rank=16)
    assert L["proj_down"].shape == (256, 48) and L["proj_up"].shape == (128, 48)
    # the folded branch equals the SVDQuant branch plus the additive LoRA branch
    # (w8a8_lora.py:355-382: y + (x@Aᵀ)@Bᵀ)
    full = O.lowrank_down(x, L["proj_down"]).double() @ L["proj_up"].double().t()
    parts = (O.lowrank_down(x, L["proj_down"][:, :32]).double() @ L["proj_up"][:, :32].double().t()
             + O.lowrank_down(x, L["proj_down"][:, 32:]).double() @ L["proj_up"][:, 32:].double().t())
    assert O.rel_l2(full, parts) < 1e-2


def test_fold_baseline_matches_two_branch_forward():
    x = O.synth_activation(8, 256, seed=9)
    L = O.synth_svdq_layer(256, 128, 32, seed=10, x_calib=x)
    lin = O.FoldedLinear(L["w_packed"], L["w_scale"], L["smooth"], L["proj_down"], L["proj_up"],
                         L["bias"], compute=torch.float32)
    got = lin(x.float())
    xs = x.float() / L["smooth"].float()
    want = (xs @ O.dequant_int4(L["w_packed"], L["w_scale"]).t()
            + (x.float() @ L["proj_down"].float()) @ L["proj_up"].float().t() + L["bias"].float())
    assert O.rel_l2(got, want) < 1e-5
