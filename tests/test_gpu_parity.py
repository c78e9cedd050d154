"""GPU parity of the CUDA path against the CPU oracle.

Bit-exact: INT4/INT8/FP8 activation codes and scales, int32 group partials.
bf16 outputs: rel-L2 <= 1e-3 against the oracle's bf16 output (the
correctly rounded bf16 of its float64 result), and max-abs <= 2e-2 beyond
the bf16 rounding of the float64 result itself."""
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import ops, native

ROOT = Path(__file__).resolve().parent.parent
from gen_worker_b200.modules import (build_fp8_rowwise_linear, build_svdq_int4_linear,
                                     build_svdq_nvfp4_linear, build_w8a8_int8_linear)

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
ABS_TOL = 2e-2


def _layer_case(m, k, n, rank, seed, lora=0, bias=True, smooth=True):
    x = O.synth_activation(m, k, seed)
    L = O.synth_svdq_layer(k, n, rank, seed + 1, x, lora_rank=lora, bias=bias, smooth=smooth)
    return x, L


def _quant_gpu_down_t(L):
    if L["proj_down"] is None:
        return None
    return ops.prepare_w4a4_weights(None, L["proj_down"].cuda(),
                                    L["proj_up"].cuda())["proj_down_t"]


def _quant_gpu(x, L):
    p = ops.prepare_w4a4_weights(L["w_scale"].cuda(),
                                 None if L["proj_down"] is None else L["proj_down"].cuda(),
                                 None if L["proj_up"] is None else L["proj_up"].cuda())
    sm = None if L["smooth"] is None else L["smooth"].cuda()
    codes, ascale, la = ops.svdq_w4a4_quant(x.cuda(), sm, p["proj_down_t"])
    torch.cuda.synchronize()
    return p, codes, ascale, la


@pytest.mark.parametrize("m,k", [(1, 128), (16, 256), (77, 3072), (333, 3072), (128, 12288),
                                 (4736, 1024)])
def test_int4_activation_codes_and_scales_bit_exact(cuda_ready, m, k):
    x, L = _layer_case(m, k, 128, 32, seed=m + k)
    _, codes, ascale, la = _quant_gpu(x, L)
    want_codes, want_scale = O.quant_int4(O.smooth_bf16(x, L["smooth"]))
    assert torch.equal(codes.cpu(), want_codes)
    assert torch.equal(ascale.cpu().view(torch.int16), want_scale.view(torch.int16))
    la_ref = O.lowrank_down(x, L["proj_down"])
    assert O.rel_l2(la.cpu()[:, :32], la_ref) < 1e-2
    # the hot-path quantiser writes the same codes in operand form (the
    # load-time weight expansion applies the same map), and the same scales
    # as scale-operand rows
    c2, sk8, la2 = ops.svdq_w4a4_quant_mma(x.cuda(), L["smooth"].cuda(), _quant_gpu_down_t(L))
    want_k8 = ops.svdq_w4a4_scale_k8(ascale)
    assert torch.equal(c2, ops.expand_w4a4_weight(codes))
    assert torch.equal(sk8.view(torch.int16), want_k8.view(torch.int16))
    # one-hot rows: group g's scale at k = g mod 8, zeros elsewhere
    g = torch.arange(k // 64, device=sk8.device)
    onehot = torch.nn.functional.one_hot(g % 8, 8).bool()[:, None, :]
    assert torch.all(sk8.masked_fill(onehot, 0) == 0)
    assert torch.equal(sk8[g, :, g % 8].t().contiguous().view(torch.int16),
                       ascale.view(torch.int16))
    assert torch.equal(la2, la)


def test_int4_activation_bit_exact_over_wide_value_ranges(cuda_ready):
    """25M elements spanning many binades and smoothing factors in [1e-3, 1e3]:
    the kernel's divides (reciprocal + remainder correction) must round
    exactly like the oracle's IEEE divides, codes and scales bit for bit."""
    gen = torch.Generator().manual_seed(7)
    m, k = 2048, 12288
    mant = torch.rand(m, k, generator=gen) + 0.5
    expo = torch.randint(-20, 12, (m, k), generator=gen).float()
    sign = torch.where(torch.rand(m, k, generator=gen) < 0.5, -1.0, 1.0)
    x = (sign * mant * torch.pow(2.0, expo))
    # rows whose groups clamp the scale: all-zero, tiny (amax / 7 below the
    # smallest f16 subnormal) and huge (amax / 7 above the f16 maximum)
    x[0] = 0.0
    x[1] = x[1] * 2.0 ** -40
    x[2] = x[2] * 2.0 ** 12
    x = x.to(torch.bfloat16)
    smooth = torch.pow(10.0, torch.rand(k, generator=gen) * 6 - 3).to(torch.bfloat16)
    codes, ascale, _ = ops.svdq_w4a4_quant(x.cuda(), smooth.cuda(), None)
    want_codes, want_scale = O.quant_int4(O.smooth_bf16(x, smooth))
    assert torch.equal(codes.cpu(), want_codes)
    assert torch.equal(ascale.cpu().view(torch.int16), want_scale.view(torch.int16))
    # the operand-form quantiser (the GEMM's input on the hot path) on the
    # same values: the operand bytes of the same codes, the same scales
    c8, sk8, _ = ops.svdq_w4a4_quant_mma(x.cuda(), smooth.cuda(), None)
    assert torch.equal(c8, ops.expand_w4a4_weight(want_codes.cuda()))
    assert torch.equal(sk8.view(torch.int16),
                       ops.svdq_w4a4_scale_k8(want_scale.cuda()).view(torch.int16))


def test_int4_activation_without_smoothing(cuda_ready):
    x, L = _layer_case(64, 512, 128, 0, seed=5, smooth=False)
    _, codes, ascale, _ = _quant_gpu(x, L)
    want_codes, want_scale = O.quant_int4(O.smooth_bf16(x, None))
    assert torch.equal(codes.cpu(), want_codes)
    assert torch.equal(ascale.cpu().view(torch.int16), want_scale.view(torch.int16))


@pytest.mark.parametrize("m,k,n", [(128, 128, 128), (200, 384, 256), (256, 3072, 384)])
def test_int4_group_partials_bit_exact(cuda_ready, m, k, n):
    x, L = _layer_case(m, k, n, 0, seed=m + n)
    _, codes, _, _ = _quant_gpu(x, L)
    got = ops.svdq_w4a4_group_partials(codes, ops.expand_w4a4_weight(L["w_packed"].cuda()))
    want = O.int4_group_partials(codes.cpu(), L["w_packed"])
    assert torch.equal(got.cpu(), want)
    assert native.device_error() == 0


@pytest.mark.parametrize("m,k,n,rank,lora,gelu", [
    (128, 128, 128, 0, 0, False),
    (256, 3072, 384, 32, 0, False),
    (77, 512, 256, 32, 0, True),
    (300, 1024, 128, 32, 16, False),   # rank 48 (LoRA folded)
    (64, 256, 128, 16, 0, False),
    (264, 512, 256, 16, 0, False),     # M % 8 == 0 with a partial last row tile
])
def test_int4_linear_matches_oracle(cuda_ready, m, k, n, rank, lora, gelu):
    x, L = _layer_case(m, k, n, rank, seed=3 * m + n, lora=lora)
    buf = {"weight": L["w_packed"], "weight_scale": L["w_scale"], "smooth_factor": L["smooth"],
           "proj_down": L["proj_down"], "proj_up": L["proj_up"], "bias": L["bias"]}
    mod = build_svdq_int4_linear(buf, gelu=gelu, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.svdq_int4_linear(x, L["smooth"], L["w_packed"], L["w_scale"], L["proj_down"],
                              L["proj_up"], L["bias"], gelu=gelu)
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


@pytest.mark.parametrize("m,k,n,rank", [(300, 1024, 256, 32), (128, 512, 128, 0)])
def test_packed_activation_gemm_matches_operand_form(cuda_ready, m, k, n, rank):
    """gwb_svdq_w4a4_gemm_packed (packed codes unpacked in shared memory)
    gives the same output as the operand-form GEMM."""
    x, L = _layer_case(m, k, n, rank, seed=17 * m)
    p, codes, ascale, la = _quant_gpu(x, L)
    sk8 = ops.svdq_w4a4_scale_k8(ascale)
    w_q8 = ops.expand_w4a4_weight(L["w_packed"].cuda())
    bias = L["bias"].cuda()
    a = ops.svdq_w4a4_gemm_packed(codes, sk8, w_q8, p["w_scale_k8"], la if rank else None,
                                  p["proj_up_pad"], bias, False)
    b = ops.svdq_w4a4_gemm(ops.expand_w4a4_weight(codes), sk8, w_q8, p["w_scale_k8"],
                           la if rank else None, p["proj_up_pad"], bias, False)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("m,k,n", [(77, 1024, 256), (1024, 3072, 640)])
def test_int4_gemm_promotion_matches_exact_sum(cuda_ready, m, k, n):
    """Without bias and low-rank branch the GEMM returns bf16(sum_g a_scale *
    w_scale * V_g) with the sum kept in f32: compared with the same sum in
    float64 from the bit-exact group partials, the error stays within the
    bf16 output rounding plus a few f32 ulps of the sum of magnitudes."""
    x, L = _layer_case(m, k, n, 0, seed=11 * m + n)
    p, codes, ascale, _ = _quant_gpu(x, L)
    w_q8 = ops.expand_w4a4_weight(L["w_packed"].cuda())
    part = ops.svdq_w4a4_group_partials(codes, w_q8).double()           # [G, M, N]
    sa = ascale.double().t()[:, :, None]                                    # [G, M, 1]
    sw = L["w_scale"].cuda().double().t()[:, None, :]                       # [G, 1, N]
    terms = part * sa * sw
    exact = terms.sum(0)
    mag = terms.abs().sum(0)
    a_q8, a_sk8, _ = ops.svdq_w4a4_quant_mma(x.cuda(), L["smooth"].cuda(), None)
    y = ops.svdq_w4a4_gemm(a_q8, a_sk8, w_q8, p["w_scale_k8"], None, None, None, False)
    err = (y.double() - exact).abs()
    # bf16 output rounding (2^-9 relative) plus f32 accumulation (G * 2^-24)
    bound = exact.abs() * 2.0 ** -8 + mag * (k // 64) * 2.0 ** -23 + 1e-30
    assert bool((err <= bound).all()), float((err / bound).max())
    assert native.device_error() == 0


@pytest.mark.parametrize("m,k", [(1, 128), (77, 3072), (256, 12288)])
def test_int8_activation_bit_exact(cuda_ready, m, k):
    x = O.synth_activation(m, k, seed=m)
    q, s = ops.w8a8_quant(x.cuda())
    wq, ws = O.quant_int8_rows(x)
    assert torch.equal(q.cpu(), wq)
    assert torch.equal(s.cpu(), ws)


@pytest.mark.parametrize("m,k,n,gelu", [(128, 128, 256, False), (333, 3072, 512, True),
                                         (64, 1024, 256, False)])
def test_w8a8_linear_matches_oracle(cuda_ready, m, k, n, gelu):
    x = O.synth_activation(m, k, seed=k + n)
    L = O.synth_w8a8_layer(k, n, seed=m)
    mod = build_w8a8_int8_linear({"weight": L["w_q"], "weight_scale": L["w_scale"],
                                  "bias": L["bias"]}, gelu=gelu, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.w8a8_int8_linear(x, L["w_q"], L["w_scale"], L["bias"], gelu=gelu)
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


# ---------------------------------------------------------------- FP8 rowwise
@pytest.mark.parametrize("m,k", [(1, 128), (77, 3072), (256, 12288), (48, 512)])
def test_fp8_activation_bit_exact(cuda_ready, m, k):
    """e4m3 codes and f32 row scales bit-identical to the oracle's
    restatement of the reference's _quant_src (pinned by the golden
    fixture); the (48, 512) case is the fixture's own input."""
    if (m, k) == (48, 512):
        x = torch.load(Path(__file__).parent / "golden" / "reference_golden.pt")["fp8_x"]
    else:
        x = O.synth_activation(m, k, seed=m + 3) * torch.pow(
            2.0, torch.randint(-10, 10, (m, 1), generator=torch.Generator().manual_seed(m))
        ).to(torch.bfloat16)
        x = x.to(torch.bfloat16)
    q, s = ops.fp8_quant(x.cuda())
    want_q, want_s = O.quant_fp8_rows(x)
    assert torch.equal(q.cpu(), want_q)
    assert torch.equal(s.cpu(), want_s)


@pytest.mark.parametrize("m,k,n,gelu", [(128, 128, 256, False), (333, 3072, 512, True),
                                        (1024, 3072, 1024, False)])
def test_fp8_linear_matches_oracle(cuda_ready, m, k, n, gelu):
    x = O.synth_activation(m, k, seed=5 * m)
    L = O.synth_fp8_layer(k, n, seed=m + n)
    mod = build_fp8_rowwise_linear({"weight": L["w_q"], "weight_scale": L["w_scale"],
                                    "bias": L["bias"]}, gelu=gelu, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.fp8_rowwise_linear(x, L["w_q"], L["w_scale"], L["bias"], gelu=gelu)
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


# ---------------------------------------------------------------- NVFP4
@pytest.mark.parametrize("m,k,smooth", [(128, 512, False), (333, 3072, True),
                                        (1024, 12288, False), (64, 256, False)])
def test_nvfp4_quant_bit_exact(cuda_ready, m, k, smooth):
    """Codes, blocked e4m3 scales and s2 bit-identical to the oracle's
    restatement of quantize_activation_torch (pinned to the reference by the
    golden fixture); the shapes are the reference's own identity probes
    (nvfp4_quant.py:21) plus the fixture's."""
    if (m, k) == (64, 256):
        x = torch.load(Path(__file__).parent / "golden" / "reference_golden.pt")["nvfp4_x"]
    else:
        x = O.synth_activation(m, k, seed=m + k)
    sm = (torch.rand(k, generator=torch.Generator().manual_seed(k)) + 0.5).to(torch.bfloat16) \
        if smooth else None
    codes, sblk, work = ops.nvfp4_quant(x.cuda(), None if sm is None else sm.cuda())
    xs = O.smooth_bf16(x, sm)
    s2 = O.nvfp4_s2(xs)
    want_codes, want_blk = O.quant_nvfp4(xs, s2)
    assert torch.equal(work.cpu()[1:2], s2.reshape(1))
    assert torch.equal(codes.cpu(), want_codes)
    assert torch.equal(sblk.cpu(), want_blk)


@pytest.mark.parametrize("m,k,rank,smooth", [(300, 3072, 32, True), (128, 512, 16, False),
                                            (1000, 1024, 64, True)])
def test_nvfp4_quant_lowrank_matches_separate_passes(cuda_ready, m, k, rank, smooth):
    """The fused amax + down-projection pass: codes, scales and s2 identical
    to gwb_nvfp4_quant, la = bf16(x · proj_down) on raw x within bf16
    rounding of the exact product."""
    gen = torch.Generator().manual_seed(m + k)
    x = O.synth_activation(m, k, seed=m)
    sm = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16) if smooth else None
    down = (torch.randn(k, rank, generator=gen) * 0.05).to(torch.bfloat16)
    down_t = down.t().contiguous().cuda()
    smc = None if sm is None else sm.cuda()
    c1, b1, w1, la = ops.nvfp4_quant_lowrank(x.cuda(), smc, down_t)
    c0, b0, w0 = ops.nvfp4_quant(x.cuda(), smc)
    assert torch.equal(c1, c0) and torch.equal(b1, b0)
    assert torch.equal(w1[:2], w0[:2])
    want = x.double() @ down.double()
    la_rec = ops.nvfp4_la_from_la3(la, w1).cpu()
    assert O.rel_l2(la_rec, want) <= 4e-3
    # the three-part form: u_hi repeated, and (u_hi + u_lo) * s2 within bf16
    # rounding of the exact product (the reference rounds x · proj_down to bf16)
    assert torch.equal(la[:, :rank], la[:, 2 * rank:])
    bound = want.abs() * 2.0 ** -8 + (x.double().abs() @ down.double().abs()) * k * 2.0 ** -24
    assert bool(((la_rec.double() - want).abs() <= bound + 1e-30).all())
    assert native.device_error() == 0


def test_nvfp4_quant_rounding_ties(cuda_ready):
    """Codes at the e2m1 rounding ties and at -0: with amax = 2688 the
    per-tensor s2 is 1, and a 16-block whose largest magnitude is 6 gets the
    block scale 1, so q = x exactly. The reference's rule (count of bounds
    below |q|, plus one at 0.75, 1.75 and 2.5; sign bit when q < 0) differs
    from round-to-nearest-even at 2.5 and 3.5."""
    ties = [6.0, 2.5, 3.5, -2.5, -3.5, -0.0, 0.25, 0.75, 1.25, 1.75, 5.0, -0.25, -0.1,
            0.1, -5.0, -6.0]
    x = torch.zeros(128, 64)
    x[0, :16] = torch.tensor(ties)
    x[1, :16] = -torch.tensor(ties)
    x[2, 16] = 2688.0
    x[3, 32:48] = torch.tensor(ties) * 0.5
    x = x.to(torch.bfloat16)
    codes, sblk, work = ops.nvfp4_quant(x.cuda(), None)
    s2 = O.nvfp4_s2(x)
    want_codes, want_blk = O.quant_nvfp4(x, s2)
    assert float(s2) == 1.0
    assert torch.equal(codes.cpu(), want_codes)
    assert torch.equal(sblk.cpu(), want_blk)


@pytest.mark.parametrize("m,k,n,rank,per_channel", [(128, 256, 256, 0, False),
                                                    (300, 3072, 256, 32, False),
                                                    (512, 1024, 768, 32, True),
                                                    (1000, 3072, 1024, 48, False)])
def test_nvfp4_linear_matches_oracle(cuda_ready, m, k, n, rank, per_channel):
    gen = torch.Generator().manual_seed(m + n)
    x = O.synth_activation(m, k, seed=7 * m)
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
    smooth = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16)
    packed, blocked, ws2 = O.quant_nvfp4_weight(w.float() * smooth.float())
    if per_channel:
        ws2 = ws2.reshape(1, 1) * (torch.rand(1, n, generator=gen) + 0.5)
    down = (torch.randn(k, rank, generator=gen) * 0.02).to(torch.bfloat16) if rank else None
    up = (torch.randn(n, rank, generator=gen) * 0.02).to(torch.bfloat16) if rank else None
    bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
    mod = build_svdq_nvfp4_linear({"weight": packed, "weight_scale": blocked,
                                   "weight_scale_2": ws2, "smooth_factor": smooth,
                                   "proj_down": down, "proj_up": up, "bias": bias}, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.svdq_nvfp4_linear(x, smooth, packed, blocked, ws2, down, up, bias)
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


def test_nvfp4_linear_from_nunchaku_tensors(cuda_ready):
    """The reference's packers' output (nunchaku v1 storage), decoded by the
    native codec into the module, runs the NVFP4 GEMM and matches the oracle
    on the reference's own decoded buffers."""
    from gen_worker_b200 import codec
    gold = torch.load(ROOT / "tests" / "golden" / "reference_golden.pt")
    t = {k[len("nk_packed_"):]: v for k, v in gold.items() if k.startswith("nk_packed_")}
    t["wscales"] = t["wscales"].view(torch.float8_e4m3fn)
    mod = codec.build_svdq_nvfp4_from_nunchaku(t, 256, 256, device="cuda")
    x = O.synth_activation(96, 256, seed=5)
    y = mod(x.cuda()).cpu()
    want = O.svdq_nvfp4_linear(x, gold["nk_buf_smooth"], gold["nk_buf_weight"],
                               gold["nk_buf_weight_scale"], gold["nk_buf_weight_scale_2"],
                               gold["nk_buf_proj_down"], gold["nk_buf_proj_up"], gold["nk_buf_bias"])
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


# ---------------------------------------------------------------- empty and full-size inputs
def test_empty_inputs_give_empty_outputs(cuda_ready):
    """M = 0 (an empty token batch) is a no-op on every lane."""
    x, L = _layer_case(8, 256, 256, 16, seed=1)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cuda")
    assert mod(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")).shape == (0, 256)
    W = O.synth_w8a8_layer(256, 256, seed=2)
    m8 = build_w8a8_int8_linear({"weight": W["w_q"], "weight_scale": W["w_scale"],
                                 "bias": W["bias"]}, device="cuda")
    assert m8(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")).shape == (0, 256)
    F = O.synth_fp8_layer(256, 256, seed=3)
    mf = build_fp8_rowwise_linear({"weight": F["w_q"], "weight_scale": F["w_scale"],
                                   "bias": F["bias"]}, device="cuda")
    assert mf(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")).shape == (0, 256)
    assert native.device_error() == 0


@pytest.mark.parametrize("k,n", [(15360, 3072), (3072, 21504)])
def test_w4a4_full_size_rows_match_oracle(cuda_ready, k, n):
    """BASELINE config 4's widest linears at the full token count (M =
    16896): rows are quantised and multiplied independently, so 48 sampled
    output rows must equal the oracle run on those rows alone."""
    m = 16896
    gen = torch.Generator().manual_seed(k + n)
    x = O.synth_activation(m, k, seed=k)
    rows = torch.randperm(m, generator=gen)[:48].sort().values
    L = O.synth_svdq_layer(k, n, 32, seed=n, x_calib=x[rows])
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cuda")
    y = mod(x.cuda())[rows.cuda()].cpu()
    want = O.svdq_int4_linear(x[rows], L["smooth"], L["w_packed"], L["w_scale"],
                              L["proj_down"], L["proj_up"], L["bias"])
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0



@pytest.mark.parametrize("m,k,n,rank,gelu", [(300, 512, 256, 32, False), (128, 3072, 384, 0, True),
                                             (77, 1024, 128, 128, False),
                                             (1000, 3072, 1024, 48, False)])
def test_stored_weight_gemm_matches_operand_form(cuda_ready, m, k, n, rank, gelu):
    """gwb_svdq_w4a4_gemm_stored (weight and scales as stored, expanded in
    shared memory) and gwb_svdq_w4a4_gemm_packed_stored (activations packed
    too) give bit-identical outputs to the operand-form GEMM: the stored
    8-group scale rows against the one-hot activation rows form the same
    exact scale products."""
    x, L = _layer_case(m, k, n, rank, seed=13 * m + k)
    p, codes, ascale, la = _quant_gpu(x, L)
    w = L["w_packed"].cuda()
    ws = L["w_scale"].cuda()
    a_q8, a_sk8, la2 = ops.svdq_w4a4_quant_mma(x.cuda(), L["smooth"].cuda(), p["proj_down_t"])
    lr = la2 if rank else None
    bias = L["bias"].cuda()
    ref = ops.svdq_w4a4_gemm(a_q8, a_sk8, ops.expand_w4a4_weight(w), p["w_scale_k8"], lr,
                             p["proj_up_pad"], bias, gelu)
    got = ops.svdq_w4a4_gemm_stored(a_q8, a_sk8, w, ws, lr, p["proj_up_pad"], bias, gelu)
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    got2 = ops.svdq_w4a4_gemm_packed_stored(codes, ops.svdq_w4a4_scale_k8(ascale), w, ws, lr,
                                            p["proj_up_pad"], bias, gelu)
    assert torch.equal(got2.view(torch.int16), ref.view(torch.int16))
    assert native.device_error() == 0
