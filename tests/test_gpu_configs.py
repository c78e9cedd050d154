"""GPU parity at BASELINE's own configurations.

Every linear of configs 0-4 runs at its full size on the GPU; the oracle is
evaluated on sampled rows (rows of a linear are quantised and multiplied
independently, so a sampled output row must equal the oracle run on that
input row alone). Bars as elsewhere: activation codes and scales bit-exact,
bf16 outputs rel-L2 <= 1e-3 and max-abs <= 2e-2 beyond the bf16 rounding of
the float64 oracle result; the low-rank down-projection la within the bf16
rounding of the exact product plus the f32 accumulation bound."""
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import native, ops
from gen_worker_b200.modules import build_svdq_int4_linear, build_w8a8_int8_linear

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

REL_TOL = 1e-3
ABS_TOL = 2e-2

# (name, M, K, N, rank, lora_rank, gelu) — BASELINE.json configs 0, 2, 3, 4
W4A4_CONFIGS = [
    ("cfg0", 256, 3072, 3072, 32, 0, False),
    ("cfg2_qkv", 4608, 3072, 9216, 32, 0, False),
    ("cfg2_out", 4608, 3072, 3072, 32, 0, False),
    ("cfg2_fc1", 4608, 3072, 12288, 32, 0, True),
    ("cfg2_fc2", 4608, 12288, 3072, 32, 0, False),
    ("cfg3_lora48", 4608, 3072, 3072, 32, 16, False),
    ("cfg4_qkv", 16896, 3072, 9216, 32, 0, False),
    ("cfg4_out", 16896, 3072, 3072, 32, 0, False),
    ("cfg4_fc1", 16896, 3072, 12288, 32, 0, True),
    ("cfg4_fc2", 16896, 12288, 3072, 32, 0, False),
    ("cfg4_qkv_mlp", 16896, 3072, 21504, 32, 0, False),
    ("cfg4_single_out", 16896, 15360, 3072, 32, 0, False),
]


def _sample_rows(m: int, seed: int, n: int = 64) -> torch.Tensor:
    """`n` rows: the first and last 8 (partial tiles) plus seeded random ones."""
    if m <= n:
        return torch.arange(m)
    gen = torch.Generator().manual_seed(seed)
    mid = torch.randperm(m - 16, generator=gen)[: n - 16] + 8
    return torch.cat([torch.arange(8), mid, torch.arange(m - 8, m)]).unique().sort().values


def la_within_bound(la: torch.Tensor, x: torch.Tensor, down: torch.Tensor) -> bool:
    """la = bf16(x·L1) computed with f32 accumulation: within half a bf16 ulp
    (2^-8 relative, generous) of the exact product plus K f32 ulps of the sum
    of magnitudes."""
    xd, dd = x.double(), down.double()
    exact = xd @ dd
    mag = xd.abs() @ dd.abs()
    k = x.shape[1]
    bound = exact.abs() * 2.0 ** -8 + mag * k * 2.0 ** -24 + 1e-30
    return bool(((la.double() - exact).abs() <= bound).all())


@pytest.mark.parametrize("name,m,k,n,rank,lora,gelu", W4A4_CONFIGS,
                         ids=[c[0] for c in W4A4_CONFIGS])
def test_w4a4_config_matches_oracle(cuda_ready, name, m, k, n, rank, lora, gelu):
    seed = m + k + n + lora
    x = O.synth_activation(m, k, seed=seed)
    L = O.synth_svdq_layer(k, n, rank, seed=seed + 1, x_calib=x[:256], lora_rank=lora)
    rows = _sample_rows(m, seed)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]},
                                 gelu=gelu, device="cuda")
    xd = x.cuda()
    y = mod(xd)
    ys = y[rows.cuda()].cpu()
    del y
    want = O.svdq_int4_linear(x[rows], L["smooth"], L["w_packed"], L["w_scale"], L["proj_down"],
                              L["proj_up"], L["bias"], gelu=gelu)
    assert O.rel_l2(ys, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(ys, want["y64"]) <= ABS_TOL
    # the quantiser on the full tensor: sampled rows bit-exact
    p = mod.prepare()
    codes, ascale, la = ops.svdq_w4a4_quant(xd, mod.smooth_factor, p["proj_down_t"])
    rc = rows.cuda()
    assert torch.equal(codes[rc].cpu(), want["a_packed"])
    assert torch.equal(ascale[rc].cpu().view(torch.int16), want["a_scale"].view(torch.int16))
    r = L["proj_down"].shape[1]
    assert la_within_bound(la[rc].cpu()[:, :r], x[rows], L["proj_down"])
    assert native.device_error() == 0


def test_w4a4_group_partials_bit_exact_at_cfg2_shape(cuda_ready):
    """Every 64-group integer partial sum of the tcgen05 GEMM at the full
    cfg2 attention-out shape (M 4608, K 3072, N 3072), checked bit for bit on
    a sample of rows x columns spanning every tile position."""
    m, k, n = 4608, 3072, 3072
    x = O.synth_activation(m, k, seed=901)
    L = O.synth_svdq_layer(k, n, 0, seed=902, x_calib=x[:256])
    codes, _, _ = ops.svdq_w4a4_quant(x.cuda(), L["smooth"].cuda(), None)
    got = ops.svdq_w4a4_group_partials(codes, ops.expand_w4a4_weight(L["w_packed"].cuda()))
    rows = _sample_rows(m, 903, 96)
    cols = _sample_rows(n, 904, 96)
    sub = got[:, rows.cuda()][:, :, cols.cuda()].cpu()
    del got
    want = O.int4_group_partials(codes[rows.cuda()].cpu(), L["w_packed"][cols])
    assert torch.equal(sub, want)
    assert native.device_error() == 0


def test_w8a8_cfg1_matches_oracle(cuda_ready):
    """Config 1: W8A8 at the Flux MLP fc1 shape (M 4096, K 3072, N 12288)
    with the fused GELU(tanh); quantiser bit-exact on the sampled rows."""
    m, k, n = 4096, 3072, 12288
    x = O.synth_activation(m, k, seed=811)
    L = O.synth_w8a8_layer(k, n, seed=812)
    mod = build_w8a8_int8_linear({"weight": L["w_q"], "weight_scale": L["w_scale"],
                                  "bias": L["bias"]}, gelu=True, device="cuda")
    rows = _sample_rows(m, 813)
    xd = x.cuda()
    ys = mod(xd)[rows.cuda()].cpu()
    want = O.w8a8_int8_linear(x[rows], L["w_q"], L["w_scale"], L["bias"], gelu=True)
    assert O.rel_l2(ys, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(ys, want["y64"]) <= ABS_TOL
    q, s = ops.w8a8_quant(xd)
    assert torch.equal(q[rows.cuda()].cpu(), want["a_q"])
    assert torch.equal(s[rows.cuda()].cpu(), want["a_scale"])
    assert native.device_error() == 0


# ---------------------------------------------------------------- rank 128
R128 = torch.load(ROOT / "tests" / "golden" / "reference_rank128.pt")


def _r128(k, n):
    tag = f"r128_{k}x{n}_"
    t = {key[len(tag + "packed_"):]: v for key, v in R128.items()
         if key.startswith(tag + "packed_")}
    t["wscales"] = t["wscales"].view(torch.float8_e4m3fn)
    buf = {key[len(tag + "buf_"):]: v for key, v in R128.items() if key.startswith(tag + "buf_")}
    return t, buf


@pytest.mark.parametrize("m,k,n", [(128, 512, 256), (77, 3072, 384)])
def test_nvfp4_rank128_nunchaku_linear_matches_oracle(cuda_ready, m, k, n):
    """A rank-128 nunchaku v1 linear packed by the reference's own packers,
    decoded by the native codec into the NVFP4 module, at the reference's
    self-check probe shapes (svdq_fused.py:25 with rank 128 as at :430);
    N = 384 runs a half-width last N tile."""
    from gen_worker_b200 import codec
    t, buf = _r128(k, n)
    mod = codec.build_svdq_nvfp4_from_nunchaku(t, n, k, device="cuda")
    assert mod.rank == 128
    x = O.synth_activation(m, k, seed=m + k)
    y = mod(x.cuda()).cpu()
    want = O.svdq_nvfp4_linear(x, buf["smooth"], buf["weight"], buf["weight_scale"],
                               buf["weight_scale_2"], buf["proj_down"], buf["proj_up"],
                               buf["bias"])
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


@pytest.mark.parametrize("m,k,n,rank", [(128, 512, 256, 128), (77, 3072, 384, 128),
                                        (300, 1024, 256, 100)])
def test_int4_rank_up_to_128_matches_oracle(cuda_ready, m, k, n, rank):
    """The INT4 lane with the low-rank branch at rank 128 (two operand-ring
    slots of 64 ranks) and at rank 100 (padded to 112)."""
    x = O.synth_activation(m, k, seed=3 * m + rank)
    L = O.synth_svdq_layer(k, n, rank, seed=m + n, x_calib=x)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.svdq_int4_linear(x, L["smooth"], L["w_packed"], L["w_scale"], L["proj_down"],
                              L["proj_up"], L["bias"])
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    p = mod.prepare()
    _, _, la = ops.svdq_w4a4_quant(x.cuda(), mod.smooth_factor, p["proj_down_t"])
    assert la_within_bound(la.cpu()[:, :rank], x, L["proj_down"])
    assert native.device_error() == 0


@pytest.mark.parametrize("m,k,rank", [(333, 3072, 128), (128, 512, 112)])
def test_nvfp4_quant_lowrank_rank128(cuda_ready, m, k, rank):
    gen = torch.Generator().manual_seed(m + rank)
    x = O.synth_activation(m, k, seed=m)
    sm = (torch.rand(k, generator=gen) + 0.5).to(torch.bfloat16)
    down = (torch.randn(k, rank, generator=gen) * 0.05).to(torch.bfloat16)
    c1, b1, w1, la = ops.nvfp4_quant_lowrank(x.cuda(), sm.cuda(), down.t().contiguous().cuda())
    c0, b0, w0 = ops.nvfp4_quant(x.cuda(), sm.cuda())
    assert torch.equal(c1, c0) and torch.equal(b1, b0) and torch.equal(w1[:2], w0[:2])
    assert la_within_bound(ops.nvfp4_la_from_la3(la, w1).cpu(), x, down)
    assert native.device_error() == 0


def test_dual_block_chain_matches_oracle(cuda_ready):
    """The bench's dual-stream block as a chain (out -> fc1 with GELU -> fc2,
    each layer fed with the previous layer's bf16 output) at 192 tokens,
    against the oracle running the same chain on its own outputs: every
    layer's output meets the single-linear bar against the oracle fed with
    the GPU's input, and the chain's end result stays within rel-L2 5e-3 of
    the all-oracle chain (quantisation codes may flip where an input differs
    in its last bf16 bit, so the end-to-end bar is looser)."""
    m = 192
    x = O.synth_activation(m, 3072, seed=501)
    specs = [(3072, 3072, False), (3072, 12288, True), (12288, 3072, False)]
    layers = []
    calib = x[:128]
    for i, (k, n, gelu) in enumerate(specs):
        if i:
            calib = O.synth_activation(128, k, seed=510 + i)
        L = O.synth_svdq_layer(k, n, 32, seed=520 + i, x_calib=calib)
        mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                      "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                      "proj_up": L["proj_up"], "bias": L["bias"]},
                                     gelu=gelu, device="cuda")
        layers.append((L, mod, gelu))
    h_gpu, h_ref = x.cuda(), x
    for L, mod, gelu in layers:
        y = mod(h_gpu)
        step = O.svdq_int4_linear(h_gpu.cpu(), L["smooth"], L["w_packed"], L["w_scale"],
                                  L["proj_down"], L["proj_up"], L["bias"], gelu=gelu)
        assert O.rel_l2(y.cpu(), step["y"]) <= REL_TOL
        assert O.max_abs_beyond_bf16(y.cpu(), step["y64"]) <= ABS_TOL
        h_ref = O.svdq_int4_linear(h_ref, L["smooth"], L["w_packed"], L["w_scale"],
                                   L["proj_down"], L["proj_up"], L["bias"], gelu=gelu)["y"]
        h_gpu = y
    assert O.rel_l2(h_gpu.cpu(), h_ref) <= 5e-3
    assert native.device_error() == 0


@pytest.mark.parametrize("rank", [32, 128])
def test_int4_linear_is_batch_invariant(cuda_ready, rank):
    """A row's quantised codes, scales, la and output do not depend on how
    many rows share the call: rows 0..76 computed alone, inside 2112 rows (the
    8-GPU shard size) and inside 4736 rows (several tiles per CTA) are
    bit-identical. The multi-GPU shard check relies on this."""
    k, n = 3072, 384
    x = O.synth_activation(4736, k, seed=41 + rank)
    L = O.synth_svdq_layer(k, n, rank, seed=43, x_calib=x[:512])
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cuda")
    xc = x.cuda()
    q_ref = mod.quantize(xc[:77].contiguous())
    y_ref = mod(xc[:77].contiguous())
    for m in (2112, 4736):
        q = mod.quantize(xc[:m].contiguous())
        assert torch.equal(q[0][:77], q_ref[0])                         # operand-form codes
        assert torch.equal(q[1][:, :77].view(torch.int16), q_ref[1].view(torch.int16))
        assert torch.equal(q[2][:77], q_ref[2])                         # la
        assert torch.equal(mod(xc[:m].contiguous())[:77], y_ref)
    assert native.device_error() == 0
