"""AWQ W4A16 modulation lane: load-time decode (native TinyChat unpack +
scale grids + adaLN split undo) against the reference's own exporter and
packed-resident module (golden fixtures), and the GEMV kernel against the
oracle on the GPU."""
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import awq, native

GOLD = torch.load(Path(__file__).resolve().parent / "golden" / "reference_golden.pt")
REL_TOL = 1e-3
ABS_TOL = 2e-2


def _tensors(oc):
    p = f"awq{oc}_t_"
    return {k[len(p):]: v for k, v in GOLD.items() if k.startswith(p)}


@pytest.mark.parametrize("oc,ic,splits", [(256, 256, 1), (384, 128, 6)])
def test_module_buffers_match_reference(oc, ic, splits):
    m = awq.build_awq_packed_linear(_tensors(oc), oc, ic, adanorm_splits=splits)
    assert torch.equal(m.weight, GOLD[f"awq{oc}_mod_weight"])
    assert torch.equal(m.wscales, GOLD[f"awq{oc}_mod_wscales"])
    assert torch.equal(m.wzeros, GOLD[f"awq{oc}_mod_wzeros"])
    assert torch.equal(m.bias.detach(), GOLD[f"awq{oc}_mod_bias"])
    # the weight the kernel dequantises is the reference's decoded nn.Linear weight
    assert torch.equal(O.awq_dequant(m.weight, m.wscales, m.wzeros), GOLD[f"awq{oc}_dense_w"])
    assert torch.equal(m.bias.detach(), GOLD[f"awq{oc}_dense_b"])


def test_oracle_tinychat_pack_matches_reference_exporter():
    m = awq.build_awq_packed_linear(_tensors(256), 256, 256)
    codes = torch.empty(256, 256, dtype=torch.uint8)
    codes[:, 0::2], codes[:, 1::2] = m.weight & 0xF, m.weight >> 4
    assert torch.equal(O.awq_pack_qweight(codes), GOLD["awq256_t_qweight"])


def test_unpack_round_trip_at_model_size():
    """Flux dual-block modulation (3072 -> 6 x 3072)."""
    g = torch.Generator().manual_seed(3)
    n, k = 18432, 3072
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    w = awq.unpack_qweight(O.awq_pack_qweight(codes), n, k)
    assert torch.equal(w, O.pack_e2m1(codes))


def test_refusals():
    t = _tensors(256)
    with pytest.raises(awq.AwqPackedError, match="lacks required"):
        awq.build_awq_packed_linear({"qweight": t["qweight"]}, 256, 256)
    with pytest.raises(awq.AwqPackedError, match="qweight shape"):
        awq.build_awq_packed_linear(t, 256, 512)
    with pytest.raises(awq.AwqPackedError, match="adanorm_splits"):
        awq.build_awq_packed_linear(t, 256, 256, adanorm_splits=6)
    bad = dict(t, wscales=t["wscales"].clone())
    bad["wscales"][0] = 0
    with pytest.raises(awq.AwqPackedError, match="all-zero row"):
        awq.build_awq_packed_linear(bad, 256, 256)
    with pytest.raises(awq.AwqPackedError, match="GEMV needs"):
        awq.AwqPackedLinear(200, 256, bias=False)
    assert not awq.awq_packed_supported(500, 256) and awq.awq_packed_supported(512, 256)
    assert awq.num_scale_rows(3072, 64) == 48 and awq.num_scale_rows(256, 64) == 16


@pytest.mark.gpu
@pytest.mark.parametrize("oc,ic,splits", [(256, 256, 1), (384, 128, 6)])
@pytest.mark.parametrize("m", [1, 2, 3])
def test_gemv_matches_oracle_on_reference_layers(cuda_ready, oc, ic, splits, m):
    mod = awq.build_awq_packed_linear(_tensors(oc), oc, ic, adanorm_splits=splits, device="cuda")
    x = (torch.randn(m, ic, generator=torch.Generator().manual_seed(m)) * 2).to(torch.bfloat16)
    y = mod(x.cuda()).cpu()
    want = O.awq_linear(x, mod.weight.cpu(), mod.wscales.cpu(), mod.wzeros.cpu(),
                        mod.bias.detach().cpu())
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    assert native.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("n,k,m", [(18432, 3072, 1), (18432, 3072, 2), (9216, 3072, 2),
                                   (3072, 12288, 5), (3072, 3072, 20)])
def test_gemv_matches_oracle_at_flux_sizes(cuda_ready, n, k, m):
    g = torch.Generator().manual_seed(n + m)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    ws = (torch.rand(n, k // 64, generator=g) * 0.01 + 1e-3).to(torch.bfloat16)
    wz = (-torch.rand(n, k // 64, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    weight = O.pack_e2m1(codes)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    y = awq.awq_w4a16_mm(x.cuda(), weight.cuda(), ws.cuda(), wz.cuda(), bias.cuda()).cpu()
    want = O.awq_linear(x, weight, ws, wz, bias)
    assert O.rel_l2(y, want["y"]) <= REL_TOL
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= ABS_TOL
    empty = awq.awq_w4a16_mm(torch.empty(0, k, dtype=torch.bfloat16, device="cuda"),
                             weight.cuda(), ws.cuda(), wz.cuda(), None)
    assert empty.shape == (0, n)
    assert native.device_error() == 0
