"""nunchaku "v1 single-file" codec (host code in libgwb200.so) against the
reference's own packers and decoder (golden fixtures) and against the
oracle's storage-order restatement at model sizes. No GPU needed."""
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import codec
from gen_worker_b200.modules import SvdqB200LayoutError

GOLD = torch.load(Path(__file__).resolve().parent / "golden" / "reference_golden.pt")
N = K = 256


def _packed():
    t = {k[len("nk_packed_"):]: v for k, v in GOLD.items() if k.startswith("nk_packed_")}
    t["wscales"] = t["wscales"].view(torch.float8_e4m3fn)
    return t


def test_oracle_storage_order_matches_reference_packers():
    assert torch.equal(O.nunchaku_pack_qweight(GOLD["nk_codes"]),
                       GOLD["nk_packed_qweight"].view(torch.uint8))
    assert torch.equal(O.nunchaku_pack_wscales(GOLD["nk_scales"]), GOLD["nk_packed_wscales"])
    assert torch.equal(O.nunchaku_pack_vector(GOLD["nk_wc"]), GOLD["nk_packed_wcscales"])
    assert torch.equal(O.nunchaku_pack_vector(GOLD["nk_smooth"]),
                       GOLD["nk_packed_smooth_factor"])
    assert torch.equal(O.nunchaku_pack_vector(GOLD["nk_bias"]), GOLD["nk_packed_bias"])
    assert torch.equal(O.nunchaku_pack_lowrank(GOLD["nk_down"], down=True),
                       GOLD["nk_packed_proj_down"])
    assert torch.equal(O.nunchaku_pack_lowrank(GOLD["nk_up"], down=False),
                       GOLD["nk_packed_proj_up"])


def test_decode_matches_reference_convert_linear():
    b = codec.decode_nunchaku_linear(_packed(), N, K)
    assert torch.equal(b["weight"], GOLD["nk_buf_weight"])
    assert torch.equal(b["weight_scale"].view(torch.uint8), GOLD["nk_buf_weight_scale"])
    assert torch.equal(b["weight_scale_2"], GOLD["nk_buf_weight_scale_2"])
    assert b["second_kind"] == "per_channel" and b["rank"] == 32
    assert torch.equal(b["proj_down"], GOLD["nk_buf_proj_down"])
    assert torch.equal(b["proj_up"], GOLD["nk_buf_proj_up"])
    assert torch.equal(b["smooth_factor"], GOLD["nk_buf_smooth"])
    assert torch.equal(b["bias"], GOLD["nk_buf_bias"])
    t = _packed()
    pt = {"qweight": t["qweight"], "wscales": t["wscales"], "wtscale": torch.tensor([0.0125])}
    bpt = codec.decode_nunchaku_linear(pt, N, K)
    assert torch.equal(bpt["weight_scale_2"], GOLD["nk_pt_weight_scale_2"])
    assert bpt["second_kind"] == "per_tensor" and bpt["rank"] == 0
    assert bpt["smooth_factor"] is None and bpt["bias"] is None


@pytest.mark.parametrize("scheme", ["int8", "fp8_e4m3"])
def test_quantized_lowrank_matches_reference(scheme):
    tag = "nk_" + scheme + "_"
    qd, qu = GOLD[tag + "qdown"], GOLD[tag + "qup"]
    if scheme == "fp8_e4m3":
        qd, qu = qd.view(torch.float8_e4m3fn), qu.view(torch.float8_e4m3fn)
    t = _packed()
    tq = {"qweight": t["qweight"], "wscales": t["wscales"], "wcscales": t["wcscales"],
          "proj_down": qd, "proj_down_scale": GOLD[tag + "sdown"], "proj_up": qu,
          "proj_up_scale": GOLD[tag + "sup"]}
    b = codec.decode_nunchaku_linear(tq, N, K, lowrank_quant=scheme)
    assert b["lowrank_quant"] == scheme
    assert torch.equal(b["proj_down"], GOLD[tag + "down"])
    assert torch.equal(b["proj_up"], GOLD[tag + "up"])


def test_split_matches_reference_split_decoded():
    parts = codec.split_nvfp4_buffers(codec.decode_nunchaku_linear(_packed(), N, K), (128, 128))
    for i, p in enumerate(parts):
        assert torch.equal(p["weight"], GOLD[f"nk_split{i}_weight"])
        assert torch.equal(p["weight_scale"].view(torch.uint8), GOLD[f"nk_split{i}_weight_scale"])
        assert torch.equal(p["weight_scale_2"], GOLD[f"nk_split{i}_weight_scale_2"])
        assert torch.equal(p["proj_up"], GOLD[f"nk_split{i}_proj_up"])
        assert torch.equal(p["bias"], GOLD[f"nk_split{i}_bias"])
        assert torch.equal(p["proj_down"], parts[0]["proj_down"])


@pytest.mark.parametrize("n,k,r", [(3072, 3072, 32), (9216, 3072, 32), (3072, 12288, 48)])
def test_decode_round_trip_at_model_sizes(n, k, r):
    """Flux shapes (qkv 3072->9216, fc2 12288->3072, rank 48): codec(oracle
    pack(x)) equals the buffers built directly from x."""
    g = torch.Generator().manual_seed(n + k + r)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    scales = torch.randint(0, 0x7F, (n, k // 16), generator=g, dtype=torch.uint8)
    wc = torch.rand(n, generator=g)
    smooth = torch.rand(k, generator=g).to(torch.bfloat16)
    rp = (r + 15) // 16 * 16
    down = torch.randn(k, rp, generator=g).to(torch.bfloat16)
    up = torch.randn(n, rp, generator=g).to(torch.bfloat16)
    t = {"qweight": O.nunchaku_pack_qweight(codes),
         "wscales": O.nunchaku_pack_wscales(scales).view(torch.float8_e4m3fn),
         "wcscales": O.nunchaku_pack_vector(wc),
         "smooth_factor": O.nunchaku_pack_vector(smooth),
         "proj_down": O.nunchaku_pack_lowrank(down, down=True),
         "proj_up": O.nunchaku_pack_lowrank(up, down=False)}
    b = codec.decode_nunchaku_linear(t, n, k)
    assert torch.equal(b["weight"], O.pack_e2m1(codes))
    assert torch.equal(b["weight_scale"].view(torch.uint8), O.to_blocked_scales(scales))
    assert torch.equal(b["weight_scale_2"].reshape(-1), wc)
    assert torch.equal(b["smooth_factor"], smooth)
    assert torch.equal(b["proj_down"], down) and torch.equal(b["proj_up"], up)


def test_refusals():
    t = _packed()
    with pytest.raises(SvdqB200LayoutError, match="lacks required"):
        codec.decode_nunchaku_linear({"qweight": t["qweight"]}, N, K)
    with pytest.raises(SvdqB200LayoutError, match="second-level weight scale"):
        codec.decode_nunchaku_linear({"qweight": t["qweight"], "wscales": t["wscales"]}, N, K)
    with pytest.raises(SvdqB200LayoutError, match="branch incomplete"):
        codec.decode_nunchaku_linear({k: v for k, v in t.items() if k != "proj_up"}, N, K)
    with pytest.raises(SvdqB200LayoutError, match="multiples of 128"):
        codec.decode_nunchaku_linear(t, N, 192)
    with pytest.raises(SvdqB200LayoutError, match="was requested"):
        codec.decode_nunchaku_linear(t, N, K, lowrank_quant="int8")
    with pytest.raises(SvdqB200LayoutError, match="is not one of"):
        codec.decode_nunchaku_linear(t, N, K, lowrank_quant="int4")
    tq = dict(t, proj_down=GOLD["nk_int8_qdown"], proj_down_scale=GOLD["nk_int8_sdown"])
    with pytest.raises(SvdqB200LayoutError, match="different storage schemes"):
        codec.decode_nunchaku_linear(tq, N, K)
    tq = dict(t, proj_down=GOLD["nk_int8_qdown"], proj_up=GOLD["nk_int8_qup"],
              proj_up_scale=GOLD["nk_int8_sup"])
    with pytest.raises(SvdqB200LayoutError, match="proj_down_scale. is absent"):
        codec.decode_nunchaku_linear(tq, N, K)
    with pytest.raises(SvdqB200LayoutError, match="entries for"):
        codec.decode_nunchaku_linear(dict(t, wcscales=t["wcscales"][:128]), N, K)
    b = codec.decode_nunchaku_linear(t, N, K)
    with pytest.raises(SvdqB200LayoutError, match="cover"):
        codec.split_nvfp4_buffers(b, (128, 64))
    with pytest.raises(SvdqB200LayoutError, match="multiple of 128 rows"):
        codec.split_nvfp4_buffers(b, (192, 64))


R128 = torch.load(Path(__file__).resolve().parent / "golden" / "reference_rank128.pt")


def r128_packed(k: int, n: int) -> dict:
    """The rank-128 nunchaku tensors of shape (k, n) packed by the reference's
    own packers (``tests/golden/make_golden.py``)."""
    tag = f"r128_{k}x{n}_packed_"
    t = {key[len(tag):]: v for key, v in R128.items() if key.startswith(tag)}
    t["wscales"] = t["wscales"].view(torch.float8_e4m3fn)
    return t


@pytest.mark.parametrize("k,n", [(512, 256), (3072, 384)])
def test_rank128_decode_matches_reference_convert_linear(k, n):
    """Rank 128, the rank of the reference's self-check and of its own
    synthesised test linears: the native decode is bit-identical to
    ``convert_linear`` at the self-check probe shapes."""
    b = codec.decode_nunchaku_linear(r128_packed(k, n), n, k)
    tag = f"r128_{k}x{n}_buf_"
    assert b["rank"] == 128
    assert torch.equal(b["weight"], R128[tag + "weight"])
    assert torch.equal(b["weight_scale"].view(torch.uint8), R128[tag + "weight_scale"])
    assert torch.equal(b["weight_scale_2"], R128[tag + "weight_scale_2"])
    assert torch.equal(b["proj_down"], R128[tag + "proj_down"])
    assert torch.equal(b["proj_up"], R128[tag + "proj_up"])
    assert torch.equal(b["smooth_factor"], R128[tag + "smooth"])
    assert torch.equal(b["bias"], R128[tag + "bias"])
