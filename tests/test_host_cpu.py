"""Host-side logic without a GPU: library load + exported symbols, producer
rules vs the oracle, load-time repacks, op validation."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import native, ops
from gen_worker_b200.modules import (Fp8RowwiseLinear, SvdqInt4Linear, W8A8Int8Linear,
                                     SvdqB200LayoutError, quantize_fp8_rows, quantize_int4_rows,
                                     quantize_int8_rows, swap_linears, build_svdq_int4_linear)

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    text = (ROOT / "include" / "gwb200.h").read_text()
    return sorted(set(re.findall(r"\b(gwb_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = native.lib()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(native.EXPORTED)
    assert "sm_100a" in native.build_info()


def test_status_strings():
    assert native.status_string(0) == "success"
    assert "aligned" in native.status_string(2)


def test_without_gpu_the_ops_refuse_loudly():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(ops.SvdqB200Error):
        ops.svdq_w4a4_quant(torch.zeros(4, 128, dtype=torch.bfloat16), None, None)
    assert native.extension_reason() is not None


def test_entry_points_reject_bad_shapes_before_touching_memory():
    lib = native.lib()
    # K not a multiple of 128 / N not a multiple of 128 -> GWB_E_SHAPE (1), no launch
    assert lib.gwb_svdq_w4a4_gemm(None, None, None, None, None, None, None, 4, 128, 100, 0, 0,
                                  None, None) == 1
    assert lib.gwb_svdq_w4a4_gemm(None, None, None, None, None, None, None, 4, 100, 128, 0, 0,
                                  None, None) == 1
    assert lib.gwb_svdq_w4a4_quant(None, None, None, 4, 128, 24, None, None, None, None) == 1
    assert lib.gwb_svdq_w4a4_quant_mma(None, None, None, 4, 100, 0, None, None, None, None) == 1
    assert lib.gwb_svdq_w4a4_scale_k8(None, 4, 100, None, None) == 1
    assert lib.gwb_w8a8_linear(None, None, None, None, 4, 128, 100, 0, None, None, None, None) == 1
    # null data pointers with valid sizes -> GWB_E_SHAPE (1), no launch
    assert lib.gwb_svdq_w4a4_quant(None, None, None, 4, 128, 0, None, None, None, None) == 1
    assert lib.gwb_svdq_w4a4_quant_mma(None, None, None, 4, 128, 0, None, None, None, None) == 1
    assert lib.gwb_svdq_w4a4_gemm(None, None, None, None, None, None, None, 4, 128, 128, 0, 0,
                                  None, None) == 1
    assert lib.gwb_svdq_w4a4_gemm_packed(None, None, None, None, None, None, None, 4, 128, 128,
                                         0, 0, None, None) == 1
    assert lib.gwb_svdq_w4a4_linear(*([None] * 7), 4, 128, 128, 0, 0, *([None] * 5)) == 1
    assert lib.gwb_svdq_w4a4_linear_noalloc(*([None] * 7), 4, 128, 128, 0, 0, None, None) == 1
    assert lib.gwb_svdq_w4a4_group_partials(None, None, 4, 128, 128, None, None) == 1
    assert lib.gwb_w8a8_quant(None, 4, 128, None, None, None) == 1
    assert lib.gwb_fp8_quant(None, 4, 128, None, None, None) == 1
    assert lib.gwb_w8a8_gemm(None, None, None, None, None, 4, 256, 128, 0, None, None) == 1
    assert lib.gwb_fp8_gemm(None, None, None, None, None, 4, 256, 128, 0, None, None) == 1
    assert lib.gwb_nvfp4_quant(None, None, 4, 128, None, None, None, None) == 1
    assert lib.gwb_awq_w4a16_mm(None, None, None, None, None, 1, 128, 128, None, None) == 1
    # M == 0 is a no-op success
    assert lib.gwb_svdq_w4a4_linear(*([None] * 7), 0, 128, 128, 0, 0, *([None] * 5)) == 0


def test_producer_matches_oracle_rules():
    w = O.synth_activation(16, 256, seed=1).float()
    p, s = quantize_int4_rows(w)
    op, os_ = O.quant_int4(w)
    assert torch.equal(p, op) and torch.equal(s, os_)
    q8, s8 = quantize_int8_rows(w)
    oq, osc = O.quant_int8_rows(w)
    assert torch.equal(q8, oq) and torch.equal(s8, osc)
    f8, fs = quantize_fp8_rows(w)
    ofq, ofs = O.quant_fp8_weight(w)
    assert torch.equal(f8.view(torch.uint8), ofq) and torch.equal(fs, ofs)


def test_prepare_repacks_layouts():
    ws = torch.rand(256, 4).to(torch.float16)
    down = torch.randn(256, 20).to(torch.bfloat16)
    up = torch.randn(128, 20).to(torch.bfloat16)
    p = ops.prepare_w4a4_weights(ws, down, up)
    assert p["w_scale_k8"] is None      # CPU tensors: the scale rows are built on the GPU
    assert p["proj_down_t"].shape == (32, 256) and torch.all(p["proj_down_t"][20:] == 0)
    assert torch.equal(p["proj_down_t"][:20], down.t())
    assert p["proj_up_pad"].shape == (128, 32) and torch.all(p["proj_up_pad"][:, 20:] == 0)
    with pytest.raises(ops.SvdqB200Error):
        ops.prepare_w4a4_weights(ws, torch.zeros(256, 144), torch.zeros(128, 144))


def test_module_surface_and_swap():
    with pytest.raises(SvdqB200LayoutError):
        SvdqInt4Linear(100, 128, rank=0, bias=False)
    with pytest.raises(SvdqB200LayoutError):
        W8A8Int8Linear(128, 128, bias=False)
    with pytest.raises(SvdqB200LayoutError):
        Fp8RowwiseLinear(128, 128, bias=False)
    f = Fp8RowwiseLinear(256, 256, bias=True)
    assert f.weight.dtype == torch.float8_e4m3fn and tuple(f.weight_scale.shape) == (256, 1)
    m = SvdqInt4Linear(256, 128, rank=32, bias=True)
    names = {n for n, _ in m.named_buffers()} | {n for n, _ in m.named_parameters()}
    assert {"weight", "weight_scale", "smooth_factor", "proj_down", "proj_up", "bias"} <= names
    assert m.layout == "int4-g64-lownib"
    model = torch.nn.Sequential(torch.nn.Linear(256, 128), torch.nn.Linear(128, 128))
    x = O.synth_activation(4, 256, seed=0)
    L = O.synth_svdq_layer(256, 128, 32, seed=1, x_calib=x)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cpu")
    assert swap_linears(model, {"0": mod}) == 1 and model[0] is mod
    with pytest.raises(SvdqB200LayoutError):
        swap_linears(model, {"7": mod})


def test_bench_clock_summary_keeps_the_timed_region(tmp_path):
    """The bench's clock record: samples taken before the timed region opened
    are dropped; a region shorter than one sampling interval falls back to
    the last sample before it instead of reporting no clocks."""
    import bench
    p = tmp_path / "clocks.csv"
    p.write_text("0, 1200, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                 "0, 1965, 1965, 700.0, 0x4, Not Active, Not Active, Not Active, Active\n")
    c = bench.ClockSampler(0, p)
    c.skip = 1
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"]
    c.skip = 2
    s = c.summary()
    assert s["samples"] == 1 and s["sm_mhz"] == 1965.0
    p.write_text("")
    assert bench.ClockSampler(0, p).summary()["reasons"] == ["unsampled"]
