"""The TORCH_LIBRARY(cozy_kernels) extension ``libgwb200_torch.so``: the
reference loader's contract (``torch.ops.load_library`` of the file named by
GEN_WORKER_NATIVE_KERNELS_LIB, then ``build_info`` and the
``probe_add_one`` numerics probe, src/gen_worker/models/native_kernels.py:
96-143) and the quantized-linear ops it adds."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import native, ops
from gen_worker_b200.modules import build_svdq_int4_linear, fp8_rowwise_from_linear

REF_SRC = Path("/root/reference/src")


def test_extension_loads_and_registers_the_ops():
    ns = native.torch_ops()
    info = ns.build_info()
    assert info.startswith(f"torch={torch.__version__.split('+')[0]}") and "sm_100a" in info
    for name in ("probe_add_one", "svdq_w4a4_quant", "svdq_w4a4_gemm", "svdq_w4a4_linear",
                 "fp8_linear"):
        assert hasattr(ns, name), name
    schema = str(ns.svdq_w4a4_gemm.default._schema)
    assert "Tensor weight, Tensor weight_scale" in schema


@pytest.mark.skipif(not REF_SRC.exists(), reason="reference sources not present")
def test_reference_loader_accepts_the_extension():
    """The reference's own ``load_extension`` / ``extension_available``
    (run in a child process with the reference's sources on its path) load
    this library from GEN_WORKER_NATIVE_KERNELS_LIB and find the probe op."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from gen_worker.models import native_kernels as nk\n"
        "assert nk.load_extension() is None, nk.load_extension()\n"
        "print(nk.extension_ops().build_info())\n"
        "assert nk.extension_available()\n" % str(REF_SRC))
    env = dict(os.environ, GEN_WORKER_NATIVE_KERNELS_LIB=str(native.TORCH_LIB),
               CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", ""))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "sm_100a" in r.stdout


@pytest.mark.gpu
def test_probe_numerics_as_the_reference_checks(cuda_ready):
    ns = native.torch_ops()
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert torch.equal(ns.probe_add_one(x), x + 1)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,rank,gelu", [(300, 3072, 384, 32, False), (77, 1024, 256, 0, True)])
def test_linear_op_matches_module(cuda_ready, m, k, n, rank, gelu):
    ns = native.torch_ops()
    x = O.synth_activation(m, k, seed=m)
    L = O.synth_svdq_layer(k, n, rank, seed=m + 1, x_calib=x)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, gelu=gelu,
                                 device="cuda")
    xd = x.cuda()
    want = mod(xd)
    p = mod.prepare()
    got = ns.svdq_w4a4_linear(xd, mod.smooth_factor, p["proj_down_t"], mod.weight,
                              mod.weight_scale, p["proj_up_pad"], mod.bias.detach(), gelu)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert native.device_error() == 0


@pytest.mark.gpu
def test_fp8_linear_op_matches_module(cuda_ready):
    ns = native.torch_ops()
    lin = torch.nn.Linear(512, 256).cuda()
    mod = fp8_rowwise_from_linear(lin, gelu=True)
    x = O.synth_activation(64, 512, seed=3).cuda()
    got = ns.fp8_linear(x, mod.weight, mod.weight_scale.reshape(-1), mod.bias.detach(), True)
    assert torch.equal(got.view(torch.int16), mod(x).view(torch.int16))
