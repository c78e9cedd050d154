"""Failure detection without a GPU fault: a device wait that runs out.

Every pipeline wait in the kernels is bounded (the counterpart of the
reference's collective timeout and stall detection,
src/gen_worker/parallel/group.py:26, :265-285). Here a kernel waits on an
mbarrier that nothing ever arrives on — a flag that nothing sets — with a
short wait limit: the wait must give up, record its code in the device
error flag, free its TMEM and return; the host reads the code, and the next
normal launch must succeed and match the oracle. Nothing faults, traps or
hangs."""
import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import native
from gen_worker_b200.modules import build_svdq_int4_linear

pytestmark = pytest.mark.gpu

GWB_ERR_TIMEOUT_MMA = 2
GWB_ERR_TIMEOUT_EPILOGUE = 3


def _stall(lib, code: int) -> int:
    stream = torch.cuda.current_stream().cuda_stream
    assert native.device_error() == 0
    assert lib.gwb_set_wait_limit(200_000) == 0       # ~0.1 ms of SM clock
    try:
        assert lib.gwb_test_stalled_wait(code, stream) == 0
        return native.device_error()                  # synchronises, reads and clears
    finally:
        assert lib.gwb_set_wait_limit(0) == 0         # back to the default limit


def test_bounded_wait_runs_out_and_the_context_stays_usable(cuda_ready):
    lib = native.require()
    # twice in a row: each run must have freed its TMEM for the next to allocate
    assert _stall(lib, GWB_ERR_TIMEOUT_MMA) == GWB_ERR_TIMEOUT_MMA
    assert _stall(lib, GWB_ERR_TIMEOUT_EPILOGUE) == GWB_ERR_TIMEOUT_EPILOGUE
    assert native.device_error() == 0                 # the flag was cleared
    # the next normal launches (quantiser + 512-column TMEM GEMM) run and match
    m, k, n = 256, 3072, 384
    x = O.synth_activation(m, k, seed=71)
    L = O.synth_svdq_layer(k, n, 32, seed=72, x_calib=x)
    mod = build_svdq_int4_linear({"weight": L["w_packed"], "weight_scale": L["w_scale"],
                                  "smooth_factor": L["smooth"], "proj_down": L["proj_down"],
                                  "proj_up": L["proj_up"], "bias": L["bias"]}, device="cuda")
    y = mod(x.cuda()).cpu()
    want = O.svdq_int4_linear(x, L["smooth"], L["w_packed"], L["w_scale"], L["proj_down"],
                              L["proj_up"], L["bias"])
    assert O.rel_l2(y, want["y"]) <= 1e-3
    assert O.max_abs_beyond_bf16(y, want["y64"]) <= 2e-2
    assert native.device_error() == 0


def test_wait_limit_entry_rejects_nothing_on_cpu_side(cuda_ready):
    """gwb_set_wait_limit(0) restores the default; a code <= 0 is refused
    before any launch."""
    lib = native.require()
    assert lib.gwb_set_wait_limit(0) == 0
    assert lib.gwb_test_stalled_wait(0, None) == 1
