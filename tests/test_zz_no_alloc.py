"""gwb_svdq_w4a4_linear_noalloc against gwb_svdq_w4a4_linear.

The no-allocation entry point exists for callers that cannot allocate device
memory themselves (their memory is owned by another framework's pool or a
fixed start-up budget, or their serving loop forbids cudaMalloc once it is
running); it keeps the linear's intermediates in a fixed array inside the
library. Both entry points are called through the C ABI on the same inputs,
twice in a row with different inputs (the shared array keeps the previous
call's contents, which must not leak into the next result), and the outputs
must agree within the parity tolerance used for the oracle (here they are
expected to be identical: the kernels are the same).

This file is collected last on purpose: it runs after every other test, and
also passes when run alone in a fresh process."""
import pytest
import torch

from oracle import svdq_oracle as O
from gen_worker_b200 import native, ops

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _call(lib, name, *args):
    rc = getattr(lib, name)(*args)
    assert rc == 0, f"{name}: {native.status_string(rc)}"


def _layer(dev, k, n, rank, seed):
    x0 = O.synth_activation(64, k, seed=seed)
    L = O.synth_svdq_layer(k, n, rank, seed=seed + 1, x_calib=x0)
    p = ops.prepare_w4a4_weights(L["w_scale"].to(dev),
                                 None if rank == 0 else L["proj_down"].to(dev),
                                 None if rank == 0 else L["proj_up"].to(dev),
                                 weight=L["w_packed"].to(dev))
    return L, p


def _both(lib, dev, L, p, m, k, n, seed):
    """One call of each entry point on the same seeded input; returns both outputs."""
    stream = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    rp = 0 if p["proj_down_t"] is None else int(p["proj_down_t"].shape[0])
    x = O.synth_activation(m, k, seed=seed).to(dev)
    smooth, bias = L["smooth"].to(dev), L["bias"].to(dev)
    codes = torch.empty(m, k, dtype=torch.uint8, device=dev)
    ascale = torch.empty(k // 64, m, 8, dtype=torch.float16, device=dev)
    la = torch.empty(m, max(rp, 1), dtype=torch.bfloat16, device=dev)
    y_ref = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    y_na = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    _call(lib, "gwb_svdq_w4a4_linear", x.data_ptr(), smooth.data_ptr(), ptr(p["proj_down_t"]),
          p["w_q8"].data_ptr(), p["w_scale_k8"].data_ptr(), ptr(p["proj_up_pad"]),
          bias.data_ptr(), m, n, k, rp, 0, codes.data_ptr(), ascale.data_ptr(),
          la.data_ptr() if rp else None, y_ref.data_ptr(), stream)
    _call(lib, "gwb_svdq_w4a4_linear_noalloc", x.data_ptr(), smooth.data_ptr(),
          ptr(p["proj_down_t"]), p["w_q8"].data_ptr(), p["w_scale_k8"].data_ptr(),
          ptr(p["proj_up_pad"]), bias.data_ptr(), m, n, k, rp, 0, y_na.data_ptr(), stream)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    return y_ref.cpu(), y_na.cpu()


@pytest.mark.parametrize("m,k,n,rank", [(300, 3072, 384, 32), (128, 1024, 256, 0)])
def test_noalloc_linear_matches_allocating_entry_point(cuda_ready, m, k, n, rank):
    lib = native.require()
    dev = torch.device("cuda", 0)
    L, p = _layer(dev, k, n, rank, seed=41)
    for seed in (43, 44):   # two calls in a row, different inputs
        y_ref, y_na = _both(lib, dev, L, p, m, k, n, seed)
        assert not torch.isnan(y_na.float()).any()
        assert O.rel_l2(y_na, y_ref) <= REL_TOL


def test_noalloc_shrinking_calls_do_not_see_stale_scratch(cuda_ready):
    """A large call (rank 32) leaves its intermediates in the shared array;
    the smaller calls after it (rank 0, then rank 16) must not pick any of
    them up."""
    lib = native.require()
    dev = torch.device("cuda", 0)
    k, n = 1024, 256
    for m, rank, seed in ((2000, 32, 51), (96, 0, 52), (200, 16, 53)):
        L, p = _layer(dev, k, n, rank, seed=seed)
        y_ref, y_na = _both(lib, dev, L, p, m, k, n, seed + 100)
        assert not torch.isnan(y_na.float()).any()
        assert O.rel_l2(y_na, y_ref) <= REL_TOL


def test_noalloc_rejects_requests_beyond_its_capacity(cuda_ready):
    lib = native.require()
    # 20000 x 3072 needs 20000*(3072+768+64) bytes > 32 MiB -> GWB_E_CAPACITY (8),
    # refused before any pointer is touched
    rc = lib.gwb_svdq_w4a4_linear_noalloc(None, None, None, None, None, None, None,
                                          20000, 3072, 3072, 32, 0, None, None)
    assert rc == 8, native.status_string(rc)
