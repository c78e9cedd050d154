"""Token (M) sharding on 2 gloo ranks (CPU): each rank quantises and runs the
two-branch forward of its own row shard with replicated weights; the
all-gathered result equals the unsharded one bit for bit, because INT4
group scales are per row (shard-invariant, unlike the per-tensor scale that
``parallel/cp.py:285-302`` refuses)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import svdq_oracle as O

M, K, N, R = 64, 256, 128, 32


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    x = O.synth_activation(M, K, seed=11)
    L = O.synth_svdq_layer(K, N, R, seed=12, x_calib=x)
    return x, L


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, L = _case()
    m = M // world
    y = O.svdq_int4_linear(x[rank * m:(rank + 1) * m], L["smooth"], L["w_packed"], L["w_scale"],
                           L["proj_down"], L["proj_up"], L["bias"])["y"]
    yf = y.float().contiguous()            # bf16 -> f32 is exact; gloo has no bf16
    parts = [torch.empty_like(yf) for _ in range(world)]
    dist.all_gather(parts, yf)
    if rank == 0:
        q.put(torch.cat(parts).to(torch.bfloat16))
    dist.barrier()
    dist.destroy_process_group()


def test_token_sharded_forward_is_bit_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, L = _case()
    want = O.svdq_int4_linear(x, L["smooth"], L["w_packed"], L["w_scale"], L["proj_down"],
                              L["proj_up"], L["bias"])["y"]
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
