"""Expert-parallel MoE on 2 GPUs (NCCL all-to-all): bit-identical to the single-GPU kernel.

A row's partial depends only on that row's operands (fixed K order inside the tensor core, per-token
activation shift), and both paths use the same combine, so the expert-parallel output of every rank
must equal moe_decode of the same tokens on one GPU bit for bit.  Needs >= 2 GPUs."""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

E_R, N_SH, H, I, T = 64, 2, 2048, 1408, 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, fixed, out):
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "qwen-mtp-mac_b200"))
    from qmtp import moe
    from qmtp.moe_ep import ExpertParallelMoE, local_expert_table

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        E = E_R + N_SH
        wts = []
        for shape in ((E, I, H), (E, I, H), (E, H, I)):
            w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            wts.extend(moe.quantize(w, mode))
            del w
        loc = local_expert_table(*wts, E_R, N_SH, rank, world)
        gt = torch.Generator(device=dev)
        gt.manual_seed(100 + rank)
        x = torch.randn((T, H), generator=gt, device=dev).to(torch.bfloat16)
        idx, sc = moe.route(torch.randn((T, E_R), generator=gt, device=dev), 6, N_SH)
        layer = ExpertParallelMoE(E_R, N_SH, lambda xr, e, out=None: moe.experts(xr, *loc, e, limit=None, mode=mode,
                                                                                 out=out),
                                  lambda tab, ro, s: moe.combine(tab, ro, s),
                                  capacity=(lambda T_, S_: T_ * S_) if fixed else None)
        y_ep = layer(x, idx, sc)
        y_one = moe.moe_decode(x, *wts, idx, sc, limit=None, mode=mode)
        torch.cuda.synchronize()
        out[rank] = (bool(torch.equal(y_ep.view(torch.int16), y_one.view(torch.int16))),
                     float((y_ep.float() - y_one.float()).abs().max()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fixed", [False, True], ids=["exact-splits", "fixed-capacity"])
@pytest.mark.parametrize("mode", ["mxfp4", "nvfp4"])
def test_expert_parallel_bit_identical_on_two_gpus(mode, fixed):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), mode, fixed, out), nprocs=world, start_method="spawn",
                       join=True)
    for r in range(world):
        same, diff = out[r]
        assert same, (r, diff)
