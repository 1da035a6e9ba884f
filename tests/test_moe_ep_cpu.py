"""Expert-parallel MoE host logic on CPU: 2 gloo ranks, oracle expert compute (no GPU).

Every rank routes its own tokens to routed experts on both ranks (all-to-all dispatch / combine) and
runs the shared experts locally; the result must equal the single-process oracle MoE of the same
tokens (experiments/deepseek_moe/kernels.py:35-107 restated) within the fp32 / bf16 tolerance."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E_R, N_SH, H, I, T, TOPK = 4, 2, 64, 64, 6, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer():
    from oracle import ops
    from tests._util import randn_bf16

    E = E_R + N_SH
    return [ops.quantize_fp4(randn_bf16(shape, seed, 0.05), "mxfp4")
            for seed, shape in ((1, (E, I, H)), (2, (E, I, H)), (3, (E, H, I)))]


def _tokens(rank):
    from oracle import ops
    from tests._util import randn_bf16, rng

    x = randn_bf16((T, H), 100 + rank)
    idx, sc = ops.moe_route(rng(200 + rank).standard_normal((T, E_R)).astype(np.float32), TOPK, N_SH, 1.0)
    return x, idx, sc


def _worker(rank, world, port, out, fixed):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qwen-mtp-mac_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle import ops
    from qmtp.moe_ep import ExpertParallelMoE

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    (wg, sg), (wu, su), (wd, sd) = _layer()
    per = E_R // world
    sel = list(range(rank * per, (rank + 1) * per)) + list(range(E_R, E_R + N_SH))
    loc = [a[sel] for a in (wg, sg, wu, su, wd, sd)]

    def compute(x_rows, ids, out=None):
        n = x_rows.shape[0]
        y = torch.zeros((n, H), dtype=torch.float32)
        keep = (ids >= 0).nonzero().reshape(-1)  # empty rows (id -1) of a fixed-capacity dispatch
        if len(keep):
            xb = x_rows[keep].numpy().view(np.uint16)
            _, yf = ops.moe(xb, *loc, ids[keep].numpy().reshape(-1, 1), np.ones((len(keep), 1), np.float32),
                            "mxfp4", None)
            y[keep] = torch.from_numpy(yf)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def combine(table, row_of, scores):
        tab = table.numpy()
        ro = row_of.numpy()
        sc = scores.numpy()
        y = np.zeros((ro.shape[0], H), np.float32)
        for j in range(ro.shape[1]):  # slot order, fp32 fused multiply-add as the kernel
            ok = ro[:, j] >= 0
            y[ok] = (sc[ok, j:j + 1].astype(np.float64) * tab[ro[ok, j]] + y[ok]).astype(np.float32)
        return torch.from_numpy(ops.f32_to_bf16(y).view(np.int16))

    x, idx, sc = _tokens(rank)
    from tests._moe_dispatch_ref import ref_dispatch
    layer = ExpertParallelMoE(E_R, N_SH, compute, combine, capacity=(lambda T_, S_: T_ * S_) if fixed else None,
                              dispatch=ref_dispatch)
    y = layer(torch.from_numpy(x.view(np.int16)), torch.from_numpy(idx), torch.from_numpy(sc))
    out[rank] = y.numpy().view(np.uint16).copy()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("fixed", [False, True], ids=["exact-splits", "fixed-capacity"])
def test_expert_parallel_matches_single_process(fixed):
    from oracle import ops

    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out, fixed), nprocs=world, start_method="spawn",
                       join=True)
    layer = _layer()
    for rank in range(world):
        x, idx, sc = _tokens(rank)
        _, ref = ops.moe(x, *[a for m in layer for a in m], idx, sc, "mxfp4", None)
        y = ops.bf16_to_f32(out[rank]).astype(np.float64)
        m = np.abs(ref).max()
        assert np.all(np.abs(y - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-5 * m), rank
