"""Vocabulary-sharded two-stage head on 2 GPUs over NCCL (GPU; skipped with fewer than 2 devices).

Each rank holds half of the vocabulary rows (bf16 weight and 4-bit coarse copy); ShardedTwoStageHead
all-gathers the shards' candidate lists and merges them.  Both ranks must return exactly what the
single-GPU TwoStageHead returns on the whole vocabulary (config 3: V = 248320, D = 4096, M = 3)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qwen-mtp-mac_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    import torch.distributed as dist

    from qmtp.lm_head2 import ShardedTwoStageHead, TwoStageHead
    from qmtp.qmv_kernel import QuantizedLinear, quantize

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    V, D, M = 248320, 4096, 3
    W = (torch.randn(V, D, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    h = torch.randn(M, D, generator=g, device=dev).to(torch.bfloat16)
    W[5] = W[V - 3] = (h[0].float() * 0.05).to(torch.bfloat16)  # a tie across the two shards
    coarse = QuantizedLinear(*quantize(W))
    whole = TwoStageHead(W, 64, coarse)
    ref = [t.cpu() for t in whole.select(h)]
    sharded = ShardedTwoStageHead.from_full(W, 64, coarse=coarse)
    for _ in range(2):
        got = [t.cpu() for t in sharded.select(h)]
    torch.cuda.synchronize()
    out[rank] = (all(torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                                 b.view(torch.int16) if b.dtype == torch.bfloat16 else b) for a, b in zip(ref, got)),
                 int(ref[0][0, 0]), int(ref[0][0, 1]), sharded.v0)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_head_equals_single_gpu_head():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    for rank in range(world):
        same, first, second, v0 = out[rank]
        assert same, rank
        assert (first, second) == (5, 248317)
    assert out[1][3] == 124160
