"""Vocabulary-sharded two-stage head, host logic on CPU: 2 and 3 gloo ranks with the C oracle as the
per-shard head (no GPU).

Each rank runs the oracle head on its rows of the vocabulary and turns its best k into candidate
words with global indices; ShardedTwoStageHead all-gathers the words and fine logits and merges them.
Every rank must end with exactly the oracle's single-device result (lm_head2.py:111-117 restated):
the same k indices in the same order, the same fine logits, the same argmax."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

V, D, M, K = 3001, 512, 3, 64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights():
    from oracle import ops
    from tests._util import randn_bf16

    W = randn_bf16((V, D), 5, 0.02)
    h = randn_bf16((M, D), 6)
    # equal rows on both sides of the shard boundaries, aligned with a token so that they rank first
    # for it (ties are broken by the lower global index)
    hf = ops.bf16_to_f32(h)
    for m, (a, c) in enumerate(((10, 2999), (1499, 1501), (1000, 2001))):
        W[a] = W[c] = ops.f32_to_bf16(0.05 * hf[m])
    wq, s, b = ops.quantize_affine(W)
    return W, wq, s, b, h


def key16(b):
    b = b.astype(np.uint64)
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)


def words_of(coarse_vals, gidx):
    return ((key16(coarse_vals) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - gidx.astype(np.uint64))).view(np.int64)


def merge_ref(words, fine, k):
    """CPU stand-in for qmtp_lmhead2_merge: per row the k largest words (unsigned) in order."""
    G, Mr, _ = words.shape
    w = words.numpy().view(np.uint64)
    f = fine.view(torch.int16).numpy().view(np.uint16)
    idx = np.empty((Mr, k), np.int32)
    fv = np.empty((Mr, k), np.uint16)
    amax = np.empty(Mr, np.int32)
    for m in range(Mr):
        flat = w[:, m, :].reshape(-1)
        ff = f[:, m, :].reshape(-1)
        order = sorted(range(flat.size), key=lambda i: int(flat[i]), reverse=True)[:k]
        gi = (np.uint64(0xFFFFFFFF) - (flat[order] & np.uint64(0xFFFFFFFF))).astype(np.int64)
        idx[m] = gi
        fv[m] = ff[order]
        fw = [(int(key16(np.array([fv[m, j]]))[0]) << 32) | (0xFFFFFFFF - int(gi[j])) for j in range(k)]
        amax[m] = 0xFFFFFFFF - (max(fw) & 0xFFFFFFFF)
    return torch.from_numpy(idx), torch.from_numpy(fv.view(np.int16)).view(torch.bfloat16), torch.from_numpy(amax)


def _worker(rank, world, port, out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "qwen-mtp-mac_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle import ops
    from qmtp.lm_head2 import ShardedTwoStageHead

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    W, wq, s, b, h = _weights()
    v0, vs = ShardedTwoStageHead.split(V, world, rank)
    Ws, wqs, ss, bs = W[v0:v0 + vs], wq[v0:v0 + vs], s[v0:v0 + vs], b[v0:v0 + vs]

    def local(h2, k):
        hb = h2.numpy().view(np.uint16)
        coarse = ops.qmv_affine(hb, wqs, ss, bs)
        li = ops.topk_bf16(coarse, k)
        fine, _ = ops.rescore_bf16(Ws, hb, li)
        cv = np.take_along_axis(coarse, li, axis=1)
        return torch.from_numpy(words_of(cv, li + v0)), torch.from_numpy(fine.view(np.int16)).view(torch.bfloat16)

    head = ShardedTwoStageHead(None, v0, V, K, local=local, merge=merge_ref)
    idx, fine, amax = head.select(torch.from_numpy(h.view(np.int16)))
    out[rank] = (idx.numpy().copy(), fine.view(torch.int16).numpy().view(np.uint16).copy(), amax.numpy().copy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_head_matches_single_device(world):
    from oracle import ops

    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    W, wq, s, b, h = _weights()
    _, ridx, rfine, ramax = ops.two_stage_head(h, wq, s, b, W, K)
    assert [tuple(ridx[m, :2]) for m in range(M)] == [(10, 2999), (1499, 1501), (1000, 2001)]
    for rank in range(world):
        idx, fine, amax = out[rank]
        assert np.array_equal(idx, ridx), rank
        assert np.array_equal(fine, rfine), rank
        assert np.array_equal(amax, ramax), rank


def test_split_covers_the_vocabulary():
    from qmtp.lm_head2 import ShardedTwoStageHead

    for Vt, G in ((248320, 8), (3001, 3), (10, 4), (7, 7)):
        parts = [ShardedTwoStageHead.split(Vt, G, r) for r in range(G)]
        assert parts[0][0] == 0 and sum(p[1] for p in parts) == Vt
        assert all(parts[r][0] + parts[r][1] == parts[r + 1][0] for r in range(G - 1))
        assert max(p[1] for p in parts) - min(p[1] for p in parts) <= 1
