"""Two-stage head kernels (libqmtp) against the oracle: index sets, order and logits bit-exact (GPU)."""
import numpy as np
import pytest
import torch

from oracle import ops
from tests._util import randn_bf16, to_np, to_torch

pytestmark = pytest.mark.gpu


def _head(V, D, seed, dev):
    from qmtp.lm_head2 import TwoStageHead
    from qmtp.qmv_kernel import QuantizedLinear

    W = randn_bf16((V, D), seed, 0.02)
    wq, s, b = ops.quantize_affine(W)
    head = TwoStageHead(to_torch(W, dev), 64, QuantizedLinear(to_torch(wq, dev), to_torch(s, dev), to_torch(b, dev)))
    return head, W, wq, s, b


@pytest.mark.parametrize("V,D,M", [(16384, 1024, 64), (248320, 4096, 3), (50000, 4096, 1), (1000, 2048, 2)])
def test_two_stage_head_bit_exact(V, D, M, dev):
    head, W, wq, s, b = _head(V, D, V + D, dev)
    h = randn_bf16((M, D), 7)
    idx, fine, amax = head.select(to_torch(h, dev))
    _, ridx, rfine, ramax = ops.two_stage_head(h, wq, s, b, W, 64)
    assert np.array_equal(to_np(idx).view(np.int32), ridx)
    assert np.array_equal(to_np(fine), rfine)
    assert np.array_equal(to_np(amax).view(np.int32), ramax)


def test_reference_call_contract(dev):
    head, W, wq, s, b = _head(16384, 1024, 3, dev)
    h = randn_bf16((1, 2, 1024), 8)
    logits = head(to_torch(h, dev))
    assert logits.shape == (1, 2, 16384)
    fin = torch.isfinite(logits.float())
    assert (fin.sum(-1) == 64).all()
    _, ridx, rfine, _ = ops.two_stage_head(h.reshape(2, 1024), wq, s, b, W, 64)
    got = to_np(logits.reshape(2, -1))
    for m in range(2):
        assert np.array_equal(got[m, ridx[m]], rfine[m])


def test_argmax_and_ties(dev):
    from qmtp.lm_head2 import argmax

    r = np.random.default_rng(9)
    vals = ops.f32_to_bf16(r.standard_normal((3, 248320)).astype(np.float32))
    vals[1, 1000] = vals[1, 7] = ops.f32_to_bf16(np.float32([50.0]))[0]
    got = to_np(argmax(to_torch(vals, dev))).view(np.int32)
    assert np.array_equal(got, ops.argmax_bf16(vals)) and got[1] == 7


def test_topk_many_ties(dev):
    """A row of equal values: the lowest indices win (index-set bit-exact)."""
    from qmtp import _lib

    vals = np.full((2, 30000), ops.f32_to_bf16(np.float32([1.5]))[0], np.uint16)
    vals[1, 29999] = ops.f32_to_bf16(np.float32([2.0]))[0]
    v = to_torch(vals, dev)
    k = 64
    idx = torch.empty((2, k), dtype=torch.int32, device=dev)
    ws = torch.empty(_lib.lib().qmtp_topk_workspace(2, 30000, k), dtype=torch.uint8, device=dev)
    _lib.check(_lib.lib().qmtp_topk_rescore(v.data_ptr(), 30000, 2, 30000, k, None, None, 0, idx.data_ptr(), None,
                                            None, ws.data_ptr(), ws.numel(), _lib.stream()), "topk")
    assert np.array_equal(to_np(idx).view(np.int32), ops.topk_bf16(vals, k))


@pytest.mark.parametrize("G,V,M,k", [(2, 248320, 3, 64), (3, 248320, 1, 64), (8, 248320, 3, 64), (5, 50000, 2, 256),
                                     (4, 1000, 3, 64)])
def test_vocab_shards_merge_to_the_whole_head(G, V, M, k, dev):
    """qmtp_lmhead2_shard on G vocabulary shards (run here one after another on one GPU) and
    qmtp_lmhead2_merge of their lists give qmtp_lmhead2's result on the whole vocabulary bit for bit,
    including ties across shard boundaries."""
    from qmtp import _lib
    from qmtp.lm_head2 import ShardedTwoStageHead

    D = 4096 if V > 10000 else 1024
    W = randn_bf16((V, D), V + G, 0.02)
    h = randn_bf16((M, D), 3)
    hf = ops.bf16_to_f32(h)
    bounds = [ShardedTwoStageHead.split(V, G, r) for r in range(G)]
    for m in range(M):  # a tied pair straddling a boundary, ranked first for token m
        a, c = bounds[0][1] - 1 - m, bounds[-1][0] + m
        W[a] = W[c] = ops.f32_to_bf16(0.05 * hf[m])
    wq, s, b = ops.quantize_affine(W)
    Wt, wqt, st, bt, ht = (to_torch(x, dev) for x in (W, wq, s, b, h))
    L = _lib.lib()
    words = torch.empty((G, M, k), dtype=torch.int64, device=dev)
    fine = torch.empty((G, M, k), dtype=torch.bfloat16, device=dev)
    for r, (v0, vs) in enumerate(bounds):
        ws = torch.empty(L.qmtp_lmhead2_shard_workspace(M, vs, k), dtype=torch.uint8, device=dev)
        _lib.check(L.qmtp_lmhead2_shard(ht.data_ptr(), wqt[v0:].data_ptr(), st[v0:].data_ptr(), bt[v0:].data_ptr(),
                                        Wt[v0:].data_ptr(), M, vs, D, k, v0, words[r].data_ptr(), fine[r].data_ptr(),
                                        ws.data_ptr(), ws.numel(), _lib.stream()), "shard")
    idx = torch.empty((M, k), dtype=torch.int32, device=dev)
    fv = torch.empty((M, k), dtype=torch.bfloat16, device=dev)
    amax = torch.empty((M,), dtype=torch.int32, device=dev)
    _lib.check(L.qmtp_lmhead2_merge(words.data_ptr(), fine.data_ptr(), G, M, k, idx.data_ptr(), fv.data_ptr(),
                                    amax.data_ptr(), _lib.stream()), "merge")
    _, ridx, rfine, ramax = ops.two_stage_head(h, wq, s, b, W, k)
    assert all(ridx[m, 0] == bounds[0][1] - 1 - m and ridx[m, 1] == bounds[-1][0] + m for m in range(M))
    assert np.array_equal(to_np(idx).view(np.int32), ridx)
    assert np.array_equal(to_np(fv), rfine)
    assert np.array_equal(to_np(amax).view(np.int32), ramax)


@pytest.mark.parametrize("V,D,M,k", [(248320, 4096, 3, 64), (50000, 4096, 1, 256), (4096, 1024, 2, 64)])
def test_two_stage_head_nvfp4_coarse_bit_exact(V, D, M, k, dev):
    """The reference's own head format (lm_head2.py:19, NVFP4 g16 coarse copy): index sets, order,
    exact logits and argmax bit-exact against the oracle; the coarse copy built on the GPU from the
    bf16 weight equals the oracle's quantizer."""
    from qmtp.lm_head2 import TwoStageHead
    from qmtp.qmv_kernel import QuantizedLinear

    W = randn_bf16((V, D), V + 3, 0.02)
    h = randn_bf16((M, D), 11)
    nq, ns = ops.quantize_fp4(W, "nvfp4")
    head = TwoStageHead(to_torch(W, dev), k, QuantizedLinear(to_torch(nq, dev), to_torch(ns, dev), None,
                                                             group_size=16, mode="nvfp4"))
    idx, fine, amax = head.select(to_torch(h, dev))
    _, ridx, rfine, ramax = ops.two_stage_head_nvfp4(h, nq, ns, W, k)
    assert np.array_equal(to_np(idx).view(np.int32), ridx)
    assert np.array_equal(to_np(fine), rfine)
    assert np.array_equal(to_np(amax).view(np.int32), ramax)
    if V == 4096:
        built = TwoStageHead(to_torch(W, dev), k, mode="nvfp4")
        assert np.array_equal(to_np(built.coarse.weight).view(np.uint32), nq.view(np.uint32))
        assert np.array_equal(to_np(built.coarse.scales), ns)
        got = [to_np(t) for t in built.select(to_torch(h, dev))]
        assert np.array_equal(got[0].view(np.int32), ridx)


@pytest.mark.parametrize("k,M", [(512, 3), (2048, 3), (1000, 1)])
def test_two_stage_head_large_k_bit_exact(k, M, dev):
    """Candidate sets above 256 (k_for up to 2048, lm_head2.py:32-36): the radix-select path gives the
    oracle's index set, order, exact logits and argmax at V = 248320, ties included."""
    W2 = randn_bf16((248320, 4096), 5, 0.02)
    h = randn_bf16((M, 4096), 13)
    hf = ops.bf16_to_f32(h)
    W2[7] = W2[200000] = ops.f32_to_bf16(0.05 * hf[0])  # a tied pair ranked first for token 0
    wq2, s2, b2 = ops.quantize_affine(W2)
    from qmtp.lm_head2 import TwoStageHead
    from qmtp.qmv_kernel import QuantizedLinear

    head = TwoStageHead(to_torch(W2, dev), 64, QuantizedLinear(to_torch(wq2, dev), to_torch(s2, dev), to_torch(b2, dev)))
    idx, fine, amax = head.select(to_torch(h, dev), k=k)
    _, ridx, rfine, ramax = ops.two_stage_head(h, wq2, s2, b2, W2, k)
    assert ridx[0, 0] == 7 and ridx[0, 1] == 200000
    assert np.array_equal(to_np(idx).view(np.int32), ridx)
    assert np.array_equal(to_np(fine), rfine)
    assert np.array_equal(to_np(amax).view(np.int32), ramax)
