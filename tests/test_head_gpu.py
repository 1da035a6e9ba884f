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
