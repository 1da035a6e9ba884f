"""qmv with neighbouring decoder ops fused in (libqmtp qmtp_qmv_ex) against the oracle's separate ops,
bit-exact (GPU): RMSNorm -> qmv and SwiGLU -> qmv (prologues), qmv -> SwiGLU and qmv (+ residual) ->
RMSNorm (epilogues), and the L2 prefetch hint (no effect on results)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import ops
from tests._util import affine_layer, randn_bf16, rng, to_np, to_torch

pytestmark = pytest.mark.gpu


def _call(x_t, ldx, pre, pre_w_t, eps, wq, s, b, M, N, K, res_t=None, epi=0, norm=None, prefetch=()):
    """norm = (norm_w tensor, eps) for epi = NORM; returns y (and norm_y) as numpy."""
    from qmtp import _lib

    dev = x_t.device
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    W = [to_torch(a, dev) for a in (wq, s, b)]
    a = _lib.QmvArgs()
    a.x, a.ldx = x_t.data_ptr(), ldx
    a.w, a.scales, a.biases = W[0].data_ptr(), W[1].data_ptr(), W[2].data_ptr()
    a.y, a.res = y.data_ptr(), (res_t.data_ptr() if res_t is not None else None)
    a.M, a.N, a.K, a.ldy = M, N, K, N
    a.pre, a.pre_w, a.pre_eps = pre, (pre_w_t.data_ptr() if pre_w_t is not None else None), eps
    a.epi = epi
    keep = []
    if norm is not None:
        ny = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        sync = torch.zeros(4, dtype=torch.int32, device=dev)
        keep += [ny, sync]
        a.norm_y, a.norm_w, a.ld_norm, a.norm_eps = ny.data_ptr(), norm[0].data_ptr(), N, norm[1]
        a.sync = sync.data_ptr()
    for i, t in enumerate(prefetch):
        a.prefetch[i], a.prefetch_bytes[i] = t.data_ptr(), t.numel() * t.element_size()
    _lib.check(_lib.lib().qmtp_qmv_ex(ctypes.byref(a), _lib.stream()), "qmtp_qmv_ex")
    torch.cuda.synchronize()
    if norm is not None:
        assert int(keep[1][0]) == 0  # the arrival counter is left at 0 for the next call
        return to_np(y), to_np(keep[0])
    return to_np(y)


@pytest.mark.parametrize("K,N,M,pad", [(1024, 640, 3, 0), (4096, 1536, 3, 8), (4096, 256, 1, 0), (1024, 384, 6, 16)])
def test_rmsnorm_fused_bit_exact(K, N, M, pad, dev):
    _, wq, s, b = affine_layer(N, K, seed=K + N)
    ldx = K + pad
    xs = randn_bf16((M, ldx), 3, 2.0)
    w = ops.f32_to_bf16(1.0 + 0.2 * rng(4).standard_normal(K).astype(np.float32))
    eps = 1e-6
    xn = om.rmsnorm(np.ascontiguousarray(xs[:, :K]), w, eps)
    want = ops.qmv_affine(xn, wq, s, b)
    got = _call(to_torch(xs, dev), ldx, 1, to_torch(w, dev), eps, wq, s, b, M, N, K)
    assert np.array_equal(got, want)
    res = randn_bf16((M, N), 5)
    want_r = om.add(res, want)
    got_r = _call(to_torch(xs, dev), ldx, 1, to_torch(w, dev), eps, wq, s, b, M, N, K, res_t=to_torch(res, dev))
    assert np.array_equal(got_r, want_r)


@pytest.mark.parametrize("I,N,M", [(2048, 1024, 3), (12288, 512, 3), (2048, 256, 5)])
def test_swiglu_fused_bit_exact(I, N, M, dev):
    _, wq, s, b = affine_layer(N, I, seed=I + N)
    gu = randn_bf16((M, 2 * I), 6, 3.0)
    act = np.empty((M, I), np.uint16)
    ops.lib().qo_swiglu(gu.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(2 * I), ctypes.c_int(M), ctypes.c_int(I),
                        act.ctypes.data_as(ctypes.c_void_p))
    want = ops.qmv_affine(act, wq, s, b)
    got = _call(to_torch(gu, dev), 2 * I, 2, None, 0.0, wq, s, b, M, N, I)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("K,I,M", [(1024, 1536, 3), (4096, 3000, 3), (2048, 517, 1), (1024, 640, 6)])
def test_swiglu_epilogue_bit_exact(K, I, M, dev):
    """gate_up projection with the activation in its epilogue == qmv over [gate | up] then swiglu."""
    _, wq, s, b = affine_layer(2 * I, K, seed=K + I)
    x = randn_bf16((M, K), 7, 2.0)
    gu = ops.qmv_affine(x, wq, s, b)
    want = np.empty((M, I), np.uint16)
    ops.lib().qo_swiglu(gu.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(2 * I), ctypes.c_int(M), ctypes.c_int(I),
                        want.ctypes.data_as(ctypes.c_void_p))
    got = _call(to_torch(x, dev), K, 0, None, 0.0, wq, s, b, M, I, K, epi=1)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("K,N,M", [(4096, 4096, 3), (12288, 4096, 3), (2048, 2048, 1), (1024, 1024, 5)])
def test_norm_epilogue_bit_exact(K, N, M, dev):
    """residual projection whose last CTA applies the next RMSNorm == qmv_res then rmsnorm."""
    _, wq, s, b = affine_layer(N, K, seed=K + 3 * N)
    x = randn_bf16((M, K), 8, 1.0)
    res = randn_bf16((M, N), 9, 2.0)
    w = ops.f32_to_bf16(1.0 + 0.2 * rng(10).standard_normal(N).astype(np.float32))
    eps = 1e-6
    want_y = om.add(res, ops.qmv_affine(x, wq, s, b))
    want_n = om.rmsnorm(want_y, w, eps)
    for rep in range(2):  # the counter must be reusable
        got_y, got_n = _call(to_torch(x, dev), K, 0, None, 0.0, wq, s, b, M, N, K, res_t=to_torch(res, dev), epi=2,
                             norm=(to_torch(w, dev), eps))
        assert np.array_equal(got_y, want_y)
        assert np.array_equal(got_n, want_n)


def test_prefetch_hint_keeps_results(dev):
    K, N, M = 4096, 2048, 3
    _, wq, s, b = affine_layer(N, K, seed=11)
    x = randn_bf16((M, K), 12, 1.0)
    want = ops.qmv_affine(x, wq, s, b)
    nxt = [torch.empty(n, dtype=torch.uint8, device=dev) for n in (3 << 20, 12345 * 16 + 7, 64)]
    got = _call(to_torch(x, dev), K, 0, None, 0.0, wq, s, b, M, N, K, prefetch=nxt)
    assert np.array_equal(got, want)
