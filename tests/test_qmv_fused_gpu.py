"""qmv with the producer of x fused into its load (libqmtp qmtp_qmv_affine_g64_ex) against the
oracle's separate ops: RMSNorm -> qmv and SwiGLU -> qmv, bit-exact (GPU)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import ops
from tests._util import affine_layer, randn_bf16, rng, to_np, to_torch

pytestmark = pytest.mark.gpu


def _call(x_t, ldx, pre, pre_w_t, eps, wq, s, b, M, N, K, res_t=None):
    from qmtp import _lib

    dev = x_t.device
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    W = [to_torch(a, dev) for a in (wq, s, b)]
    rc = _lib.lib().qmtp_qmv_affine_g64_ex(x_t.data_ptr(), ldx, pre, pre_w_t.data_ptr() if pre_w_t is not None else None,
                                           eps, W[0].data_ptr(), W[1].data_ptr(), W[2].data_ptr(), y.data_ptr(),
                                           res_t.data_ptr() if res_t is not None else None, M, N, K, N, _lib.stream())
    _lib.check(rc, "qmtp_qmv_affine_g64_ex")
    torch.cuda.synchronize()
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
