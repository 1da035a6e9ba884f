"""Oracle qmv against plain float64 math and its own invariants (CPU)."""
import numpy as np
import pytest

from oracle import ops
from tests._util import affine_layer, randn_bf16


def _rel(y_bits, ref):
    y = ops.bf16_to_f32(y_bits).astype(np.float64)
    return np.abs(y - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_qmv_affine_reference_test_shape(M):
    # tests/test_kernels.py:28-37 shape and criterion (N=1024, K=2048, W ~ N(0,1)/sqrt(K), < 1e-2)
    N, K = 1024, 2048
    w = ops.f32_to_bf16(np.random.default_rng(0).standard_normal((N, K), dtype=np.float32) / np.float32(K ** 0.5))
    wq, s, b = ops.quantize_affine(w)
    x = randn_bf16((M, K), 1)
    ref = ops.bf16_to_f32(x).astype(np.float64) @ ops.dequant_affine(wq, s, b).T
    assert _rel(ops.qmv_affine(x, wq, s, b), ref) < 1e-2


@pytest.mark.parametrize("M", [1, 4])
def test_qmv_affine_config1_tolerance(M):
    # config 1: W 12288x4096 ~ N(0,0.02), x ~ N(0,1); bf16 GEMV tolerance max rel err <= 2e-2
    _, wq, s, b = affine_layer(12288, 4096, seed=0)
    x = randn_bf16((M, 4096), 1)
    ref = ops.bf16_to_f32(x).astype(np.float64) @ ops.dequant_affine(wq, s, b).T
    assert _rel(ops.qmv_affine(x, wq, s, b), ref) < 2e-2


def test_qmv_affine_is_batch_invariant():
    _, wq, s, b = affine_layer(300, 4096, seed=3)
    x = randn_bf16((4, 4096), 4)
    full = ops.qmv_affine(x, wq, s, b)
    for m in range(4):
        assert np.array_equal(ops.qmv_affine(x[m:m + 1], wq, s, b)[0], full[m])


def test_quantize_affine_roundtrip():
    w, wq, s, b = affine_layer(64, 1024, seed=5)
    err = np.abs(ops.dequant_affine(wq, s, b) - ops.bf16_to_f32(w))
    sf = np.repeat(ops.bf16_to_f32(s), 64, axis=1)
    assert np.all(err <= sf * 0.5 + np.abs(ops.bf16_to_f32(w)) * 2 ** -7 + 1e-6)


def test_qmv_nvfp4_vs_float64():
    r = np.random.default_rng(7)
    N, K, M = 256, 2048, 3
    wq = r.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
    s = r.integers(118 - 64, 126 - 64 + 8, (N, K // 16), dtype=np.int64).astype(np.uint8)  # e4m3 ~ 2^-2..2^0
    x = randn_bf16((M, K), 8)
    e2m1, e4m3, _ = ops.decode_tables()
    q = np.empty((N, K), np.float64)
    for i in range(8):
        q[:, i::8] = e2m1[(wq >> (4 * i)) & 15]
    wd = q * np.repeat(e4m3[s].astype(np.float64), 16, axis=1)
    ref = ops.bf16_to_f32(x).astype(np.float64) @ wd.T
    assert _rel(ops.qmv_nvfp4(x, wq, s), ref) < 1e-2
