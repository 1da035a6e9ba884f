"""Oracle two-stage head (CPU): lm_head2.py's contract and tests/test_kernels.py:116-126."""
import numpy as np

from oracle import ops
from tests._util import randn_bf16


def test_two_stage_head_reference_test_shape():
    # tests/test_kernels.py:116-126: V=16384, D=512 -> this oracle needs D % 1024 == 0 for the coarse
    # qmv, so D = 1024 here; 64 rows, k = 64; candidate logits bit-equal to the full bf16 matmul
    # in this build's dot order; argmax agreement >= 98 %.
    V, D, M = 16384, 1024, 64
    W = ops.f32_to_bf16(np.random.default_rng(5).standard_normal((V, D), dtype=np.float32) / np.float32(D ** 0.5))
    h = randn_bf16((M, D), 6)
    wq, s, b = ops.quantize_affine(W)
    coarse, idx, fine, amax = ops.two_stage_head(h, wq, s, b, W, 64)
    assert idx.shape == (M, 64) and all(len(set(r)) == 64 for r in idx.tolist())
    full_amax = np.empty(M, np.int32)
    Wf = ops.bf16_to_f32(W).astype(np.float64)
    hf = ops.bf16_to_f32(h).astype(np.float64)
    for m in range(M):
        for j in (0, 17, 63):
            exact = float(Wf[idx[m, j]] @ hf[m])
            assert fine[m, j] == ops.f32_to_bf16(np.float32([ops.dot_bf16(W[idx[m, j]], h[m])]))[0]
            assert abs(float(ops.bf16_to_f32(fine[m, j:j + 1])[0]) - exact) <= 2 ** -8 * abs(exact) + 1e-6
        full_bf16 = ops.f32_to_bf16((Wf @ hf[m]).astype(np.float32))  # the full bf16 matmul's logits
        full_amax[m] = int(ops.argmax_bf16(full_bf16[None])[0])
    assert (amax == full_amax).mean() >= 0.98


def test_topk_order_and_ties():
    vals = ops.f32_to_bf16(np.float32([[1.0, 3.0, 3.0, -2.0, 3.0, 0.5, np.inf, -np.inf]]))
    assert ops.topk_bf16(vals, 4).tolist() == [[6, 1, 2, 4]]
    assert ops.argmax_bf16(vals).tolist() == [6]
    same = ops.f32_to_bf16(np.float32([[2.0] * 10]))
    assert ops.topk_bf16(same, 3).tolist() == [[0, 1, 2]]
