"""4-bit format decoders of the oracle pinned against the reference's own bit tricks (CPU).

qmv_kernel.py:16-29 (deq8, e4m3_scale) and experiments/deepseek_moe/kernels.py:13-32 (dot8,
e8m0_scale) decode with half-precision bit manipulation and fold 2^14 into the scale; they are
re-executed here in numpy and must agree with the oracle's tables exactly.
"""
import numpy as np

from oracle import ops


def _ref_e2m1_times_2m14(nib):
    w = np.uint32(nib)
    bits = ((w & 0x00070007) << 9) | ((w & 0x00080008) << 12)
    return np.array([bits & 0xFFFF], dtype=np.uint16).view(np.float16).astype(np.float32)[0]


def test_e2m1_matches_reference_half_trick():
    e2m1, _, _ = ops.decode_tables()
    for n in range(16):
        assert np.float32(_ref_e2m1_times_2m14(n)) * np.float32(16384.0) == e2m1[n], n
    assert e2m1[:8].tolist() == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def test_e4m3_matches_reference_scale():
    _, e4m3, _ = ops.decode_tables()
    for s in range(256):
        half = np.array([(s & 0x7F) << 7], dtype=np.uint16).view(np.float16).astype(np.float32)[0]
        ref = half * np.float32(4194304.0) / np.float32(16384.0)  # reference folds 2^14 in
        assert ref == e4m3[s], s
    assert e4m3[0x7E] == 448.0


def test_e8m0_matches_reference_scale():
    _, _, e8m0 = ops.decode_tables()
    for s in range(1, 241):
        ref = np.array([(s + 14) << 23], dtype=np.uint32).view(np.float32)[0] / np.float32(16384.0)
        assert ref == e8m0[s], s
