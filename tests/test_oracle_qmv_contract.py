"""The C oracle's affine qmv against an independent restatement of the same arithmetic contract in
pure Python: exact integer group sums, float32 roundings done with exact rationals (CPU).

Contract (oracle/qmtp_oracle.c qo_qmv_affine): per token and group of 64, x_q = RNE(x * 2^(19-E)) with
E = floor(log2 max|x|); per row, S_g = sum q * x_q exactly; per 512-k slice two chains of four groups
H = fma(float(S_g), s_g * 2^(E-19), H); H = fma(b_g, float(sum x_q) * 2^(E-19), H); slices added in
order; bf16 output."""
import math
from fractions import Fraction

import numpy as np
import pytest

from oracle import ops
from tests._util import affine_layer, randn_bf16


def f32_round(fr: Fraction) -> float:
    """Nearest float32 to an exact rational (ties to even, subnormals, overflow to inf)."""
    if fr == 0:
        return 0.0
    sign = -1.0 if fr < 0 else 1.0
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    e = max(e, -126)
    quantum = Fraction(2) ** (e - 23)
    q = a / quantum
    n = math.floor(q)
    rem = q - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
        n += 1
    v = n * quantum
    if v > Fraction(2 - 2 ** -23) * Fraction(2) ** 127:
        return sign * math.inf
    return sign * float(v)


def fma32(a: float, b: float, c: float) -> float:
    return f32_round(Fraction(a) * Fraction(b) + Fraction(c))


def f32(v) -> float:
    return float(np.float32(v))


def grid(x_bits: np.ndarray):
    """x_q (exact ints) and the per-group factors c, xf of one token row."""
    K = x_bits.size
    xq = np.zeros(K, dtype=np.int64)
    cs, xfs = [], []
    vals = ops.bf16_to_f32(x_bits).astype(np.float64)
    for g in range(K // 64):
        v = vals[64 * g:64 * g + 64]
        amax = np.abs(v).max()
        if amax == 0:
            cs.append(0.0)
            xfs.append(0.0)
            continue
        E = math.floor(math.log2(amax))
        for e in range(64):
            t = Fraction(v[e]) * Fraction(2) ** (19 - E)
            n = math.floor(t)
            rem = t - n
            if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
                n += 1
            xq[64 * g + e] = n
        c = 2.0 ** (E - 19) if E - 19 >= -149 else 0.0
        cs.append(f32(c))
        xfs.append(f32(np.float32(float(xq[64 * g:64 * g + 64].sum())) * np.float32(c)))
    return xq, cs, xfs


def qmv_contract(x, wq, s, b):
    M, K = x.shape
    N = wq.shape[0]
    q = np.zeros((N, K), dtype=np.int64)
    for i in range(8):
        q[:, i::8] = (wq >> (4 * i)) & 15
    sf, bf = ops.bf16_to_f32(s), ops.bf16_to_f32(b)
    out = np.zeros((M, N), dtype=np.float32)
    for m in range(M):
        xq, cs, xfs = grid(x[m])
        for n in range(N):
            y = 0.0
            for sl in range(K // 512):
                H = [0.0, 0.0]
                for h in range(2):
                    for gi in range(4):
                        g = 8 * sl + 4 * h + gi
                        S = int((q[n, 64 * g:64 * g + 64] * xq[64 * g:64 * g + 64]).sum())
                        assert abs(S) < 2 ** 31
                        t = f32(S)
                        H[h] = fma32(t, f32(np.float32(sf[n, g]) * np.float32(cs[g])), H[h])
                        H[h] = fma32(float(bf[n, g]), xfs[g], H[h])
                P = f32(np.float32(H[0]) + np.float32(H[1]))
                y = P if sl == 0 else f32(np.float32(y) + np.float32(P))
            out[m, n] = y
    return ops.f32_to_bf16(out)


@pytest.mark.parametrize("M,N,K,seed", [(2, 6, 1024, 0), (1, 4, 512, 1), (3, 3, 1536, 2)])
def test_oracle_follows_the_contract(M, N, K, seed):
    _, wq, s, b = affine_layer(N, K, seed=seed)
    x = randn_bf16((M, K), seed + 10)
    assert np.array_equal(ops.qmv_affine(x, wq, s, b), qmv_contract(x, wq, s, b))


def test_oracle_follows_the_contract_on_wide_ranges():
    """Groups mixing magnitudes 2^-20 .. 2^20, all-zero groups and subnormal-only groups."""
    r = np.random.default_rng(9)
    M, N, K = 2, 3, 512
    _, wq, s, b = affine_layer(N, K, seed=4)
    mag = r.uniform(-20, 20, (M, K))
    x = ops.f32_to_bf16((np.sign(r.standard_normal((M, K))) * 2.0 ** mag).astype(np.float32))
    x[0, 64:128] = 0
    x[1, 128:192] = r.integers(1, 128, 64).astype(np.uint16) | (r.integers(0, 2, 64).astype(np.uint16) << 15)
    assert np.array_equal(ops.qmv_affine(x, wq, s, b), qmv_contract(x, wq, s, b))


def test_nonfinite_group_makes_the_row_nan():
    _, wq, s, b = affine_layer(5, 1024, seed=6)
    x = randn_bf16((2, 1024), 7)
    x[1, 300] = 0x7F80  # +inf
    y = ops.bf16_to_f32(ops.qmv_affine(x, wq, s, b))
    assert np.isfinite(y[0]).all() and np.isnan(y[1]).all()
