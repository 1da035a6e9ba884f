"""Oracle exp/log and the bf16 activation formulas of gdn_fused.py:22-41 (CPU)."""
import numpy as np

from oracle import ops


def _ulp_diff(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def test_exp_within_1ulp_of_libm():
    r = np.random.default_rng(0)
    x = np.concatenate([r.standard_normal(400_000).astype(np.float32) * 30,
                        np.linspace(-87.0, 88.7, 200_001, dtype=np.float32),
                        np.float32([0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30])])
    got = ops.exp(x)
    ref = np.exp(x.astype(np.float64))
    norm = (ref > 1.2e-38) & (ref < 3.0e38)
    assert _ulp_diff(got[norm], ref[norm].astype(np.float32)).max() <= 1
    assert ops.exp(np.float32([np.inf, -np.inf, 100.0, -200.0])).tolist() == [np.inf, 0.0, np.inf, 0.0]
    assert np.isnan(ops.exp(np.float32([np.nan]))[0])


def test_log_within_2ulp_of_libm():
    r = np.random.default_rng(1)
    x = np.concatenate([np.exp(r.uniform(-87, 88, 400_000)).astype(np.float32),
                        (1.0 + r.uniform(-0.3, 0.3, 200_000)).astype(np.float32),
                        (1.0 + np.float32(2.0) ** -np.arange(1, 24, dtype=np.float32)),
                        np.float32([1e-40, 3e-45, 1.0, 2.0, 0.5])])
    got = ops.log(x)
    ref = np.log(x.astype(np.float64)).astype(np.float32)
    assert _ulp_diff(got, ref).max() <= 2
    sp = ops.log(np.float32([0.0, -1.0, np.inf]))
    assert sp[0] == -np.inf and np.isnan(sp[1]) and sp[2] == np.inf


def _reference_bf16_math(xf):
    """gdn_fused.py:22-41 restated in numpy with correctly rounded exp/log (float64 -> float32)."""
    R = ops.bf16_round
    f = np.float32
    ex = lambda v: np.exp(v.astype(np.float64)).astype(np.float32)
    lg = lambda v: np.log(v.astype(np.float64)).astype(np.float32)
    with np.errstate(all="ignore"):
        y = R(f(1) / R(f(1) + R(ex(np.abs(xf)))))
        sig = np.where(xf < 0, y, R(f(1) - y))
        silu = R(xf * sig)
        hi = np.where(xf > 0, xf, f(0))
        lo = np.where(xf < 0, xf, f(0))
        e = R(ex(R(lo - hi)))
        xp1 = f(1) + e
        l1p = np.where(xp1 == f(1), e, R(e * (lg(xp1) / (xp1 - f(1)))))
        sp = R(hi + l1p)
    return sig, silu, sp


def test_bf16_formulas_follow_reference_structure():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    xf = ops.bf16_to_f32(bits)
    finite = np.isfinite(xf)
    got = ops.bf16_formulas(bits)
    ref = _reference_bf16_math(xf)
    for name, r in zip(("sigmoid", "silu", "softplus"), ref):
        g = got[name]
        same = (g == r) | (np.isnan(g) & np.isnan(r))
        miss = np.count_nonzero(~same[finite])
        # identical on every finite bf16 input to the reference formulas evaluated with a
        # correctly rounded exp/log
        assert miss == 0, (name, miss)
        assert np.all(ops.bf16_round(g[finite]) == g[finite])


def test_silu_f32_accuracy():
    x = ops.bf16_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    x = x[np.isfinite(x) & (np.abs(x) < 80)]
    got = ops.bf16_formulas(ops.f32_to_bf16(x))["silu_f32"]
    ref = x.astype(np.float64) / (1 + np.exp(-x.astype(np.float64)))
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)
    assert np.median(rel) < 1e-7 and rel[np.abs(ref) > 1e-30].max() < 5e-7
