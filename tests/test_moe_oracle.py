"""MoE oracle (CPU): fp4 quantizer rules, router semantics and the expert FFN restatement.

The reference (experiments/deepseek_moe/kernels.py) has no CPU path and no golden vectors; its
decoders are pinned in test_formats.py.  Here the oracle's MoE is checked against independent
numpy float64 math written from kernels.py:35-107 and bench_moe.py:40-42."""
import numpy as np
import pytest

from oracle import ops
from tests._util import randn_bf16, rng

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float64)


def _nearest_e2m1(v):
    """RNE onto the e2m1 grid, saturating at 6; ties to the even code."""
    a = np.abs(v)
    code = np.zeros(a.shape, np.int64)
    for c in range(1, 8):
        mid = (E2M1[c - 1] + E2M1[c]) / 2
        take = (a > mid) | ((a == mid) & (c % 2 == 0))
        code = np.where(take, c, code)
    return np.where(np.signbit(v) & (code > 0), -E2M1[code], E2M1[code])


@pytest.mark.parametrize("mode", ["mxfp4", "nvfp4"])
def test_quantizer_is_nearest_grid_point(mode):
    G = 32 if mode == "mxfp4" else 16
    w = randn_bf16((48, 256), 1, 0.02)
    w[0, :G] = 0                       # all-zero group
    w[1, :G] = ops.f32_to_bf16(np.float32(1e-30))  # tiny group
    wq, s = ops.quantize_fp4(w, mode)
    deq = ops.dequant_fp4(wq, s, mode).astype(np.float64)
    wf = ops.bf16_to_f32(w).astype(np.float64).reshape(48, -1, G)
    _, e4m3, e8m0 = ops.decode_tables()
    sc = (e8m0 if mode == "mxfp4" else e4m3)[s].astype(np.float64)[..., None]
    want = np.where(sc > 0, _nearest_e2m1(np.divide(wf, sc, out=np.zeros_like(wf), where=sc > 0)) * sc, 0)
    assert np.array_equal(deq.reshape(want.shape), want)
    assert np.all(deq.reshape(48, -1, G)[0, 0] == 0)


def test_mxfp4_scale_rule():
    # OCP MX: s = floor(log2(amax)) - 2 + 127; the max element lands in [4, 8) -> saturates to 6 above 6
    w = np.zeros((1, 32), np.float32)
    w[0, 0] = 1.0
    w[0, 1] = 7.5       # amax 7.5 -> floor(log2) = 2 -> scale 1 -> 7.5 saturates to 6
    w[0, 2] = -0.25     # tie between 0 and 0.5 -> 0 (even)
    w[0, 3] = 0.75      # tie between 0.5 and 1 -> 1 (even code)
    wq, s = ops.quantize_fp4(ops.f32_to_bf16(w), "mxfp4")
    assert s[0, 0] == 127
    d = ops.dequant_fp4(wq, s, "mxfp4")[0]
    assert list(d[:4]) == [1.0, 6.0, 0.0, 1.0]


def test_nvfp4_scale_rule():
    w = np.zeros((1, 16), np.float32)
    w[0, 0] = 6.0        # amax / 6 = 1 -> e4m3 1.0 = code 0x38
    w[0, 1] = -2.5       # tie 2 / 3 -> 2 (even code 4)
    wq, s = ops.quantize_fp4(ops.f32_to_bf16(w), "nvfp4")
    assert s[0, 0] == 0x38
    d = ops.dequant_fp4(wq, s, "nvfp4")[0]
    assert d[0] == 6.0 and d[1] == -2.0


def _route_np(lg, top_k, n_shared, rs):
    T, E = lg.shape
    idx = np.zeros((T, top_k + n_shared), np.int64)
    sc = np.zeros((T, top_k + n_shared), np.float64)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-lg[t, e], e))[:top_k]
        p = np.exp(lg[t].astype(np.float64) - lg[t].max())
        p /= p.sum()
        w = p[order] / p[order].sum() * rs
        idx[t, :top_k] = order
        sc[t, :top_k] = w
        idx[t, top_k:] = E + np.arange(n_shared)
        sc[t, top_k:] = 1.0
    return idx, sc


def test_router_matches_softmax_topk_renorm():
    lg = rng(3).standard_normal((64, 64)).astype(np.float32)
    lg[0, 5] = lg[0, 9] = 4.0  # tie: lower id first
    idx, sc = ops.moe_route(lg, 6, 2, 1.5)
    ridx, rsc = _route_np(lg, 6, 2, 1.5)
    assert np.array_equal(idx, ridx)
    assert idx[0, 0] == 5 and idx[0, 1] == 9
    assert np.allclose(sc, rsc, rtol=2e-6, atol=0)


def test_router_nan_ranks_last():
    lg = np.full((1, 8), np.nan, np.float32)
    lg[0, 6] = -1.0
    idx, _ = ops.moe_route(lg, 3, 0, 1.0)
    assert list(idx[0]) == [6, 0, 1]


def _moe_np(x, mats, idx, sc, mode, limit):
    Wg, Wu, Wd = [ops.dequant_fp4(q, s, mode).astype(np.float64) for q, s in mats]
    xf = ops.bf16_to_f32(x).astype(np.float64)
    T = x.shape[0]
    y = np.zeros((T, Wd.shape[1]))
    for t in range(T):
        for j in range(idx.shape[1]):
            e = idx[t, j]
            g = np.minimum(Wg[e] @ xf[t], limit)
            u = np.clip(Wu[e] @ xf[t], -limit, limit)
            h = (g / (1 + np.exp(-g)) * u).astype(np.float32).astype(np.float64)
            y[t] += np.float64(sc[t, j]) * (Wd[e] @ h)
    return y


def make_layer(E, H, I, mode, seed=0, std=0.02):
    g = ops.quantize_fp4(randn_bf16((E, I, H), seed, std), mode)
    u = ops.quantize_fp4(randn_bf16((E, I, H), seed + 1, std), mode)
    d = ops.quantize_fp4(randn_bf16((E, H, I), seed + 2, std), mode)
    return g, u, d


@pytest.mark.parametrize("mode,limit", [("mxfp4", np.inf), ("nvfp4", np.inf), ("mxfp4", 0.05)])
def test_moe_oracle_matches_float64(mode, limit):
    E, H, I, T = 6, 128, 96, 5
    (wg, sg), (wu, su), (wd, sd) = make_layer(E, H, I, mode, 11)
    x = randn_bf16((T, H), 4)
    idx, sc = ops.moe_route(rng(5).standard_normal((T, E - 2)).astype(np.float32), 3, 2)
    yb, yf = ops.moe(x, wg, sg, wu, su, wd, sd, idx, sc, mode, None if np.isinf(limit) else limit)
    ref = _moe_np(x, [(wg, sg), (wu, su), (wd, sd)], idx, sc, mode, limit)
    assert np.abs(yf - ref).max() <= 1e-6 * np.abs(ref).max()
    assert np.array_equal(yb, ops.f32_to_bf16(yf))
