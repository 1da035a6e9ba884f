"""Oracle GatedDeltaNet (CPU): snapshot semantics, fused == unfused, and float64 agreement.

Mirrors tests/test_kernels.py:40-60 (snapshot step == T sequential single-token updates, bit-exact)
and :63-95 (the fused path equals the unfused one, bit-exact), with the oracle as both sides.
"""
import numpy as np
import pytest

from oracle import ops
from tests._util import randn_bf16, rng


def _l2norm_bf16(x):
    xf = x.astype(np.float64)
    return ops.f32_to_bf16((xf / np.linalg.norm(xf, axis=-1, keepdims=True)).astype(np.float32))


def config2_inputs(T=3, B=1, Hk=16, Hv=32, D=128, seed=0):
    r = rng(seed)
    q = _l2norm_bf16(r.standard_normal((B, T, Hk, D)).astype(np.float32))
    k = _l2norm_bf16(r.standard_normal((B, T, Hk, D)).astype(np.float32))
    v = ops.f32_to_bf16(r.standard_normal((B, T, Hv, D)).astype(np.float32))
    a = r.standard_normal((B, T, Hv))
    g = np.exp(-np.log1p(np.exp(a))).astype(np.float32)
    beta = (1 / (1 + np.exp(-r.standard_normal((B, T, Hv))))).astype(np.float32)
    state = (r.standard_normal((B, Hv, D, D)) * 0.1).astype(np.float32)
    return q, k, v, g, beta, state


def test_snapshot_equals_sequential_steps():
    q, k, v, g, beta, state = config2_inputs(T=4)
    y, s_final, mids = ops.gdn_step(q, k, v, g, beta, state)
    s = state
    for t in range(4):
        yt, s, _ = ops.gdn_step(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1], s)
        assert np.array_equal(yt[:, 0], y[:, t])
        if t < 3:
            assert np.array_equal(mids[t], s)
    assert np.array_equal(s_final, s)


def test_step_matches_float64():
    q, k, v, g, beta, state = config2_inputs(T=3, seed=1)
    y, s_final, mids = ops.gdn_step(q, k, v, g, beta, state)
    B, T, Hk, D = k.shape
    Hv = v.shape[2]
    S = state.astype(np.float64)
    for t in range(T):
        kk = np.repeat(ops.bf16_to_f32(k[:, t]).astype(np.float64), Hv // Hk, axis=1)  # [B, Hv, D]
        qq = np.repeat(ops.bf16_to_f32(q[:, t]).astype(np.float64), Hv // Hk, axis=1)
        vv = ops.bf16_to_f32(v[:, t]).astype(np.float64)
        S = S * g[:, t, :, None, None]
        kv = np.einsum("bhvk,bhk->bhv", S, kk)
        delta = (vv - kv) * beta[:, t, :, None]
        S = S + delta[..., None] * kk[:, :, None, :]
        yy = np.einsum("bhvk,bhk->bhv", S, qq)
        assert np.abs(ops.bf16_to_f32(y[:, t]) - yy).max() <= 2 ** -8 * np.abs(yy).max() + 1e-6
        ref_state = S if t == T - 1 else None
        if t < T - 1:
            assert np.abs(mids[t] - S).max() <= 1e-5 * np.abs(S).max()
    assert np.abs(s_final - ref_state).max() / np.abs(ref_state).max() <= 1e-5  # fp32 state tolerance is 1e-3


def fused_inputs(S=3, Hk=16, Hv=32, D=128, KC=4, seed=0):
    r = rng(seed)
    C = 2 * Hk * D + Hv * D
    win = randn_bf16((S + KC - 1, C), seed + 1)
    conv_w = randn_bf16((C, KC), seed + 2, 0.5)
    a = randn_bf16((S, Hv), seed + 3)
    b = randn_bf16((S, Hv), seed + 4)
    A_log = np.log(r.uniform(1, 16, Hv)).astype(np.float32)
    dt_bias = randn_bf16((Hv,), seed + 5)
    state = (r.standard_normal((Hv, D, D)) * 0.1).astype(np.float32)
    return dict(win=win, conv_w=conv_w, a=a, b=b, A_log=A_log, dt_bias=dt_bias, state=state,
                Hk=Hk, Hv=Hv, Dk=D, Dv=D, KC=KC)


@pytest.mark.parametrize("S", [1, 3])
def test_fused_equals_sequential_tokens(S):
    d = fused_inputs(S=S, seed=7)
    y, so, sm = ops.gdn_fused(**d)
    st = d["state"]
    for t in range(S):
        dt = dict(d, win=d["win"][t:t + d["KC"]], a=d["a"][t:t + 1], b=d["b"][t:t + 1], state=st)
        yt, st, _ = ops.gdn_fused(**dt)
        assert np.array_equal(yt[0], y[t])
        if t < S - 1:
            assert np.array_equal(sm[t], st)
    assert np.array_equal(so, st)


def test_fused_delta_rule_equals_snapshot_step():
    """gdn_core == gated_delta_snapshot fed with gdn_core's own q, k, v, g, beta (the reference's
    fused kernel is bit-exact with the mlx path that calls the snapshot kernel)."""
    d = fused_inputs(S=3, seed=11)
    y, so, sm = ops.gdn_fused(**d)
    q, k, v, g, beta = ops.gdn_fused_prep(**d)
    for arr in (q, k, v):
        assert np.array_equal(ops.bf16_round(arr), arr)  # bf16-exact, so the bf16 API loses nothing
    ys, ss, ms = ops.gdn_step(ops.f32_to_bf16(q)[None], ops.f32_to_bf16(k)[None], ops.f32_to_bf16(v)[None],
                              g[None], beta[None], d["state"][None])
    assert np.array_equal(ops.f32_to_bf16(y), ys[0])
    assert np.array_equal(so, ss[0]) and np.array_equal(sm, ms[:, 0])


def test_norm_gate_matches_float64():
    r = rng(3)
    S, H, D = 3, 32, 128
    y = ops.bf16_round((r.standard_normal((S, H, D))).astype(np.float32))
    z = randn_bf16((S, H * D), 4)
    w = ops.f32_to_bf16((1 + 0.2 * r.standard_normal(D)).astype(np.float32))
    out = ops.bf16_to_f32(ops.gdn_norm_gate(y, z, w, 1e-6)).reshape(S, H, D).astype(np.float64)
    yf = y.astype(np.float64)
    rr = 1 / np.sqrt((yf ** 2).mean(-1, keepdims=True) + 1e-6)
    zf = ops.bf16_to_f32(z).reshape(S, H, D).astype(np.float64)
    ref = ops.bf16_to_f32(w).astype(np.float64) * yf * rr * zf / (1 + np.exp(-zf))
    assert np.abs(out - ref).max() <= 3 * 2 ** -8 * np.abs(ref).max()
