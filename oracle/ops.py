"""numpy front-end of the C oracle (TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py).

bf16 tensors are numpy uint16 bit patterns throughout.  Each wrapper names the C function (and
through it the reference file:line) it forwards to.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import build as _build

_lib = None
_lock = threading.Lock()
_P = ctypes.c_void_p
_I = ctypes.c_int


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                L = ctypes.CDLL(str(_build.build()))
                L.qo_exp.argtypes = [ctypes.c_float]
                L.qo_exp.restype = ctypes.c_float
                L.qo_log.argtypes = [ctypes.c_float]
                L.qo_log.restype = ctypes.c_float
                L.qo_dot_bf16.argtypes = [_P, _P, _I]
                L.qo_dot_bf16.restype = ctypes.c_float
                _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(_P)


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits; NaN -> 0x7FC0 (the library's rule)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(a) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(a))


# ---------------------------------------------------------------- elementwise math
def exp(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().qo_exp_arr(_p(x), _p(y), ctypes.c_long(x.size))
    return y


def log(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().qo_log_arr(_p(x), _p(y), ctypes.c_long(x.size))
    return y


def bf16_formulas(x_bits) -> dict:
    """sigmoid_bf, silu_bf, softplus_bf (gdn_fused.py:22-41) and silu_f32 over bf16 bit patterns."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    out = {k: np.empty(x.size, np.float32) for k in ("sigmoid", "silu", "softplus", "silu_f32")}
    lib().qo_bf16_formulas(_p(x), _I(x.size), _p(out["sigmoid"]), _p(out["silu"]), _p(out["softplus"]),
                           _p(out["silu_f32"]))
    return out


def decode_tables():
    """(e2m1[16], e4m3[256], e8m0[256]) as float32."""
    a, b, c = np.empty(16, np.float32), np.empty(256, np.float32), np.empty(256, np.float32)
    lib().qo_decode_tables(_p(a), _p(b), _p(c))
    return a, b, c


# ---------------------------------------------------------------- quantized GEMV
def quantize_affine(w_bf16: np.ndarray, group_size: int = 64):
    """C qo_quantize_affine: bf16 [N, K] -> (wq uint32 [N, K/8], scales bf16, biases bf16)."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    N, K = w.shape
    wq = np.empty((N, K // 8), np.uint32)
    s = np.empty((N, K // group_size), np.uint16)
    b = np.empty((N, K // group_size), np.uint16)
    lib().qo_quantize_affine(_p(w), _p(wq), _p(s), _p(b), _I(N), _I(K), _I(group_size))
    return wq, s, b


def qmv_affine(x_bf16, wq, s, b) -> np.ndarray:
    """C qo_qmv_affine (canonical qmv, qmv_kernel.py:31-75 order of roles): y bf16 [M, N]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, np.shape(x_bf16)[-1])
    wq = np.ascontiguousarray(wq).view(np.uint32)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.empty((M, N), np.uint16)
    rc = lib().qo_qmv_affine(_p(x), _p(wq), _p(s), _p(b), _p(y), _I(M), _I(N), _I(K))
    if rc != 0:
        raise ValueError("qo_qmv_affine: unsupported shape")
    return y


def qmv_nvfp4(x_bf16, wq, s_u8) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, np.shape(x_bf16)[-1])
    wq = np.ascontiguousarray(wq).view(np.uint32)
    s = np.ascontiguousarray(s_u8, dtype=np.uint8)
    M, K = x.shape
    N = wq.shape[0]
    y = np.empty((M, N), np.uint16)
    rc = lib().qo_qmv_nvfp4(_p(x), _p(wq), _p(s), _p(y), _I(M), _I(N), _I(K))
    if rc != 0:
        raise ValueError("qo_qmv_nvfp4: unsupported shape")
    return y


def dequant_affine(wq, s, b, group_size: int = 64) -> np.ndarray:
    """float64 dequantized weights (for tolerance checks against plain math)."""
    wq = np.ascontiguousarray(wq).view(np.uint32)
    N = wq.shape[0]
    K = wq.shape[1] * 8
    q = np.empty((N, K), np.float64)
    for i in range(8):
        q[:, i::8] = (wq >> (4 * i)) & 15
    sf = np.repeat(bf16_to_f32(s).astype(np.float64), group_size, axis=1)
    bf = np.repeat(bf16_to_f32(b).astype(np.float64), group_size, axis=1)
    return sf * q + bf


# ---------------------------------------------------------------- GatedDeltaNet
def gdn_step(q, k, v, g, beta, state):
    """C qo_gdn_step (gdn_kernel.py:11-88): returns (y bf16, state_out, state_mid [T-1,...])."""
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    g = np.ascontiguousarray(g, np.float32)
    beta = np.ascontiguousarray(beta, np.float32)
    state = np.ascontiguousarray(state, np.float32)
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2:]
    y = np.empty((B, T, Hv, Dv), np.uint16)
    so = np.empty_like(state)
    sm = np.empty((max(T - 1, 1),) + state.shape, np.float32)
    rc = lib().qo_gdn_step(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(state), _p(y), _p(so), _p(sm),
                           _I(B), _I(T), _I(Hk), _I(Hv), _I(Dk), _I(Dv))
    assert rc == 0
    return y, so, sm


def gdn_fused(win, conv_w, a, b, A_log, dt_bias, state, Hk, Hv, Dk, Dv, KC, snap=True):
    """C qo_gdn_fused (gdn_fused.py:43-112), B = 1.  win bf16 [S+KC-1, C]; a, b bf16 [S, Hv];
    state fp32 [Hv, Dv, Dk] -> (y fp32 [S, Hv, Dv], state_out, state_mid [S-1, Hv, Dv, Dk])."""
    win = np.ascontiguousarray(win, np.uint16).reshape(-1, 2 * Hk * Dk + Hv * Dv)
    S = win.shape[0] - (KC - 1)
    a = np.ascontiguousarray(a, np.uint16).reshape(S, -1)
    b = np.ascontiguousarray(b, np.uint16).reshape(S, -1)
    conv_w = np.ascontiguousarray(conv_w, np.uint16)
    A_log = np.ascontiguousarray(A_log, np.float32)
    dt_bias = np.ascontiguousarray(dt_bias, np.uint16)
    state = np.ascontiguousarray(state, np.float32).reshape(Hv, Dv, Dk)
    y = np.empty((S, Hv, Dv), np.float32)
    so = np.empty_like(state)
    sm = np.empty((max(S - 1, 1), Hv, Dv, Dk), np.float32)
    rc = lib().qo_gdn_fused(_p(win), _p(conv_w), _p(a), _p(b), _I(a.shape[1]), _p(A_log), _p(dt_bias), _p(state),
                            _p(y), _p(so), _p(sm) if snap else None, _I(S), _I(Hk), _I(Hv), _I(Dk), _I(Dv), _I(KC))
    assert rc == 0
    return y, so, sm


def swiglu(gu, I):
    """C qo_swiglu (mlx-lm SwiGLU with the bf16 formulas of gdn_fused.py:22-41): gu bf16 [S, >=2I] =
    [gate | up] -> bf16(silu(gate) * up) [S, I]."""
    gu = np.ascontiguousarray(gu, np.uint16)
    S = gu.shape[0]
    out = np.empty((S, I), np.uint16)
    lib().qo_swiglu(_p(gu), _I(gu.shape[1]), _I(S), _I(I), _p(out))
    return out


def gdn_norm_gate(y, z, w, eps):
    """C qo_gdn_norm_gate (gdn_fused.py:114-129): y fp32 [S, H, Dv], z bf16 [S, H*Dv] -> bf16 [S, H*Dv]."""
    y = np.ascontiguousarray(y, np.float32)
    S, H, Dv = y.shape
    z = np.ascontiguousarray(z, np.uint16).reshape(S, H * Dv)
    w = np.ascontiguousarray(w, np.uint16)
    out = np.empty((S, H * Dv), np.uint16)
    lib().qo_gdn_norm_gate(_p(y), _p(z), _I(H * Dv), _p(w), _p(out), _I(S), _I(H), _I(Dv), ctypes.c_float(eps))
    return out


def gdn_fused_prep(win, conv_w, a, b, A_log, dt_bias, Hk, Hv, Dk, Dv, KC, **_):
    """C qo_gdn_fused_prep: (q [S,Hk,Dk], k [S,Hk,Dk], v [S,Hv,Dv], g [S,Hv], beta [S,Hv]) as fp32."""
    win = np.ascontiguousarray(win, np.uint16).reshape(-1, 2 * Hk * Dk + Hv * Dv)
    S = win.shape[0] - (KC - 1)
    a = np.ascontiguousarray(a, np.uint16).reshape(S, -1)
    b = np.ascontiguousarray(b, np.uint16).reshape(S, -1)
    out = [np.empty((S, Hk, Dk), np.float32), np.empty((S, Hk, Dk), np.float32), np.empty((S, Hv, Dv), np.float32),
           np.empty((S, Hv), np.float32), np.empty((S, Hv), np.float32)]
    rc = lib().qo_gdn_fused_prep(_p(win), _p(np.ascontiguousarray(conv_w, np.uint16)), _p(a), _p(b), _I(a.shape[1]),
                                 _p(np.ascontiguousarray(A_log, np.float32)),
                                 _p(np.ascontiguousarray(dt_bias, np.uint16)), *[_p(o) for o in out],
                                 _I(S), _I(Hk), _I(Hv), _I(Dk), _I(Dv), _I(KC))
    assert rc == 0
    return tuple(out)


# ---------------------------------------------------------------- two-stage lm_head (lm_head2.py)
def topk_bf16(vals, k):
    v = np.ascontiguousarray(vals, np.uint16)
    v2 = v.reshape(-1, v.shape[-1])
    out = np.empty((v2.shape[0], k), np.int32)
    assert lib().qo_topk_bf16(_p(v2), _I(v2.shape[0]), _I(v2.shape[1]), _I(v2.shape[1]), _I(k), _p(out)) == 0
    return out


def rescore_bf16(W, h, idx):
    W = np.ascontiguousarray(W, np.uint16)
    h = np.ascontiguousarray(h, np.uint16).reshape(-1, W.shape[1])
    idx = np.ascontiguousarray(idx, np.int32)
    M, k = idx.shape
    fine = np.empty((M, k), np.uint16)
    amax = np.empty(M, np.int32)
    assert lib().qo_rescore_bf16(_p(W), _p(h), _p(idx), _I(M), _I(k), _I(W.shape[1]), _p(fine), _p(amax)) == 0
    return fine, amax


def argmax_bf16(vals):
    v = np.ascontiguousarray(vals, np.uint16)
    v2 = v.reshape(-1, v.shape[-1])
    out = np.empty(v2.shape[0], np.int32)
    lib().qo_argmax_bf16(_p(v2), _I(v2.shape[0]), _I(v2.shape[1]), _I(v2.shape[1]), _p(out))
    return out


def draft_prob(logits, token):
    """C qo_draft_prob: softmax(logits)[token] (the draft head's argmax probability, mtp.py:222-223)."""
    v = np.ascontiguousarray(logits, np.uint16).reshape(-1)
    lib().qo_draft_prob.restype = ctypes.c_float
    return float(lib().qo_draft_prob(_p(v), _I(v.size), _I(int(token))))


def n_drafts(probs, tau):
    """mtp.py:229-238: drafts to verify -- while the running product stays >= tau (at least 1)."""
    n, acc = 0, 1.0
    for p in probs:
        acc *= p
        if n and acc < tau:
            break
        n += 1
    return n


def two_stage_head(h, wq, s, b, W, k=64):
    """lm_head2.py:23-29 restated: (coarse bf16 [M,V], idx [M,k], fine bf16 [M,k], argmax [M])."""
    coarse = qmv_affine(h, wq, s, b)
    idx = topk_bf16(coarse, k)
    fine, amax = rescore_bf16(W, h, idx)
    return coarse, idx, fine, amax


def two_stage_head_nvfp4(h, wq, s_u8, W, k=64):
    """lm_head2.py:14-29 with the reference's NVFP4 g16 coarse copy (lm_head2.py:19) restated:
    (coarse bf16 [M,V], idx [M,k], fine bf16 [M,k], argmax [M])."""
    coarse = qmv_nvfp4(h, wq, s_u8)
    idx = topk_bf16(coarse, k)
    fine, amax = rescore_bf16(W, h, idx)
    return coarse, idx, fine, amax


def dot_bf16(w_row, h_row) -> np.float32:
    """C qo_dot_bf16: the fine-logit dot product in its fixed order (fp32, before bf16 rounding)."""
    w = np.ascontiguousarray(w_row, np.uint16)
    h = np.ascontiguousarray(h_row, np.uint16)
    return np.float32(lib().qo_dot_bf16(_p(w), _p(h), _I(w.size)))


# ---------------------------------------------------------------- MXFP4 / NVFP4 MoE (experiments/deepseek_moe)
FP4_FORMATS = {"mxfp4": (0, 32), "nvfp4": (1, 16)}


def quantize_fp4(w_bf16, mode: str = "mxfp4"):
    """C qo_quantize_fp4: bf16 [..., N, K] -> (w uint32 [..., N, K/8], scales uint8 [..., N, K/G])."""
    fmt, G = FP4_FORMATS[mode]
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    lead, K = w.shape[:-1], w.shape[-1]
    N = int(np.prod(lead))
    wq = np.empty(lead + (K // 8,), np.uint32)
    s = np.empty(lead + (K // G,), np.uint8)
    assert lib().qo_quantize_fp4(_I(fmt), _p(w), ctypes.c_long(N), _I(K), _p(wq), _p(s)) == 0
    return wq, s


def dequant_fp4(wq, s, mode: str = "mxfp4") -> np.ndarray:
    fmt, _ = FP4_FORMATS[mode]
    wq = np.ascontiguousarray(wq, np.uint32)
    s = np.ascontiguousarray(s, np.uint8)
    K = wq.shape[-1] * 8
    N = int(np.prod(wq.shape[:-1]))
    out = np.empty(wq.shape[:-1] + (K,), np.float32)
    lib().qo_dequant_fp4(_I(fmt), _p(wq), _p(s), ctypes.c_long(N), _I(K), _p(out))
    return out


def moe_route(logits, top_k: int = 6, n_shared: int = 2, routed_scale: float = 1.0):
    """C qo_moe_route: fp32 [T, E] -> (idx int32 [T, top_k+n_shared], scores fp32)."""
    lg = np.ascontiguousarray(logits, np.float32)
    T, E = lg.shape
    S = top_k + n_shared
    idx = np.empty((T, S), np.int32)
    sc = np.empty((T, S), np.float32)
    lib().qo_moe_route(_p(lg), _I(T), _I(E), _I(top_k), _I(n_shared), ctypes.c_float(routed_scale), _p(idx), _p(sc))
    return idx, sc


def moe(x_bf16, wg, sg, wu, su, wd, sd, idx, scores, mode: str = "mxfp4", limit=None):
    """C qo_moe (experiments/deepseek_moe/kernels.py:35-107 for T tokens): (y bf16 [T,H], y fp32 [T,H])."""
    fmt, _ = FP4_FORMATS[mode]
    x = np.ascontiguousarray(x_bf16, np.uint16)
    x = x.reshape(-1, x.shape[-1])
    T, H = x.shape
    idx = np.ascontiguousarray(idx, np.int32).reshape(T, -1)
    scores = np.ascontiguousarray(scores, np.float32).reshape(T, -1)
    E, I = wg.shape[0], wg.shape[1]
    arrs = [np.ascontiguousarray(a) for a in (wg, sg, wu, su, wd, sd)]
    yb = np.empty((T, H), np.uint16)
    yf = np.empty((T, H), np.float32)
    lim = np.float32(np.inf if limit is None else limit)
    rc = lib().qo_moe(_I(fmt), _p(x), *[_p(a) for a in arrs], _p(idx), _p(scores), _I(T), _I(idx.shape[1]), _I(E),
                      _I(H), _I(I), ctypes.c_float(lim), _p(yf), _p(yb))
    if rc != 0:
        raise ValueError(f"qo_moe: rc {rc}")
    return yb, yf


# ---------------------------------------------------------------- speculative sampling (T > 0)
def philox4x32_10(ctr, key) -> np.ndarray:
    """C qo_philox4x32_10: Philox4x32-10 of a 4-word counter under a 2-word key."""
    c = np.ascontiguousarray(ctr, np.uint32)
    k = np.ascontiguousarray(key, np.uint32)
    o = np.empty(4, np.uint32)
    lib().qo_philox4x32_10(_p(c), _p(k), _p(o))
    return o


def sample(idx, fine, drafts, temperature, top_k=0, top_p=1.0, min_p=0.0, V=None, seed=0, ctr=0, first_row=-1):
    """C qo_sample over candidate rows idx int32 [R, K] / fine bf16 [R, K]: verify mode (first_row < 0)
    returns (n_acc, emitted tokens); first mode returns the token drawn from row first_row."""
    idx = np.ascontiguousarray(idx, np.int32)
    fine = np.ascontiguousarray(fine, np.uint16)
    R, K = idx.shape
    d = np.ascontiguousarray(drafts if drafts is not None else [], np.int32)
    k = int(d.size)
    out = np.zeros(max(k + 1, 1), np.int32)
    f = lib().qo_sample
    f.restype = ctypes.c_int
    n = f(_p(idx), _p(fine), _I(K), _I(K), _p(d) if k else None, _I(k), _I(first_row), ctypes.c_float(temperature),
          _I(top_k), ctypes.c_float(top_p), ctypes.c_float(min_p), _I(V if V is not None else 1 << 30),
          ctypes.c_uint32(seed & 0xFFFFFFFF), ctypes.c_uint32((seed >> 32) & 0xFFFFFFFF), ctypes.c_uint32(ctr),
          _p(out))
    if n < 0:
        raise ValueError("qo_sample: bad arguments")
    if first_row >= 0:
        return int(out[0])
    return n, [int(v) for v in out[:n + 1]]


def sample_dist(idx, fine, temperature, top_k=0, top_p=1.0, min_p=0.0, V=None):
    """C qo_sample_dist: (kept vocabulary ids in order, their probabilities) of one candidate row."""
    idx = np.ascontiguousarray(idx, np.int32).ravel()
    fine = np.ascontiguousarray(fine, np.uint16).ravel()
    K = idx.size
    oi, op = np.empty(K, np.int32), np.empty(K, np.float32)
    f = lib().qo_sample_dist
    f.restype = ctypes.c_int
    n = f(_p(idx), _p(fine), _I(K), ctypes.c_float(temperature), _I(top_k), ctypes.c_float(top_p),
          ctypes.c_float(min_p), _I(V if V is not None else 1 << 30), _p(oi), _p(op))
    if n < 0:
        raise ValueError("qo_sample_dist: bad arguments")
    return oi[:n], op[:n]
