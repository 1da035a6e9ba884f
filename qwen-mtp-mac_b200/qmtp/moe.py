"""MXFP4 / NVFP4 MoE expert decode -- the experiments/deepseek_moe surface of qwen-mtp-mac on B200.

Reference: experiments/deepseek_moe/kernels.py:133-155 ``moe_decode(x, wg, sg, wu, su, wd, sd, idx,
scores, *, limit=10.0, nsg=1, rows_gu=4, rows_down=2)`` -- batch 1, two Metal dispatches.  Here the
same call also takes T tokens at once (x [T, H], idx / scores [T, NE]) and runs as a grouped
tcgen05 GEMM over the experts (see csrc/moe.cu).  ``nsg``, ``rows_gu`` and ``rows_down`` are Metal
launch shapes; they are accepted and ignored.

Weights use the reference layout (kernels.py:3-5): w uint32 [E, N, K/8] with 8 e2m1 nibbles per word
(low nibble = lowest k), scales uint8 [E, N, K/32] e8m0 (mode "mxfp4") or [E, N, K/16] e4m3 ("nvfp4").

``route`` builds (idx, scores) from router logits the way bench_moe.py:40-42 does for one token:
top-k routed experts with softmax weights renormalised over the k, times ``routed_scale``, then the
shared experts with weight 1.
"""
from __future__ import annotations

import math

import torch

from . import _lib

MODES = {"mxfp4": (0, 32), "nvfp4": (1, 16)}


def _mode(mode: str):
    try:
        return MODES[mode]
    except KeyError:
        raise ValueError(f"unknown fp4 mode {mode!r} (expected 'mxfp4' or 'nvfp4')") from None


def quantize(w: torch.Tensor, mode: str = "mxfp4"):
    """bf16 [..., N, K] -> (w [..., N, K/8] int32 holding the uint32 words, scales uint8 [..., N, K/G])."""
    fmt, G = _mode(mode)
    if w.dtype != torch.bfloat16:
        raise ValueError("quantize expects bf16 weights")
    _lib.require_cuda(w)
    w = w.contiguous()
    K = w.shape[-1]
    if K % G:
        raise ValueError(f"K = {K} is not a multiple of the {mode} group size {G}")
    N = w.numel() // K
    wq = torch.empty(w.shape[:-1] + (K // 8,), dtype=torch.int32, device=w.device)
    sc = torch.empty(w.shape[:-1] + (K // G,), dtype=torch.uint8, device=w.device)
    _lib.check(_lib.lib().qmtp_quantize_fp4(fmt, w.data_ptr(), N, K, wq.data_ptr(), sc.data_ptr(), _lib.stream()),
               "qmtp_quantize_fp4")
    return wq, sc


def route(logits: torch.Tensor, top_k: int = 6, n_shared: int = 2, routed_scale: float = 1.0):
    """fp32 [T, E] -> (idx int32 [T, top_k + n_shared], scores fp32 [T, top_k + n_shared])."""
    _lib.require_cuda(logits)
    lg = logits.float().contiguous().reshape(-1, logits.shape[-1])
    T, E = lg.shape
    S = top_k + n_shared
    idx = torch.empty((T, S), dtype=torch.int32, device=lg.device)
    sc = torch.empty((T, S), dtype=torch.float32, device=lg.device)
    _lib.check(_lib.lib().qmtp_moe_route(lg.data_ptr(), T, E, top_k, n_shared, float(routed_scale), idx.data_ptr(),
                                         sc.data_ptr(), _lib.stream()), "qmtp_moe_route")
    return idx, sc


_WS: dict = {}


def _workspace(device, T, S, E, H, I) -> torch.Tensor:
    key = (device, T, S, E, H, I)
    ws = _WS.get(key)
    if ws is None:
        n = _lib.lib().qmtp_moe_workspace(T, S, E, H, I)
        ws = torch.empty(n + 256, dtype=torch.uint8, device=device)
        _WS.clear()  # keep one shape resident
        _WS[key] = ws
    return ws


def _aligned(ws: torch.Tensor) -> int:
    p = ws.data_ptr()
    return (p + 255) & ~255


def moe_decode(x, wg, sg, wu, su, wd, sd, idx, scores, *, limit=10.0, nsg=1, rows_gu=4, rows_down=2,
               mode: str = "mxfp4", out: torch.Tensor | None = None):
    """y = sum_j scores[j] * Wd[idx[j]] (silu(min(Wg x, L)) * clamp(Wu x, -L, L)) (kernels.py:133-155).

    x bf16 [H] or [T, H]; idx int32 [NE] or [T, NE]; scores fp32 like idx.  ``limit=None`` (or inf)
    disables the SwiGLU clamp.  Returns bf16 with x's shape."""
    fmt, G = _mode(mode)
    del nsg, rows_gu, rows_down
    _lib.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("moe_decode expects bf16 activations")
    H = x.shape[-1]
    x2 = x.reshape(-1, H).contiguous()
    T = x2.shape[0]
    idx2 = idx.reshape(T, -1).to(torch.int32).contiguous()
    sc2 = scores.reshape(T, -1).to(torch.float32).contiguous()
    S = idx2.shape[1]
    E, I = wg.shape[0], wg.shape[1]
    if wg.shape[-1] * 8 != H or wd.shape[1] != H or wd.shape[-1] * 8 != I or sg.shape[-1] * G != H:
        raise ValueError("moe_decode: weight shapes do not match x / mode")
    lim = math.inf if limit is None else float(limit)
    y = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    ws = _workspace(x.device, T, S, E, H, I)
    need = _lib.lib().qmtp_moe_workspace(T, S, E, H, I)
    ts = [t.contiguous() for t in (wg, sg, wu, su, wd, sd)]
    _lib.check(_lib.lib().qmtp_moe(fmt, x2.data_ptr(), *[t.data_ptr() for t in ts], idx2.data_ptr(), sc2.data_ptr(),
                                   y.data_ptr(), T, S, E, H, I, lim, _aligned(ws), need, _lib.stream()), "qmtp_moe")
    return y.reshape(x.shape)


def experts(x_rows: torch.Tensor, wg, sg, wu, su, wd, sd, expert: torch.Tensor, *, limit=None,
            mode: str = "mxfp4", out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row expert FFN without the routing weight: fp32 [n, H], row r through expert[r].

    The expert-parallel building block (the rows a rank received for its local experts)."""
    fmt, G = _mode(mode)
    _lib.require_cuda(x_rows)
    H = x_rows.shape[-1]
    x2 = x_rows.reshape(-1, H).contiguous()
    n = x2.shape[0]
    e = expert.reshape(n).to(torch.int32).contiguous()
    E, I = wg.shape[0], wg.shape[1]
    y = out if out is not None else torch.empty((n, H), dtype=torch.float32, device=x_rows.device)
    if n == 0:
        return y
    ws = _workspace(x_rows.device, n, 1, E, H, I)
    need = _lib.lib().qmtp_moe_workspace(n, 1, E, H, I)
    lim = math.inf if limit is None else float(limit)
    ts = [t.contiguous() for t in (wg, sg, wu, su, wd, sd)]
    _lib.check(_lib.lib().qmtp_moe_experts(fmt, x2.data_ptr(), *[t.data_ptr() for t in ts], e.data_ptr(), y.data_ptr(),
                                           n, E, H, I, lim, _aligned(ws), need, _lib.stream()), "qmtp_moe_experts")
    return y


def combine(partials: torch.Tensor, row_of: torch.Tensor, scores: torch.Tensor, out: torch.Tensor | None = None):
    """y[t] = sum_j scores[t, j] * partials[row_of[t, j]] in slot order (fp32 sum, bf16 result)."""
    _lib.require_cuda(partials)
    T, S = row_of.shape
    H = partials.shape[-1]
    y = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=partials.device)
    r = row_of.to(torch.int32).contiguous()
    sc = scores.to(torch.float32).contiguous()
    _lib.check(_lib.lib().qmtp_moe_combine(partials.data_ptr(), r.data_ptr(), sc.data_ptr(), T, S, H, y.data_ptr(),
                                           _lib.stream()), "qmtp_moe_combine")
    return y


def dispatch(idx: torch.Tensor, x: torch.Tensor, n_routed: int, n_shared: int, world: int, cap: int,
             send_x: torch.Tensor, send_e: torch.Tensor, sh_x: torch.Tensor, sh_e: torch.Tensor,
             pos: torch.Tensor, counts: torch.Tensor) -> None:
    """Fixed-capacity expert-parallel dispatch into caller buffers (qmtp_moe_dispatch): send_x
    [world * cap, H], send_e [world * cap], sh_x [T * S, H], sh_e [T * S], pos [T * S], counts
    [world + 1]; see include/qmtp.h for the layout."""
    _lib.require_cuda(x)
    T, S = idx.shape
    H = x.shape[-1]
    i32 = idx.to(torch.int32).contiguous()
    _lib.check(_lib.lib().qmtp_moe_dispatch(i32.data_ptr(), T, S, x.data_ptr(), H, n_routed, n_shared, world, cap,
                                            send_x.data_ptr(), send_e.data_ptr(), sh_x.data_ptr(), sh_e.data_ptr(),
                                            pos.data_ptr(), counts.data_ptr(), _lib.stream()), "qmtp_moe_dispatch")
