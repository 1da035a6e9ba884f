"""Fused GatedDeltaNet middle section (decode / verify, B = 1) -- the gdn_fused.py surface.

Reference: gdn_fused.py:149-167 ``gdn_middle(self, qkv, z, a, b, conv_state, state, snap)`` with its
two kernels ``gdn_core`` (conv1d + silu, q/k RMS norms, gates, delta rule, snapshots) and
``gdn_norm_gate`` (rms_norm(y) * w * silu(z)).  Both run as sm_100a kernels of libqmtp
(csrc/gdn.cu) with the bf16 rounding points of gdn_fused.py:22-41.

``layer`` is any object with the attributes the reference reads from mlx-lm's GatedDeltaNet:
num_k_heads, num_v_heads, head_k_dim, head_v_dim, conv_kernel_size, conv1d_weight (bf16 [C, KC]),
A_log (fp32 [Hv]), dt_bias (bf16 [Hv]), norm_weight (bf16 [Dv]) and norm_eps.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

MAX_S = 64  # the reference caps the fused path at 16 tokens (gdn_fused.py:170); this kernel at 64


def gdn_core(layer, win, a, b, state, snap):
    """win bf16 [1, S+KC-1, C]; a, b bf16 [1, S, Hv]; state fp32 [1, Hv, Dv, Dk]
    -> (y fp32 [S, Hv, Dv], state_out [1, Hv, Dv, Dk], mids [max(S-1,1), 1, Hv, Dv, Dk])."""
    Hk, Hv, Dk, Dv, KC = (layer.num_k_heads, layer.num_v_heads, layer.head_k_dim, layer.head_v_dim,
                          layer.conv_kernel_size)
    S = win.shape[-2] - (KC - 1)
    win = win.contiguous()
    a2 = a.reshape(S, -1)
    b2 = b.reshape(S, -1)
    if a2.stride(0) != b2.stride(0) or a2.stride(1) != 1 or b2.stride(1) != 1:
        a2, b2 = a2.contiguous(), b2.contiguous()
    state = state.to(torch.float32).contiguous()
    _lib.require_cuda(win, state)
    y = torch.empty((S, Hv, Dv), dtype=torch.float32, device=win.device)
    st = torch.empty_like(state)
    mids = torch.empty((max(S - 1, 1), *state.shape), dtype=torch.float32, device=win.device)
    _lib.check(_lib.lib().qmtp_gdn_fused(
        win.data_ptr(), layer.conv1d_weight.data_ptr(), a2.data_ptr(), b2.data_ptr(), a2.stride(0),
        layer.A_log.data_ptr(), layer.dt_bias.data_ptr(), state.data_ptr(), y.data_ptr(), st.data_ptr(),
        mids.data_ptr(), S, Hk, Hv, Dk, Dv, KC, int(bool(snap)), _lib.stream()), "gdn_core")
    return y, st, mids


def gdn_norm_gate(y, z, weight, eps, out=None):
    """y fp32 [S, H, Dv]; z bf16 [..., S, H*Dv] (or [S, H, Dv]) -> out bf16 [1, S, H*Dv]."""
    S, H, Dv = y.shape
    z2 = z.reshape(S, H * Dv)
    if z2.stride(1) != 1:
        z2 = z2.contiguous()
    if out is None:
        out = torch.empty((1, S, H * Dv), dtype=torch.bfloat16, device=y.device)
    _lib.require_cuda(y, weight)
    _lib.check(_lib.lib().qmtp_gdn_norm_gate(y.data_ptr(), z2.data_ptr(), z2.stride(0), weight.data_ptr(),
                                             out.data_ptr(), out.shape[-1], S, H, Dv, float(eps), _lib.stream()),
               "gdn_norm_gate")
    return out


def gdn_middle(layer, qkv, z, a, b, conv_state, state, snap):
    """gdn_fused.py:149: qkv [1,S,C], z [1,S,Hv,Dv], a/b [1,S,Hv], conv_state [1,KC-1,C],
    state [1,Hv,Dv,Dk] -> (out [1,S,Hv*Dv] bf16, conv window [1,S+KC-1,C], state, snapshots).

    One qmtp_gdn_fused_ex call with the gated norm attached: at the decode shape (S <= 4) a single
    launch, otherwise the core and gdn_norm_gate as two."""
    Hk, Hv, Dk, Dv, KC = (layer.num_k_heads, layer.num_v_heads, layer.head_k_dim, layer.head_v_dim,
                          layer.conv_kernel_size)
    win = torch.cat([conv_state, qkv], dim=1).contiguous()
    S, C = win.shape[-2] - (KC - 1), win.shape[-1]
    a2, b2 = a.reshape(S, -1), b.reshape(S, -1)
    if a2.stride(0) != b2.stride(0) or a2.stride(1) != 1 or b2.stride(1) != 1:
        a2, b2 = a2.contiguous(), b2.contiguous()
    z2 = z.reshape(S, Hv * Dv)
    if z2.stride(1) != 1:
        z2 = z2.contiguous()
    state = state.to(torch.float32).contiguous()
    _lib.require_cuda(win, state, layer.norm_weight)
    if not z2.is_cuda:
        raise RuntimeError("qmtp ops run on CUDA tensors only (no CPU fallback)")
    dev = win.device
    y = torch.empty((S, Hv, Dv), dtype=torch.float32, device=dev)
    st = torch.empty_like(state)
    mids = torch.empty((max(S - 1, 1), *state.shape), dtype=torch.float32, device=dev)
    out = torch.empty((1, S, Hv * Dv), dtype=torch.bfloat16, device=dev)
    A = _lib.GdnArgs(conv_src=win.data_ptr(), ld_conv=C, conv_row_off=None, qkv=win.data_ptr() + 2 * (KC - 1) * C,
                     ld_qkv=C, win_out=None, win_out_row_off=None, conv_w=layer.conv1d_weight.data_ptr(),
                     a=a2.data_ptr(), b=b2.data_ptr(), ld_ab=a2.stride(0), A_log=layer.A_log.data_ptr(),
                     dt_bias=layer.dt_bias.data_ptr(), state_in=state.data_ptr(), state_out=st.data_ptr(),
                     state_mid=mids.data_ptr(), ring=None, ring_cur=None, ring_slots=0, y=y.data_ptr(), S=S, Hk=Hk,
                     Hv=Hv, Dk=Dk, Dv=Dv, KC=KC, snap=int(bool(snap)), gate_z=z2.data_ptr(), ld_gate_z=z2.stride(0),
                     gate_w=layer.norm_weight.data_ptr(), gate_out=out.data_ptr(), ld_gate_out=Hv * Dv,
                     gate_eps=float(layer.norm_eps))
    _lib.check(_lib.lib().qmtp_gdn_fused_ex(ctypes.byref(A), _lib.stream()), "gdn_middle")
    return out, win, st, mids
