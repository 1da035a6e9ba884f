"""GatedDeltaNet decode step with per-token state snapshots -- the gdn_kernel.py surface.

Reference: gdn_kernel.py:75-88 ``gated_delta_snapshot(q, k, v, g, beta, state)``.  Runs the sm_100a
kernel of libqmtp (csrc/gdn.cu): one warp per (batch, value head, dv row), the 128-float state row
held in registers across the T tokens, the state after tokens 1..T-1 written out for rollback.
"""
from __future__ import annotations

import torch

from . import _lib


def gated_delta_snapshot(q, k, v, g, beta, state):
    """q, k: [B,T,Hk,Dk] bf16; v: [B,T,Hv,Dv] bf16; g, beta: [B,T,Hv] (any float dtype, used as fp32);
    state: [B,Hv,Dv,Dk] fp32.  Returns (y bf16 [B,T,Hv,Dv], final state, states after tokens
    1..T-1 as [max(T-1,1),B,Hv,Dv,Dk])."""
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2:]
    g = g.to(torch.float32).contiguous()
    beta = beta.to(torch.float32).contiguous()
    state = state.to(torch.float32).contiguous()
    _lib.require_cuda(q, k, v, g, beta, state)
    y = torch.empty((B, T, Hv, Dv), dtype=torch.bfloat16, device=q.device)
    st = torch.empty_like(state)
    mids = torch.empty((max(T - 1, 1), *state.shape), dtype=torch.float32, device=q.device)
    _lib.check(_lib.lib().qmtp_gdn_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
                                        state.data_ptr(), y.data_ptr(), st.data_ptr(), mids.data_ptr(), B, T, Hk,
                                        Hv, Dk, Dv, _lib.stream()), "gated_delta_snapshot")
    return y, st, mids
