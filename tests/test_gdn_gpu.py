"""GatedDeltaNet kernels (libqmtp, sm_100a) against the C oracle: bit-exact (GPU)."""
import ctypes
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ops
from tests._util import to_np, to_torch
from tests.test_gdn_oracle import config2_inputs, fused_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,B,seed", [(3, 1, 0), (4, 1, 1), (1, 1, 2), (5, 2, 3)])
def test_gated_delta_snapshot_bit_exact(T, B, seed, dev):
    from qmtp.gdn_kernel import gated_delta_snapshot

    q, k, v, g, beta, state = config2_inputs(T=T, B=B, seed=seed)
    y, so, sm = gated_delta_snapshot(*(to_torch(a, dev) for a in (q, k, v, g, beta, state)))
    ry, rso, rsm = ops.gdn_step(q, k, v, g, beta, state)
    assert np.array_equal(to_np(y), ry)
    assert np.array_equal(to_np(so), rso)
    if T > 1:
        assert np.array_equal(to_np(sm), rsm)


def _layer(d, dev, norm_w=None, eps=1e-6):
    return SimpleNamespace(num_k_heads=d["Hk"], num_v_heads=d["Hv"], head_k_dim=d["Dk"], head_v_dim=d["Dv"],
                           conv_kernel_size=d["KC"], conv1d_weight=to_torch(d["conv_w"], dev),
                           A_log=to_torch(d["A_log"], dev), dt_bias=to_torch(d["dt_bias"], dev),
                           norm_weight=None if norm_w is None else to_torch(norm_w, dev), norm_eps=eps)


@pytest.mark.parametrize("S", [1, 3, 16])
def test_gdn_core_bit_exact(S, dev):
    from qmtp.gdn_fused import gdn_core

    d = fused_inputs(S=S, seed=20 + S)
    L = _layer(d, dev)
    y, so, sm = gdn_core(L, to_torch(d["win"], dev)[None], to_torch(d["a"], dev)[None], to_torch(d["b"], dev)[None],
                         to_torch(d["state"], dev)[None], snap=True)
    ry, rso, rsm = ops.gdn_fused(**d)
    assert np.array_equal(to_np(y), ry)
    assert np.array_equal(to_np(so)[0], rso)
    if S > 1:
        assert np.array_equal(to_np(sm)[:, 0], rsm)


def test_gdn_middle_and_norm_gate(dev):
    from qmtp.gdn_fused import gdn_middle

    d = fused_inputs(S=3, seed=40)
    r = np.random.default_rng(41)
    w = ops.f32_to_bf16((1 + 0.2 * r.standard_normal(128)).astype(np.float32))
    z = ops.f32_to_bf16(r.standard_normal((3, 32 * 128)).astype(np.float32))
    L = _layer(d, dev, w)
    win = to_torch(d["win"], dev)[None]
    out, wout, st, mids = gdn_middle(L, win[:, 3:], to_torch(z, dev).view(1, 3, 32, 128),
                                     to_torch(d["a"], dev)[None], to_torch(d["b"], dev)[None], win[:, :3],
                                     to_torch(d["state"], dev)[None], snap=True)
    ry, rso, rsm = ops.gdn_fused(**d)
    assert np.array_equal(to_np(wout)[0], d["win"])
    assert np.array_equal(to_np(out)[0], ops.gdn_norm_gate(ry, z, w, 1e-6))
    assert np.array_equal(to_np(st)[0], rso)


def test_gdn_ring_mode_matches_explicit(dev):
    """Device-indexed state ring + conv rows at a device offset + next-window output."""
    from qmtp import _lib

    d = fused_inputs(S=3, seed=50)
    Hk, Hv, D, KC = d["Hk"], d["Hv"], d["Dk"], d["KC"]
    C = 2 * Hk * D + Hv * D
    r = np.random.default_rng(51)
    prev = ops.f32_to_bf16(r.standard_normal((KC - 1 + 3, C)).astype(np.float32))  # previous window, 6 rows
    off = 2
    win = np.concatenate([prev[off:off + KC - 1], d["win"][KC - 1:]], axis=0)
    ry, rso, rsm = ops.gdn_fused(**dict(d, win=win))
    slots, cur = 4, 3
    ring = torch.zeros((slots, Hv, D, D), dtype=torch.float32, device=dev)
    ring[cur] = to_torch(d["state"], dev)
    ctrl = torch.tensor([cur, off], dtype=torch.int32, device=dev)
    prev_t = to_torch(prev, dev)
    qkv_t = to_torch(d["win"][KC - 1:], dev)
    win_out = torch.zeros((KC - 1 + 3, C), dtype=torch.bfloat16, device=dev)
    y = torch.empty((3, Hv, D), dtype=torch.float32, device=dev)
    a_t, b_t = to_torch(d["a"], dev), to_torch(d["b"], dev)
    cw, al, dtb = to_torch(d["conv_w"], dev), to_torch(d["A_log"], dev), to_torch(d["dt_bias"], dev)
    A = _lib.GdnArgs(conv_src=prev_t.data_ptr(), ld_conv=C, conv_row_off=ctrl.data_ptr() + 4, qkv=qkv_t.data_ptr(),
                     ld_qkv=C, win_out=win_out.data_ptr(), conv_w=cw.data_ptr(), a=a_t.data_ptr(), b=b_t.data_ptr(),
                     ld_ab=Hv, A_log=al.data_ptr(), dt_bias=dtb.data_ptr(), state_in=None, state_out=None,
                     state_mid=None, ring=ring.data_ptr(), ring_cur=ctrl.data_ptr(), ring_slots=slots,
                     y=y.data_ptr(), S=3, Hk=Hk, Hv=Hv, Dk=D, Dv=D, KC=KC, snap=1)
    _lib.check(_lib.lib().qmtp_gdn_fused_ex(ctypes.byref(A), _lib.stream()), "gdn_fused_ex")
    assert np.array_equal(to_np(y), ry)
    R = to_np(ring)
    assert np.array_equal(R[(cur + 1) % slots], rsm[0]) and np.array_equal(R[(cur + 2) % slots], rsm[1])
    assert np.array_equal(R[(cur + 3) % slots], rso)
    assert np.array_equal(to_np(win_out), win)
