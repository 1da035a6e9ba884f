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


@pytest.fixture(params=[0, 1], ids=["auto", "general"])
def gdn_mode(request):
    """Kernel choice of qmtp_gdn_fused_ex: 0 = the decode-shape kernel where it applies, 1 = always the
    general kernel (+ a separate gated-norm launch)."""
    from qmtp import _lib

    prev = _lib.lib().qmtp_gdn_set_mode(request.param)
    yield request.param
    _lib.lib().qmtp_gdn_set_mode(prev)


@pytest.mark.parametrize("S", [1, 3, 4, 16])
def test_gdn_core_bit_exact(S, gdn_mode, dev):
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


@pytest.mark.parametrize("S", [1, 3, 4, 5])
def test_gdn_middle_and_norm_gate(S, gdn_mode, dev):
    """gdn_middle = core + gated norm in one qmtp_gdn_fused_ex call: one launch with the gated norm
    over an 8-CTA cluster at S <= 4 (mode auto), two launches otherwise."""
    from qmtp.gdn_fused import gdn_middle

    d = fused_inputs(S=S, seed=40 + S)
    r = np.random.default_rng(41 + S)
    w = ops.f32_to_bf16((1 + 0.2 * r.standard_normal(128)).astype(np.float32))
    z = ops.f32_to_bf16(r.standard_normal((S, 32 * 128)).astype(np.float32))
    L = _layer(d, dev, w)
    win = to_torch(d["win"], dev)[None]
    out, wout, st, mids = gdn_middle(L, win[:, 3:], to_torch(z, dev).view(1, S, 32, 128),
                                     to_torch(d["a"], dev)[None], to_torch(d["b"], dev)[None], win[:, :3],
                                     to_torch(d["state"], dev)[None], snap=True)
    ry, rso, rsm = ops.gdn_fused(**d)
    assert np.array_equal(to_np(wout)[0], d["win"])
    assert np.array_equal(to_np(out)[0], ops.gdn_norm_gate(ry, z, w, 1e-6))
    assert np.array_equal(to_np(st)[0], rso)
    if S > 1:
        assert np.array_equal(to_np(mids)[:, 0], rsm)


@pytest.mark.parametrize("S,gate,preload", [(3, False, 0), (3, True, 0), (3, True, 1), (1, True, 1), (2, True, 0),
                                             (4, True, 1), (6, True, 1)])
def test_gdn_ring_mode_matches_explicit(S, gate, preload, gdn_mode, dev):
    """Device-indexed state ring + conv rows at a device offset + next-window output written at a
    device row offset inside the same buffer (the decoder's layout), with and without the gated norm
    (strided z and output rows, as the decoder passes them), with the previous step's state read
    before or after the dependency wait (preload; the launch before is a torch copy here)."""
    from qmtp import _lib

    d = fused_inputs(S=S, seed=50 + S)
    Hk, Hv, D, KC = d["Hk"], d["Hv"], d["Dk"], d["KC"]
    C = 2 * Hk * D + Hv * D
    R_ = KC - 1 + S
    r = np.random.default_rng(51 + S)
    buf = ops.f32_to_bf16(r.standard_normal((2 * R_, C)).astype(np.float32))  # two window halves
    off, wrow = R_ + min(2, S), 0          # conv rows from the second half, next window into the first
    win = np.concatenate([buf[off:off + KC - 1], d["win"][KC - 1:]], axis=0)
    ry, rso, rsm = ops.gdn_fused(**dict(d, win=win))
    slots, cur = S + 1, S
    ring = torch.zeros((slots, Hv, D, D), dtype=torch.float32, device=dev)
    ring[cur] = to_torch(d["state"], dev)
    ctrl = torch.tensor([cur, off, wrow], dtype=torch.int32, device=dev)
    buf_t = to_torch(buf, dev)
    ldp = C + 2 * Hv * D + 64                   # qkv rows inside a wider projection row
    proj = torch.zeros((S, ldp), dtype=torch.bfloat16, device=dev)
    proj[:, :C] = to_torch(d["win"][KC - 1:], dev)
    z = ops.f32_to_bf16(r.standard_normal((S, Hv * D)).astype(np.float32))
    proj[:, C:C + Hv * D] = to_torch(z, dev)
    w = ops.f32_to_bf16((1 + 0.2 * r.standard_normal(D)).astype(np.float32))
    w_t = to_torch(w, dev)
    out = torch.zeros((S, Hv * D + 32), dtype=torch.bfloat16, device=dev)
    y = torch.empty((S, Hv, D), dtype=torch.float32, device=dev)
    a_t, b_t = to_torch(d["a"], dev), to_torch(d["b"], dev)
    cw, al, dtb = to_torch(d["conv_w"], dev), to_torch(d["A_log"], dev), to_torch(d["dt_bias"], dev)
    A = _lib.GdnArgs(conv_src=buf_t.data_ptr(), ld_conv=C, conv_row_off=ctrl.data_ptr() + 4, qkv=proj.data_ptr(),
                     ld_qkv=ldp, win_out=buf_t.data_ptr(), win_out_row_off=ctrl.data_ptr() + 8,
                     conv_w=cw.data_ptr(), a=a_t.data_ptr(), b=b_t.data_ptr(),
                     ld_ab=Hv, A_log=al.data_ptr(), dt_bias=dtb.data_ptr(), state_in=None, state_out=None,
                     state_mid=None, ring=ring.data_ptr(), ring_cur=ctrl.data_ptr(), ring_slots=slots,
                     y=y.data_ptr(), S=S, Hk=Hk, Hv=Hv, Dk=D, Dv=D, KC=KC, snap=1, preload=preload)
    if gate:
        A.gate_z, A.ld_gate_z = proj.data_ptr() + 2 * C, ldp
        A.gate_w, A.gate_out, A.ld_gate_out, A.gate_eps = w_t.data_ptr(), out.data_ptr(), out.shape[1], 1e-6
    _lib.check(_lib.lib().qmtp_gdn_fused_ex(ctypes.byref(A), _lib.stream()), "gdn_fused_ex")
    assert np.array_equal(to_np(y), ry)
    Rg = to_np(ring)
    for t in range(S - 1):
        assert np.array_equal(Rg[(cur + 1 + t) % slots], rsm[t])
    assert np.array_equal(Rg[(cur + S) % slots], rso)
    B = to_np(buf_t)
    assert np.array_equal(B[wrow:wrow + R_], win)
    assert np.array_equal(B[R_:], buf[R_:])  # the conv half is untouched
    if gate:
        o = to_np(out)
        assert np.array_equal(o[:, :Hv * D], ops.gdn_norm_gate(ry, z, w, 1e-6))
        assert not o[:, Hv * D:].any()
