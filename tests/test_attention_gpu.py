"""Decode attention (libqmtp qmtp_attention) against the C oracle, bit-exact (GPU), over context
lengths that leave the 8 key splits empty, ragged, and longer than one fetch batch."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import ops
from tests._util import randn_bf16, to_np, to_torch

pytestmark = pytest.mark.gpu

_P, _I = ctypes.c_void_p, ctypes.c_int


@pytest.mark.parametrize("pos0", [0, 5, 6, 100, 131, 509, 1020])
def test_attention_bit_exact(pos0, dev):
    from qmtp import _lib

    S, nq, nkv, Dh, max_pos = 3, 16, 4, 256, 1024
    q = randn_bf16((S, nq, Dh), 1 + pos0, 1.0)
    g = randn_bf16((S, nq, Dh), 2 + pos0, 1.0)
    kc = randn_bf16((nkv, max_pos, Dh), 3 + pos0, 1.0)
    vc = randn_bf16((nkv, max_pos, Dh), 4 + pos0, 1.0)
    want = np.empty((S, nq * Dh), np.uint16)
    ops.lib().qo_attention(_P(q.ctypes.data), _P(g.ctypes.data), _P(kc.ctypes.data), _P(vc.ctypes.data),
                           _I(max_pos), _I(S), _I(nq), _I(nkv), _I(Dh), _I(pos0), _P(want.ctypes.data))
    t = [to_torch(a, dev) for a in (q, g, kc, vc)]
    pos = torch.tensor([pos0], dtype=torch.int32, device=dev)
    out = torch.empty((S, nq * Dh), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().qmtp_attention(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(), max_pos,
                                         S, nq, nkv, Dh, pos.data_ptr(), 0, out.data_ptr(), _lib.stream()),
               "attention")
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert np.array_equal(to_np(out), want)


@pytest.mark.parametrize("pos0,S", [(0, 3), (5, 3), (6, 1), (100, 4), (131, 3), (509, 3), (1020, 4)])
def test_attention_fused_bit_exact(pos0, S, dev):
    """qmtp_attention_fused (q/k RMS norms + RoPE + cache writes + attention in one launch), and the
    two-launch form qmtp_attn_prep + qmtp_attention, against the oracle's qo_attn_prep + qo_attention:
    the same q, gate, output and cache contents.  The caches hold random data at the new positions,
    which the fused kernel must not read."""
    from qmtp import _lib

    nq, nkv, Dh, R, max_pos, eps = 16, 4, 256, 64, 1024, 1e-6
    ld = nq * 2 * Dh + 2 * nkv * Dh + 64
    qkv = randn_bf16((S, ld), 11 + pos0, 1.0)
    qn, kn = randn_bf16((Dh,), 12, 0.3), randn_bf16((Dh,), 13, 0.3)
    rng = np.random.default_rng(14 + pos0)
    cos_t = rng.standard_normal((max_pos, R // 2)).astype(np.float32)
    sin_t = rng.standard_normal((max_pos, R // 2)).astype(np.float32)
    kc = randn_bf16((nkv, max_pos, Dh), 15 + pos0, 1.0)
    vc = randn_bf16((nkv, max_pos, Dh), 16 + pos0, 1.0)
    kc_t, vc_t = to_torch(kc, dev), to_torch(vc, dev)
    q = np.empty((S, nq, Dh), np.uint16)
    g = np.empty_like(q)
    L = ops.lib()
    L.qo_attn_prep(_P(qkv.ctypes.data), _I(ld), _I(S), _I(nq), _I(nkv), _I(Dh), _I(R), _P(qn.ctypes.data),
                   _P(kn.ctypes.data), ctypes.c_float(eps), _P(cos_t.ctypes.data), _P(sin_t.ctypes.data), _I(pos0),
                   _P(q.ctypes.data), _P(g.ctypes.data), _P(kc.ctypes.data), _P(vc.ctypes.data), _I(max_pos))
    want = np.empty((S, nq * Dh), np.uint16)
    L.qo_attention(_P(q.ctypes.data), _P(g.ctypes.data), _P(kc.ctypes.data), _P(vc.ctypes.data), _I(max_pos), _I(S),
                   _I(nq), _I(nkv), _I(Dh), _I(pos0), _P(want.ctypes.data))
    t = [to_torch(a, dev) for a in (qkv, qn, kn)]
    ct, st = torch.from_numpy(cos_t).to(dev), torch.from_numpy(sin_t).to(dev)
    pos = torch.tensor([pos0 - 1], dtype=torch.int32, device=dev)  # the position is *pos_ptr + pos_add
    out = torch.empty((S, nq * Dh), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().qmtp_attention_fused(t[0].data_ptr(), ld, S, nq, nkv, Dh, R, t[1].data_ptr(), t[2].data_ptr(),
                                               eps, ct.data_ptr(), st.data_ptr(), pos.data_ptr(), 1, kc_t.data_ptr(),
                                               vc_t.data_ptr(), max_pos, out.data_ptr(), _lib.stream()),
               "attention_fused")
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert np.array_equal(to_np(out), want)
    assert np.array_equal(to_np(kc_t), kc) and np.array_equal(to_np(vc_t), vc)
    # the two-launch form (qmtp_attn_prep, then qmtp_attention) from the same stale caches
    kc2, vc2 = to_torch(randn_bf16((nkv, max_pos, Dh), 15 + pos0, 1.0), dev), to_torch(randn_bf16((nkv, max_pos, Dh), 16 + pos0, 1.0), dev)
    qb = torch.empty((S, nq, Dh), dtype=torch.bfloat16, device=dev)
    gb = torch.empty_like(qb)
    _lib.check(_lib.lib().qmtp_attn_prep(t[0].data_ptr(), ld, S, nq, nkv, Dh, R, t[1].data_ptr(), t[2].data_ptr(), eps,
                                         ct.data_ptr(), st.data_ptr(), pos.data_ptr(), 1, qb.data_ptr(), gb.data_ptr(),
                                         kc2.data_ptr(), vc2.data_ptr(), max_pos, _lib.stream()), "attn_prep")
    out2 = torch.empty_like(out)
    _lib.check(_lib.lib().qmtp_attention(qb.data_ptr(), gb.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), max_pos, S, nq,
                                         nkv, Dh, pos.data_ptr(), 1, out2.data_ptr(), _lib.stream()), "attention")
    torch.cuda.synchronize()
    assert np.array_equal(to_np(qb), q) and np.array_equal(to_np(gb), g)
    assert np.array_equal(to_np(out2), want)
    assert np.array_equal(to_np(kc2), kc) and np.array_equal(to_np(vc2), vc)
