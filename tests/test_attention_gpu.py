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
