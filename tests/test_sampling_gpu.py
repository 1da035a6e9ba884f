"""Exact speculative sampling on the GPU (libqmtp qmtp_sample) against the C oracle (qo_sample):
identical decisions on random candidate rows, and identical sampled MTP streams (GPU)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import ops
from tests._util import to_np, to_torch
from tests.test_model_oracle import greedy_overrides, prompt

pytestmark = pytest.mark.gpu


def _call(idx, fine, drafts, sp, V, seed, ctr, dev, first_row=-1):
    from qmtp import _lib

    R, K = idx.shape
    ctrl = torch.zeros(_lib.CTRL_SIZE, dtype=torch.int32, device=dev)
    lo, hi = seed & 0xFFFFFFFF, seed >> 32
    ctrl[_lib.CTRL["SEED_LO"]] = lo - (1 << 32) if lo >= 1 << 31 else lo
    ctrl[_lib.CTRL["SEED_HI"]] = hi - (1 << 32) if hi >= 1 << 31 else hi
    ctrl[_lib.CTRL["RNG"]] = ctr
    it, ft = to_torch(idx, dev), to_torch(fine, dev)
    dt = torch.tensor(list(drafts) if drafts else [0], dtype=torch.int32, device=dev)
    out = torch.full((R,), -7, dtype=torch.int32, device=dev)
    args = _lib.SamplingArgs(*sp)
    _lib.check(_lib.lib().qmtp_sample(it.data_ptr(), ft.data_ptr(), K, K, dt.data_ptr(), len(drafts or [0]),
                                      first_row, ctypes.byref(args), V, ctrl.data_ptr(), out.data_ptr(),
                                      _lib.stream()), "sample")
    torch.cuda.synchronize()
    assert int(ctrl[_lib.CTRL["RNG"]]) == ctr + 1
    return to_np(out).view(np.int32)


@pytest.mark.parametrize("K", [64, 160, 256, 1024, 2048])
@pytest.mark.parametrize("sp", [(0.8, 0, 1.0, 0.0), (1.0, 0, 0.9, 0.0), (0.6, 20, 1.0, 0.05), (1.2, 40, 0.95, 0.01),
                                (0.9, 400, 0.97, 0.0)])
def test_sample_matches_oracle(K, sp, dev):
    rng = np.random.default_rng(K + int(10 * sp[0]))
    V = 248320
    T, top_k, top_p, min_p = sp
    for trial in range(12):
        idx = np.stack([rng.permutation(V)[:K] for _ in range(3)]).astype(np.int32)
        fine = ops.f32_to_bf16((rng.standard_normal((3, K)) * 2).astype(np.float32))
        fine[:, rng.integers(0, K, 4)] = fine[:, :1]  # ties in the logits
        drafts = [int(idx[0, rng.integers(0, 4)]), int(idx[1, rng.integers(0, K)]) if trial % 3 else 123]
        seed = int(rng.integers(0, 2 ** 63))
        ctr = int(rng.integers(0, 2 ** 31))
        got = _call(idx, fine, drafts, sp, V, seed, ctr, dev)
        n_acc, want = ops.sample(idx, fine, drafts, temperature=T, top_k=top_k, top_p=top_p, min_p=min_p, V=V,
                                 seed=seed, ctr=ctr)
        assert list(got[:n_acc + 1]) == want, (trial, list(got), want)
        assert all(int(v) == -7 for v in got[n_acc + 1:])
        row = int(rng.integers(0, 3))
        got1 = _call(idx, fine, None, sp, V, seed, ctr, dev, first_row=row)
        want1 = ops.sample(idx[row:row + 1], fine[row:row + 1], None, temperature=T, top_k=top_k, top_p=top_p,
                           min_p=min_p, V=V, seed=seed, ctr=ctr, first_row=0)
        assert int(got1[row]) == want1


def test_sample_rejects_bad_arguments(dev):
    from qmtp import _lib

    L = _lib.lib()
    z = torch.zeros(300, dtype=torch.int32, device=dev)
    for sp, K in [((0.0, 0, 1.0, 0.0), 64), ((1.0, 0, 0.0, 0.0), 64), ((1.0, -1, 1.0, 0.0), 64),
                  ((1.0, 0, 1.0, 0.0), 2049)]:
        a = _lib.SamplingArgs(*sp)
        rc = L.qmtp_sample(z.data_ptr(), z.data_ptr(), K, K, z.data_ptr(), 2, -1, ctypes.byref(a), 1000,
                           z.data_ptr(), z.data_ptr(), _lib.stream())
        assert rc < 0


@pytest.fixture(scope="module")
def small_pair():
    from qmtp import model as qm

    Wn = om.synthetic_weights(om.SMALL, seed=0)
    return om.OracleModel(om.SMALL, Wn), qm.from_numpy(Wn)


@pytest.mark.parametrize("sp,use_graph,override", [
    (dict(temperature=0.8, top_k=0, top_p=0.95, min_p=0.02, seed=11), True, False),   # 256 candidates
    (dict(temperature=1.0, top_k=20, seed=5), False, False),                          # 64 candidates
    (dict(temperature=0.7, top_k=40, top_p=0.9, seed=3), True, False),                # 160 candidates
    (dict(temperature=0.005, top_k=0, top_p=1.0, seed=9), True, True),                # drafts often accepted
    (dict(temperature=0.9, top_k=512, top_p=0.97, seed=13), True, False),             # 2048 candidates
    (dict(temperature=1.1, top_k=100, seed=17), False, False),                        # 400 candidates
])
def test_sampled_stream_matches_oracle(small_pair, sp, use_graph, override):
    from qmtp import model as qm
    from qmtp.mtp import MTPDecoder, Sampling, decode_mtp

    orc, W = small_pair
    p = prompt(37, seed=4)
    ov = (lambda: greedy_overrides(orc.generate_greedy(p, 40), om.SMALL.vocab)) if override else (lambda: None)
    s = Sampling(**sp)
    ref, rst = orc.generate_mtp(p, 40, sampling=s, draft_override=ov())
    dec = MTPDecoder(qm.SMALL, W, k=2, max_tokens=300, sampling=s)
    out, st = decode_mtp(dec, p, 40, use_graph=use_graph, draft_override=ov())
    assert out == ref
    assert st["acept"] == rst["acept"]
    if override:
        assert rst["acept"][0] > 0.3  # the drafts were accepted often enough to cover the accept path
