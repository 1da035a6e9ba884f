"""The device exp / log and bf16 activation formulas (csrc/common.cuh) on every bf16 input (GPU).

The reference checks its Metal versions of the gdn_fused.py:22-41 formulas against MLX on all 65,536
bf16 values (tests/test_kernels.py:98-113).  Here the device functions are compared with the C oracle
bit for bit on all of them, and the library's exp / log with CUDA's expf / logf (torch.exp / torch.log
on the GPU) within 2 ulp.  Also: a bounded mbarrier wait that nothing completes gives up and records
the timeout bit instead of hanging."""
import numpy as np
import pytest
import torch

from oracle import ops

pytestmark = pytest.mark.gpu

ALL = np.arange(65536, dtype=np.uint32).astype(np.uint16)


def _dev(fn, dev):
    from qmtp import _lib

    x = torch.from_numpy(ALL.view(np.int16)).to(dev)
    out = torch.empty(ALL.size, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().qmtp_math_eval(fn, x.data_ptr(), ALL.size, out.data_ptr(), _lib.stream()), "math_eval")
    return out.cpu().numpy()


def _same(a, b):
    return np.array_equal(a.view(np.uint32), b.view(np.uint32)) or (
        np.all((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))))


def _ulp(a, b):
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


def test_bf16_formulas_match_oracle_on_every_input(dev):
    ref = ops.bf16_formulas(ALL)
    for fn, key in ((2, "sigmoid"), (3, "silu"), (4, "softplus"), (5, "silu_f32")):
        got = _dev(fn, dev)
        assert _same(got, ref[key]), key


def test_exp_log_match_oracle_and_cuda(dev):
    xf = ops.bf16_to_f32(ALL)
    for fn, oracle_f, torch_f in ((0, ops.exp, torch.exp), (1, ops.log, torch.log)):
        got = _dev(fn, dev)
        assert _same(got, oracle_f(xf))
        cuda = torch_f(torch.from_numpy(xf).to(dev)).cpu().numpy()
        fin = np.isfinite(cuda) & np.isfinite(got) & (cuda != 0)
        assert np.array_equal(np.isnan(got), np.isnan(cuda))
        assert np.array_equal(np.isinf(got), np.isinf(cuda))
        assert _ulp(got[fin], cuda[fin]).max() <= 2, ("exp", "log")[fn]


def test_bounded_wait_gives_up_and_records_timeout(dev):
    from qmtp import _lib

    torch.cuda.synchronize()
    _lib.device_error(clear=True)
    res = torch.full((1,), 7, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().qmtp_wait_selftest(1000, res.data_ptr(), _lib.stream()), "wait_selftest")
    torch.cuda.synchronize()
    assert int(res.item()) == 0
    assert _lib.device_error(clear=True) & 1
    assert _lib.device_error() == 0
