"""qmtp_lmhead2_noalloc: the two-stage head without a workspace argument, for callers that cannot
allocate device memory (it runs on a static scratch area inside the library).  Called through the
C ABI twice in a row; each call must reproduce qmtp_lmhead2 (which gets a caller-allocated
workspace) bit for bit, as the parity tests of the head require.  Collected last on purpose."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _head_inputs(V, D, dev, seed):
    from qmtp.qmv_kernel import quantize

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    W = (torch.randn(V, D, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wq, s, b = quantize(W)
    return W, wq, s, b


def _run(fn_name, h, W, wq, s, b, k, dev, ws=None):
    from qmtp import _lib

    L = _lib.lib()
    M, D = h.shape
    V = W.shape[0]
    idx = torch.full((M, k), -1, dtype=torch.int32, device=dev)
    fine = torch.zeros((M, k), dtype=torch.bfloat16, device=dev)
    amax = torch.full((M,), -1, dtype=torch.int32, device=dev)
    if fn_name == "qmtp_lmhead2":
        rc = L.qmtp_lmhead2(h.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), W.data_ptr(), M, V, D, k,
                            idx.data_ptr(), fine.data_ptr(), amax.data_ptr(), None, ws.data_ptr(), ws.numel(),
                            _lib.stream())
    else:
        rc = L.qmtp_lmhead2_noalloc(h.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), W.data_ptr(), M, V, D,
                                    k, idx.data_ptr(), fine.data_ptr(), amax.data_ptr(), _lib.stream())
    _lib.check(rc, fn_name)
    torch.cuda.synchronize()
    return idx.cpu(), fine.cpu().view(torch.int16), amax.cpu()


def test_noalloc_head_matches_workspace_head_twice(dev):
    from qmtp import _lib

    V, D, k = 248320, 4096, 64
    W, wq, s, b = _head_inputs(V, D, dev, 7)
    ws = torch.empty(_lib.lib().qmtp_lmhead2_workspace(3, V, k), dtype=torch.uint8, device=dev)
    for call, (M, seed) in enumerate(((3, 11), (2, 12))):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        h = torch.randn(M, D, generator=g, device=dev).to(torch.bfloat16)
        ref = _run("qmtp_lmhead2", h, W, wq, s, b, k, dev, ws)
        got = _run("qmtp_lmhead2_noalloc", h, W, wq, s, b, k, dev)
        for r, x in zip(ref, got):
            assert torch.equal(r, x), f"call {call}"
        assert (got[0] >= 0).all() and (got[2] >= 0).all()


def test_noalloc_head_largest_request_matches_workspace_head(dev):
    """The largest request the scratch is sized for (M = 4, V = 262144, k = 64) against the
    workspace head, bit for bit, twice; one vocabulary row more is refused."""
    from qmtp import _lib

    V, D, k = 262144, 512, 64
    W, wq, s, b = _head_inputs(V, D, dev, 5)
    ws = torch.empty(_lib.lib().qmtp_lmhead2_workspace(4, V, k), dtype=torch.uint8, device=dev)
    for seed in (21, 22):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        h = torch.randn(4, D, generator=g, device=dev).to(torch.bfloat16)
        ref = _run("qmtp_lmhead2", h, W, wq, s, b, k, dev, ws)
        got = _run("qmtp_lmhead2_noalloc", h, W, wq, s, b, k, dev)
        for r, x in zip(ref, got):
            assert torch.equal(r, x), seed
    W1, wq1, s1, b1 = _head_inputs(V + 1, D, dev, 6)
    with pytest.raises(ValueError):
        _run("qmtp_lmhead2_noalloc", h, W1, wq1, s1, b1, k, dev)
    assert _lib.device_error() == 0


def test_noalloc_head_rejects_sizes_beyond_its_scratch(dev):
    from qmtp import _lib

    W, wq, s, b = _head_inputs(1024, 1024, dev, 3)
    h = torch.zeros(5, 1024, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        _run("qmtp_lmhead2_noalloc", h, W, wq, s, b, 64, dev)
    with pytest.raises(ValueError):
        _run("qmtp_lmhead2_noalloc", h[:1], W, wq, s, b, 128, dev)
    assert _lib.device_error() == 0
