"""MoE kernels (libqmtp, tcgen05) against the C oracle (GPU).

Bit-exact: the fp4 quantizer (codes and scales) and the router (expert ids and fp32 weights).
Tolerance for the expert FFN output: the weights and x enter the tensor core exactly (bf16), the
products accumulate in fp32 and h is carried as hi + lo bf16 (about 16 significant bits), so the
only sizeable difference to the oracle's double-precision value is the final rounding to bf16 (half
an ulp, 2^-9 relative).  Bound used per element: |y - y_ref| <= 2^-8 |y_ref| + 1e-4 max|y_ref|;
and the reference's own metric (bench_moe.py:120-125) max|y - y_ref| / max|y_ref| <= 4e-3."""
import math

import numpy as np
import pytest
import torch

from oracle import ops
from tests._util import randn_bf16, rng, to_np, to_torch
from tests.test_moe_oracle import make_layer

pytestmark = pytest.mark.gpu


def _check(y_gpu_bits, yf_ref):
    y = ops.bf16_to_f32(y_gpu_bits).astype(np.float64)
    ref = yf_ref.astype(np.float64)
    m = np.abs(ref).max()
    err = np.abs(y - ref)
    assert np.all(err <= 2.0 ** -8 * np.abs(ref) + 1e-4 * m), (err.max(), m)
    assert err.max() / m <= 4e-3
    return err.max() / m


@pytest.mark.parametrize("mode", ["mxfp4", "nvfp4"])
def test_quantizer_bit_exact(mode, dev):
    from qmtp import moe

    G = 32 if mode == "mxfp4" else 16
    w = randn_bf16((3, 96, 512), 2, 0.02)
    flat = w.reshape(-1, 512)
    flat[0, :G] = 0
    flat[1, :G] = ops.f32_to_bf16(np.float32(1e-38))
    flat[2, :G] = ops.f32_to_bf16(np.float32(3e4))
    flat[3, :8] = ops.f32_to_bf16(np.array([6, -2.5, 0.25, 0.75, 1.25, 1.75, 3.5, 5.0], np.float32))
    flat[4, :G] = ops.f32_to_bf16(-np.ones(G, np.float32) * 0.0)
    wq, s = ops.quantize_fp4(w, mode)
    gq, gs = moe.quantize(to_torch(w, dev), mode)
    assert np.array_equal(to_np(gq), wq)
    assert np.array_equal(gs.cpu().numpy(), s)


def test_router_bit_exact(dev):
    from qmtp import moe

    lg = rng(9).standard_normal((256, 64)).astype(np.float32)
    lg[0, 3] = lg[0, 40] = 3.0
    lg[1, 7] = np.nan
    idx, sc = ops.moe_route(lg, 6, 2, 1.0)
    gi, gs = moe.route(torch.from_numpy(lg).to(dev), 6, 2, 1.0)
    assert np.array_equal(gi.cpu().numpy(), idx)
    assert np.array_equal(gs.cpu().numpy().view(np.uint32), sc.view(np.uint32))


def _run(x, layer, idx, sc, mode, limit, dev):
    from qmtp import moe

    (wg, sg), (wu, su), (wd, sd) = layer
    t = [to_torch(a, dev) for a in (x, wg, sg, wu, su, wd, sd)]
    y = moe.moe_decode(t[0], *t[1:], torch.from_numpy(idx).to(dev), torch.from_numpy(sc).to(dev), limit=limit,
                       mode=mode)
    torch.cuda.synchronize()
    from qmtp import _lib
    assert _lib.device_error() == 0
    return to_np(y)


@pytest.mark.parametrize("mode", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("limit", [None, 0.02])
def test_moe_small(mode, limit, dev):
    E, H, I, T = 10, 256, 384, 100   # 8 routed + 2 shared; shared experts get 100 entries = 2 tiles
    layer = make_layer(E, H, I, mode, 21)
    x = randn_bf16((T, H), 5)
    idx, sc = ops.moe_route(rng(6).standard_normal((T, E - 2)).astype(np.float32), 4, 2, 1.5)
    y = _run(x, layer, idx, sc, mode, limit, dev)
    _, yf = ops.moe(x, *[a for m in layer for a in m], idx, sc, mode, limit)
    _check(y, yf)


def test_moe_ragged_routing(dev):
    # hand-made routing: empty experts, an expert with 130 entries (3 tiles, last one ragged),
    # duplicate experts in one token's slots, tiles of 1 token
    E, H, I, T, S = 7, 128, 256, 130, 3
    layer = make_layer(E, H, I, "mxfp4", 31)
    x = randn_bf16((T, H), 8)
    idx = np.zeros((T, S), np.int32)
    idx[:, 0] = 2
    idx[:, 1] = np.where(np.arange(T) % 2 == 0, 4, 2)
    idx[:, 2] = 6
    idx[0, 2] = 5
    idx[1, 2] = 0
    sc = rng(3).random((T, S)).astype(np.float32)
    y = _run(x, layer, idx, sc, "mxfp4", None, dev)
    _, yf = ops.moe(x, *[a for m in layer for a in m], idx, sc, "mxfp4", None)
    _check(y, yf)


def test_reference_batch1_call(dev):
    # moe_decode(x [H], ..., idx [NE], scores [NE]) exactly as kernels.py:133 is called
    E, H, I = 9, 256, 256
    layer = make_layer(E, H, I, "mxfp4", 41)
    x = randn_bf16((H,), 9, 0.5)
    idx = np.array([3, 0, 7, 5, 1, 2, 8], np.int32)
    s6 = np.exp(rng(1).standard_normal(6)).astype(np.float32)
    sc = np.concatenate([s6 / s6.sum() * 1.5, [1.0]]).astype(np.float32)
    y = _run(x, layer, idx, sc, "mxfp4", 10.0, dev)
    assert y.shape == (H,)
    _, yf = ops.moe(x.reshape(1, H), *[a for m in layer for a in m], idx.reshape(1, -1), sc.reshape(1, -1),
                    "mxfp4", 10.0)
    _check(y.reshape(1, H), yf)


@pytest.mark.parametrize("mode", ["mxfp4", "nvfp4"])
def test_moe_config5_full_size(mode, dev):
    """Config 5: 256 tokens, 64 routed + 2 shared experts, top-6, H 2048, I 1408, plain SwiGLU."""
    from qmtp import moe

    E, H, I, T = 66, 2048, 1408, 256
    torch.manual_seed(5)
    wts = []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = (torch.randn(shape, device=dev) * 0.02).to(torch.bfloat16)
        wts.extend(moe.quantize(w, mode))
    x = torch.randn((T, H), device=dev).to(torch.bfloat16)
    logits = torch.randn((T, 64), device=dev)
    idx, sc = moe.route(logits, 6, 2)
    y = moe.moe_decode(x, *wts, idx, sc, limit=None, mode=mode)
    torch.cuda.synchronize()
    np_w = [to_np(t) if t.dtype != torch.uint8 else t.cpu().numpy() for t in wts]
    _, yf = ops.moe(to_np(x), *np_w, idx.cpu().numpy(), sc.cpu().numpy(), mode, None)
    rel = _check(to_np(y), yf)
    assert math.isfinite(rel)
