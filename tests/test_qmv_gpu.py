"""qmv kernels (libqmtp, sm_100a) against the C oracle: bit-exact (GPU)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ops
from tests._util import affine_layer, randn_bf16, to_np, to_torch

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"
# (planner mode, through the strided _split entry point): the cost model through both entry points,
# whole tiles only, clusters wherever the shape allows them
MODES = [(0, True), (0, False), (1, True), (2, False)]


@pytest.fixture
def planner():
    """Sets the affine qmv planner mode for a test; restores the cost model afterwards."""
    from qmtp import _lib

    yield _lib.qmv_set_mode
    _lib.qmv_set_mode(0)


def _run_affine(x, wq, s, b, dev, ldy=None, split=True, res=None):
    from qmtp import qmv_kernel

    xt, wt, st, bt = (to_torch(a, dev) for a in (x, wq, s, b))
    rt = None if res is None else to_torch(res, dev)
    if ldy is None and rt is None:
        return to_np(qmv_kernel.qmv_affine(xt, wt, st, bt, split=split))
    out = torch.full((x.shape[0], ldy or wq.shape[0]), 7.0, dtype=torch.bfloat16, device=dev)
    if rt is not None:
        out.copy_(rt)
    qmv_kernel.qmv_affine(xt, wt, st, bt, out=out, res=out if rt is not None else None, split=split)
    return to_np(out)


@pytest.mark.parametrize("K", [512, 1024, 2048, 4096, 8192, 12288])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_qmv_affine_bit_exact(K, M, dev, planner):
    for N in (1, 37, 1000, 4096):
        _, wq, s, b = affine_layer(N, K, seed=K + N)
        x = randn_bf16((M, K), M)
        ref = ops.qmv_affine(x, wq, s, b)
        for mode, split in MODES:
            planner(mode)
            assert np.array_equal(_run_affine(x, wq, s, b, dev, split=split), ref), (K, M, N, mode, split)


def test_qmv_affine_many_shapes_in_turn(dev):
    """Matrices of every shape in turn through one stream (the decoder's use), twice: cluster and
    whole-tile launches of different shapes leave nothing behind that disturbs the next one."""
    from qmtp import qmv_kernel

    cases = []
    for N, K in ((24576, 4096), (1, 2048), (4096, 12288), (37, 4096), (12352, 4096), (5, 8192)):
        _, wq, s, b = affine_layer(N, K, seed=N ^ K)
        x = randn_bf16((3, K), N + 1)
        cases.append((x, wq, s, b, ops.qmv_affine(x, wq, s, b)))
    for _ in range(2):
        for x, wq, s, b, ref in cases:
            xt, wt, st, bt = (to_torch(a, dev) for a in (x, wq, s, b))
            assert np.array_equal(to_np(qmv_kernel.qmv_affine(xt, wt, st, bt)), ref), wq.shape


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_qmv_affine_config1_bit_exact(M, dev):
    _, wq, s, b = affine_layer(12288, 4096, seed=0)
    x = randn_bf16((M, 4096), 1)
    ref = ops.qmv_affine(x, wq, s, b)
    for split in (True, False):
        assert np.array_equal(_run_affine(x, wq, s, b, dev, split=split), ref)


@pytest.mark.parametrize("N,K", [(12352, 4096), (4096, 4096), (4096, 12288), (24576, 4096), (10240, 4096),
                                 (4096, 8192), (777, 12288)])
def test_qmv_affine_decoder_shapes(N, K, dev, planner):
    """The decoder's projection shapes in every planner mode: shared tiles (slice partials finished by
    the first CTA of a cluster through distributed shared memory) give the oracle's bits, repeated
    calls agree."""
    from qmtp import qmv_kernel, _lib

    _, wq, s, b = affine_layer(N, K, seed=N + K)
    x = randn_bf16((3, K), 5)
    ref = ops.qmv_affine(x, wq, s, b)
    xt, wt, st, bt = (to_torch(a, dev) for a in (x, wq, s, b))
    for mode in (0, 1, 2):
        planner(mode)
        for _ in range(2):
            got = to_np(qmv_kernel.qmv_affine(xt, wt, st, bt))
            assert np.array_equal(got, ref), (N, K, mode)
        plan = _lib.qmv_plan(N, K, True)
        T = (N + plan["rows_per_tile"] - 1) // plan["rows_per_tile"]
        assert plan["units"] == T * (K // 512)
        if plan["cluster"] > 1:  # one tile per cluster, or pair mode (2-CTA clusters owning tile runs)
            one_tile = plan["grid"] == T * plan["cluster"] and (K // 512) % plan["cluster"] == 0
            assert one_tile or (plan["cluster"] == 2 and plan["grid"] < 2 * T), plan
        if mode == 2 and N == 4096:
            assert plan["cluster"] > 1, plan
        if mode == 1:
            assert plan["cluster"] == 1 and plan["grid"] <= T
        if mode == 2 and N >= 10240 and K <= 4096:
            assert plan["cluster"] == 2 and plan["grid"] == 148, plan  # pair mode (148 SMs: 74 pairs)


def test_qmv_affine_residual_in_place(dev, planner):
    _, wq, s, b = affine_layer(4096, 12288, seed=3)
    x = randn_bf16((3, 12288), 4)
    res = randn_bf16((3, 4096), 6)
    y = ops.qmv_affine(x, wq, s, b)
    ref = ops.f32_to_bf16(ops.bf16_to_f32(res) + ops.bf16_to_f32(y))
    for mode, split in MODES:
        planner(mode)
        assert np.array_equal(_run_affine(x, wq, s, b, dev, split=split, res=res), ref), mode


def test_qmv_affine_many_rows_and_ldy(dev, planner):
    _, wq, s, b = affine_layer(333, 4096, seed=11)
    x = randn_bf16((9, 4096), 12)
    ref = ops.qmv_affine(x, wq, s, b)
    for mode, split in MODES:
        planner(mode)
        got = _run_affine(x, wq, s, b, dev, ldy=400, split=split)
        assert np.array_equal(got[:, :333], ref)
        assert np.all(got[:, 333:] == ops.f32_to_bf16(np.float32([7.0]))[0])


def test_qmv_affine_extreme_x_bit_exact(dev, planner):
    """Activations over bf16's whole finite range, all-zero groups, subnormal-only groups, and a group
    holding an infinity (its token row becomes NaN, the others are unaffected)."""
    r = np.random.default_rng(31)
    M, K, N = 4, 4096, 700
    sign = r.integers(0, 2, (M, K)).astype(np.uint16) << 15
    man = r.integers(0, 128, (M, K)).astype(np.uint16)
    kind = r.integers(0, 4, (M, K))
    exp = np.where(kind == 0, 0, np.where(kind == 1, r.integers(1, 12, (M, K)),
                   np.where(kind == 2, r.integers(110, 140, (M, K)), r.integers(200, 254, (M, K))))).astype(np.uint16)
    x = sign | (exp << 7) | man
    x[0, 0:64] = 0
    x[1, 512:576] = man[1, 512:576] | sign[1, 512:576]
    x[2, 1000] = 0x7F80
    _, wq, s, b = affine_layer(N, K, seed=8)
    ref = ops.qmv_affine(x, wq, s, b)
    assert np.isnan(ops.bf16_to_f32(ref[2])).all()
    for mode, split in MODES:
        planner(mode)
        assert np.array_equal(_run_affine(x, wq, s, b, dev, split=split), ref), mode


def test_qmv_affine_split_ldx(dev):
    from qmtp import _lib

    N, K, ldx = 1500, 4096, 4096 + 64
    _, wq, s, b = affine_layer(N, K, seed=12)
    xw = randn_bf16((3, ldx), 13)
    ref = ops.qmv_affine(np.ascontiguousarray(xw[:, :K]), wq, s, b)
    xt, wt, st, bt = (to_torch(a, dev) for a in (xw, wq, s, b))
    y = torch.empty((3, N), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().qmtp_qmv_affine_g64_split(xt.data_ptr(), ldx, wt.data_ptr(), st.data_ptr(), bt.data_ptr(),
                                                   y.data_ptr(), None, 3, N, K, N, None, 0, _lib.stream()), "split")
    assert np.array_equal(to_np(y), ref)


def test_qmv_affine_golden(dev):
    d = np.load(G / "qmv.npz")
    assert np.array_equal(_run_affine(d["x"], d["wq"], d["s"], d["b"], dev), d["y"])


def test_qmv_nvfp4_bit_exact(dev):
    from qmtp import qmv_kernel

    d = np.load(G / "qmv.npz")
    got = qmv_kernel.qmv_nvfp4(to_torch(d["x"], dev), to_torch(d["nq"], dev), to_torch(d["ns"], dev))
    assert np.array_equal(to_np(got), d["ny"])
    r = np.random.default_rng(3)
    for M, K, N in ((1, 4096, 500), (3, 4096, 12288), (4, 12288, 64)):
        nq = r.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
        ns = r.integers(54, 70, (N, K // 16), dtype=np.int64).astype(np.uint8)
        x = randn_bf16((M, K), M + K)
        got = qmv_kernel.qmv_nvfp4(to_torch(x, dev), to_torch(nq, dev), to_torch(ns, dev))
        assert np.array_equal(to_np(got), ops.qmv_nvfp4(x, nq, ns)), (M, K, N)


def test_qmv_nvfp4_extreme_x_bit_exact(dev):
    """Activations over bf16's whole finite range (subnormals, tiny and huge normals, zeros): the
    kernel moves the reference's 2^-14 weight scale onto x, which must stay exact everywhere."""
    from qmtp import qmv_kernel

    r = np.random.default_rng(21)
    for M, K, N in ((2, 1024, 300), (1, 4096, 200)):
        sign = r.integers(0, 2, (M, K)).astype(np.uint16) << 15
        man = r.integers(0, 128, (M, K)).astype(np.uint16)
        kind = r.integers(0, 4, (M, K))
        exp = np.where(kind == 0, 0,                                     # subnormal / zero
              np.where(kind == 1, r.integers(1, 12, (M, K)),              # just above 2^-126
              np.where(kind == 2, r.integers(110, 140, (M, K)),           # ordinary magnitudes
                       r.integers(200, 227, (M, K))))).astype(np.uint16)  # up to 2^99
        x = sign | (exp << 7) | man
        nq = r.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
        ns = r.integers(40, 90, (N, K // 16), dtype=np.int64).astype(np.uint8)
        got = qmv_kernel.qmv_nvfp4(to_torch(x, dev), to_torch(nq, dev), to_torch(ns, dev))
        assert np.array_equal(to_np(got), ops.qmv_nvfp4(x, nq, ns)), (M, K, N)


def test_quantize_bit_exact(dev):
    from qmtp import qmv_kernel

    w = randn_bf16((777, 4096), 21, 0.02)
    wq, s, b = qmv_kernel.quantize(to_torch(w, dev))
    rq, rs, rb = ops.quantize_affine(w)
    assert np.array_equal(to_np(wq), rq) and np.array_equal(to_np(s), rs) and np.array_equal(to_np(b), rb)


def test_qmv_rejects_bad_shapes(dev):
    from qmtp import qmv_kernel

    x = torch.zeros(2, 1000, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(8, 125, dtype=torch.int32, device=dev)
    s = torch.zeros(8, 16, dtype=torch.bfloat16, device=dev)
    for split in (True, False):
        with pytest.raises(ValueError):
            qmv_kernel.qmv_affine(x, w, s, s, split=split)
    xb = torch.zeros(2 * 1024 + 1, dtype=torch.bfloat16, device=dev)[1:].view(2, 1024)  # 2-byte offset
    w = torch.zeros(8, 128, dtype=torch.int32, device=dev)
    for split in (True, False):
        with pytest.raises(ValueError):
            qmv_kernel.qmv_affine(xb, w, s, s, split=split)


def test_no_device_error_recorded(dev):
    from qmtp import _lib

    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0


@pytest.mark.parametrize("K", [1024, 4096, 8192])
@pytest.mark.parametrize("M", [1, 3, 4])
def test_qmv_affine_norm_prologue(K, M, dev, planner):
    """The RMSNorm prologue (qmtp_qmv_affine_g64_norm) gives the bits of the oracle's rmsnorm followed
    by its qmv, in every planner mode, with a residual, and for rows over bf16's range (an infinity
    makes its token row NaN)."""
    from oracle import model as om
    from qmtp import qmv_kernel

    r = np.random.default_rng(K + M)
    for N in (37, 4096, 12352):
        _, wq, s, b = affine_layer(N, K, seed=N + K)
        x = randn_bf16((M, K), M + 40, 3.0)
        nw = ops.f32_to_bf16((1.0 + 0.1 * r.standard_normal(K)).astype(np.float32))
        if M == 4:
            x[1] = ops.f32_to_bf16(ops.bf16_to_f32(x[1]) * np.float32(2.0 ** -100))  # tiny row
            x[3, 77] = 0x7F80  # +inf
        res = randn_bf16((M, N), 9)
        xn = om.rmsnorm(x, nw, 1e-6)
        ref = ops.qmv_affine(xn, wq, s, b)
        ref_res = ops.f32_to_bf16(ops.bf16_to_f32(res) + ops.bf16_to_f32(ref))
        xt, wt, st, bt, nt = (to_torch(a, dev) for a in (x, wq, s, b, nw))
        for mode, split in MODES:
            planner(mode)
            got = to_np(qmv_kernel.qmv_affine(xt, wt, st, bt, split=split, norm=(nt, 1e-6)))
            assert np.array_equal(got, ref), (N, mode, split)
            out = to_torch(res, dev)
            qmv_kernel.qmv_affine(xt, wt, st, bt, out=out, res=out, split=split, norm=(nt, 1e-6))
            assert np.array_equal(to_np(out), ref_res), (N, mode, split, "res")
        if M == 4:
            assert np.isnan(ops.bf16_to_f32(ref[3])).all()


@pytest.mark.parametrize("K", [4096, 12288])
@pytest.mark.parametrize("M", [1, 3, 4])
def test_qmv_affine_swiglu_prologue(K, M, dev, planner):
    """The SwiGLU prologue (qmtp_qmv_affine_g64_swiglu) gives the bits of the oracle's swiglu followed by
    its qmv, in every planner mode, with a residual; gate values over a wide range."""
    from qmtp import qmv_kernel

    r = np.random.default_rng(K + 7 * M)
    for N in (37, 4096):
        _, wq, s, b = affine_layer(N, K, seed=N + K + 1)
        gu = ops.f32_to_bf16((r.standard_normal((M, 2 * K)) * np.exp(r.uniform(-4, 3, (M, 2 * K)))).astype(np.float32))
        res = randn_bf16((M, N), 19)
        x = ops.swiglu(gu, K)
        ref = ops.qmv_affine(x, wq, s, b)
        ref_res = ops.f32_to_bf16(ops.bf16_to_f32(res) + ops.bf16_to_f32(ref))
        gt, wt, st, bt = (to_torch(a, dev) for a in (gu, wq, s, b))
        for mode in (0, 1, 2):
            planner(mode)
            assert np.array_equal(to_np(qmv_kernel.qmv_affine_swiglu(gt, wt, st, bt)), ref), (N, mode)
            out = to_torch(res, dev)
            qmv_kernel.qmv_affine_swiglu(gt, wt, st, bt, out=out, res=out)
            assert np.array_equal(to_np(out), ref_res), (N, mode, "res")


@pytest.mark.parametrize("M", [1, 3, 4])
def test_qmv_affine_gated_prologue(M, dev, planner):
    """The GatedDeltaNet output gate in the out-projection's prologue (qmtp_qmv_affine_g64_gated) gives
    the bits of the oracle's gdn_norm_gate followed by its qmv (32 heads of 128, K = 4096), with the
    gate rows strided like the decoder's in_proj output, in every planner mode, with a residual."""
    from qmtp import qmv_kernel

    r = np.random.default_rng(100 + M)
    H, Dv, N = 32, 128, 4096
    K = H * Dv
    _, wq, s, b = affine_layer(N, K, seed=77)
    y = ops.bf16_to_f32(ops.f32_to_bf16((r.standard_normal((M, H, Dv)) * 0.3).astype(np.float32)))
    y[0, 5] *= np.float32(2.0 ** -30)  # a nearly silent head
    zfull = randn_bf16((M, 2 * K + 64), 23)  # the gate sits inside a wider row, as in the decoder
    z = np.ascontiguousarray(zfull[:, 64:64 + K])
    nw = ops.f32_to_bf16((1.0 + 0.2 * r.standard_normal(Dv)).astype(np.float32))
    res = randn_bf16((M, N), 29)
    x = ops.gdn_norm_gate(y, z, nw, 1e-6)
    ref = ops.qmv_affine(x, wq, s, b)
    ref_res = ops.f32_to_bf16(ops.bf16_to_f32(res) + ops.bf16_to_f32(ref))
    yt = torch.from_numpy(y.reshape(M, K).copy()).to(dev)
    zt = to_torch(zfull, dev)[:, 64:64 + K]
    wt, st, bt, nt = (to_torch(a, dev) for a in (wq, s, b, nw))
    for mode in (0, 1, 2):
        planner(mode)
        assert np.array_equal(to_np(qmv_kernel.qmv_affine_gated(yt, zt, nt, 1e-6, wt, st, bt)), ref), mode
        out = to_torch(res, dev)
        qmv_kernel.qmv_affine_gated(yt, zt, nt, 1e-6, wt, st, bt, out=out, res=out)
        assert np.array_equal(to_np(out), ref_res), (mode, "res")


@pytest.mark.parametrize("K", [512, 1024, 2048, 4096])
@pytest.mark.parametrize("M", [1, 3, 4])
def test_qmv_affine_pair_mode_tails(K, M, dev, planner):
    """Pair mode (2-CTA clusters owning runs of tiles; a tile cut in the middle is finished by rank 0
    from rank 1's partials) for every slice count up to 8: tile counts just above the cluster count
    give clusters with one tile (cut in half), two and three tiles, with a residual."""
    from qmtp import qmv_kernel

    for N in (9500, 21000):
        _, wq, s, b = affine_layer(N, K, seed=N + K + M)
        x = randn_bf16((M, K), 3 + M)
        res = randn_bf16((M, N), 4)
        ref = ops.qmv_affine(x, wq, s, b)
        ref_res = ops.f32_to_bf16(ops.bf16_to_f32(res) + ops.bf16_to_f32(ref))
        for mode in (2, 0):
            planner(mode)
            assert np.array_equal(_run_affine(x, wq, s, b, dev), ref), (N, mode)
            assert np.array_equal(_run_affine(x, wq, s, b, dev, res=res), ref_res), (N, mode, "res")
