"""The sampling oracle (C qo_sample, qo_philox4x32_10) on the CPU: Philox known-answer vectors, and
the exactness of speculative sampling (engine.py:91-152): whatever the draft, the first emitted token
is distributed as Engine._dist's p."""
import numpy as np
import pytest

from oracle import ops


def test_philox_known_answers():
    """Philox4x32-10 test vectors of the Random123 distribution (counter, key -> output)."""
    cases = [([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
             ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
             ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
              [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1])]
    for ctr, key, want in cases:
        assert [int(v) for v in ops.philox4x32_10(ctr, key)] == want


def _dist64(logits, T, top_k=0, top_p=1.0, min_p=0.0):
    """Engine._dist in float64 over candidate logits (independent restatement): prob per candidate."""
    order = sorted(range(len(logits)), key=lambda j: (-logits[j], j))
    lp = np.full(len(logits), -np.inf)
    keep = order[:top_k] if top_k > 0 else order
    z = np.array([logits[j] / T for j in keep])
    z = z - (z.max() + np.log(np.exp(z - z.max()).sum()))
    n = len(keep)
    if top_p < 1.0:
        q = np.exp(z)
        excl = np.cumsum(q) - q
        n = int(np.argmax(~(excl < top_p))) if not np.all(excl < top_p) else n
    if min_p > 0:
        n = min(n, int(np.sum(z[:n] >= z[0] + np.log(min_p))))
    z = z[:n] - (z[0] + np.log(np.exp(z[:n] - z[0]).sum()))
    for j, v in zip(keep[:n], z):
        lp[j] = v
    return np.exp(lp)


CASES = [dict(T=0.7), dict(T=1.0, top_p=0.8), dict(T=1.3, top_k=5), dict(T=0.9, min_p=0.15),
         dict(T=1.0, top_k=6, top_p=0.9, min_p=0.02)]


@pytest.mark.parametrize("case", CASES)
def test_speculative_sampling_is_exact(case):
    rng = np.random.default_rng(1)
    K = 12
    logits = ops.f32_to_bf16((rng.standard_normal(K) * 1.5).astype(np.float32))
    ids = rng.permutation(1000)[:K].astype(np.int32)
    lf = ops.bf16_to_f32(logits).astype(np.float64)
    p = _dist64(lf, case["T"], case.get("top_k", 0), case.get("top_p", 1.0), case.get("min_p", 0.0))
    idx = np.stack([ids, ids])
    fine = np.stack([logits, logits])
    kw = dict(temperature=case["T"], top_k=case.get("top_k", 0), top_p=case.get("top_p", 1.0),
              min_p=case.get("min_p", 0.0), V=1000, seed=0x1234_5678_9ABC)
    N = 12000
    for draft in (int(ids[np.argmax(p)]), int(ids[np.argsort(p)[-2]]), int(ids[np.argmin(p)]), 77777):
        counts = {}
        for c in range(N):
            n_acc, out = ops.sample(idx, fine, [draft], ctr=c, **kw)
            assert len(out) == n_acc + 1 and (n_acc == 0 or out[0] == draft)
            counts[out[0]] = counts.get(out[0], 0) + 1
        for j, pid in enumerate(ids):
            f = counts.pop(int(pid), 0) / N
            sd = np.sqrt(max(p[j] * (1 - p[j]), 1e-12) / N)
            assert abs(f - p[j]) <= 5 * sd + 1e-9, (case, draft, int(pid), f, p[j])
        assert not counts, counts  # nothing outside the candidates
    first = {}
    for c in range(N):
        t = ops.sample(idx[:1], fine[:1], None, ctr=c, first_row=0, **kw)
        first[t] = first.get(t, 0) + 1
    for j, pid in enumerate(ids):
        f = first.get(int(pid), 0) / N
        assert abs(f - p[j]) <= 5 * np.sqrt(max(p[j] * (1 - p[j]), 1e-12) / N) + 1e-9


def test_sampling_is_deterministic_per_seed_and_counter():
    rng = np.random.default_rng(2)
    K = 64
    idx = np.stack([rng.permutation(5000)[:K] for _ in range(3)]).astype(np.int32)
    fine = ops.f32_to_bf16(rng.standard_normal((3, K)).astype(np.float32))
    kw = dict(temperature=1.0, top_p=0.95, V=5000)
    d = [int(idx[0, 5]), int(idx[1, 9])]
    a = [ops.sample(idx, fine, d, seed=7, ctr=c, **kw) for c in range(50)]
    assert a == [ops.sample(idx, fine, d, seed=7, ctr=c, **kw) for c in range(50)]
    assert a != [ops.sample(idx, fine, d, seed=8, ctr=c, **kw) for c in range(50)]


@pytest.mark.parametrize("sp", [dict(temperature=0.7, top_k=20, top_p=0.9), dict(temperature=1.0, top_p=0.5),
                                dict(temperature=1.0, min_p=0.1)])
def test_distribution_is_valid(sp):
    """tests/test_kernels.py:129-139 of the reference on the restated Engine._dist (1000 candidates x 3
    rows of N(0, 9) logits): probabilities sum to 1, top_k / top_p / min_p hold."""
    rng = np.random.default_rng(7)
    for row in range(3):
        fine = ops.f32_to_bf16((rng.standard_normal(1000) * 3).astype(np.float32))
        idx = np.arange(1000, dtype=np.int32)
        kept, p = ops.sample_dist(idx, fine, V=1000, **sp)
        assert abs(float(p.astype(np.float64).sum()) - 1.0) <= 1e-4
        assert np.all(np.diff(p) <= 0)  # sorted by probability
        if sp.get("top_k"):
            assert len(kept) <= sp["top_k"]
        if sp.get("min_p"):
            assert float(p.min()) >= sp["min_p"] * float(p[0]) * (1 - 1e-5)
        # the kept set and probabilities of an independent float64 restatement
        lf = ops.bf16_to_f32(fine).astype(np.float64)
        p64 = _dist64(lf, sp["temperature"], sp.get("top_k", 0), sp.get("top_p", 1.0), sp.get("min_p", 0.0))
        assert set(kept.tolist()) == set(np.flatnonzero(p64 > 0).tolist())
        assert np.allclose(p, p64[kept], rtol=1e-5, atol=1e-7)
