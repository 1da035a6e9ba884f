"""The engine boundary (qmtp.engine.Engine, the swap point of engine.py:155-213) and the reference-
signature loop functions of mtp.py:136-303 (generate_mtp, backbone, restore, draft_chain), on the
small Qwen3.5-shaped model against decode_mtp and the oracle (GPU)."""
import pytest

from oracle import model as om
from tests.test_model_oracle import prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    from qmtp import model as qm

    Wn = om.synthetic_weights(om.SMALL, seed=0)
    return om.OracleModel(om.SMALL, Wn), qm.Model(qm.SMALL, qm.from_numpy(Wn))


def test_engine_generate_matches_generate_mtp_and_oracle(small):
    from qmtp.engine import Engine, Sampling
    from qmtp.mtp import generate_mtp

    orc, lm = small
    p = prompt(40, seed=3)
    ref, _ = orc.generate_mtp(p, 30)
    eng = Engine(lm, k=2)
    stats = {}
    got = list(eng.generate(p, 0, 30, Sampling(), stats))
    assert got == ref
    for key in ("t_start", "t_first", "prompt_tokens", "cached_tokens", "cycles", "accepted", "k"):
        assert key in stats
    assert stats["prompt_tokens"] == 40 and stats["cached_tokens"] == 0 and stats["k"] == 2
    out, st = generate_mtp(lm, lm.mtp, p, 30, (), head=None, k=2)
    assert out == ref and st["cycles"] >= 1


def test_engine_prefix_cache_and_eos(small):
    """A second request that extends the first one's prefix resumes from the kept state; an eos token
    ends the stream after it is yielded (engine.py:176-213)."""
    from qmtp.engine import Engine, Sampling

    orc, lm = small
    p = prompt(30, seed=4)
    eng = Engine(lm, k=2)
    first = list(eng.generate(p, 24, 12, Sampling(), {}))
    ref, _ = orc.generate_mtp(p, 12)
    assert first == ref
    p2 = list(p[:24]) + list(prompt(9, seed=5))
    st = {}
    second = list(eng.generate(p2, 24, 12, Sampling(), st))
    ref2, _ = orc.generate_mtp(p2, 12)
    assert second == ref2 and st["cached_tokens"] == 24
    eos = ref2[5]
    stop = list(Engine(lm, k=2, eos=(eos,)).generate(p2, 0, 12, Sampling(), {}))
    assert stop == ref2[:ref2.index(eos) + 1]


def test_engine_sampling_matches_oracle(small):
    from qmtp.engine import Engine, Sampling

    orc, lm = small
    p = prompt(20, seed=6)
    sp = Sampling(temperature=0.8, top_p=0.95, min_p=0.02, seed=7)
    ref, _ = orc.generate_mtp(p, 16, sampling=sp)
    eng = Engine(lm, k=2)
    assert list(eng.generate(p, 0, 16, sp, {})) == ref
    # the same engine goes back to greedy decoding (the sampler's graph is dropped)
    ref_g, _ = orc.generate_mtp(p, 16)
    assert list(eng.generate(p, 0, 16, Sampling(), {})) == ref_g


def test_worker_streams_a_job(small):
    from qmtp.engine import Engine, Sampling, Worker

    orc, lm = small
    p = prompt(25, seed=8)
    ref, _ = orc.generate_mtp(p, 10)
    w = Worker(lambda: Engine(lm, k=2))
    job = w.submit(p, 0, 10, Sampling())
    assert list(job.tokens()) == ref
    w.close()


def test_reference_style_loop_functions(small):
    """The reference's own loop written with backbone / restore / draft_chain (mtp.py:241-303, greedy,
    k = 2) reproduces decode_mtp's stream."""
    import torch

    from qmtp.mtp import backbone, decode_mtp, draft_chain, restore

    orc, lm = small
    p = [int(v) for v in prompt(12, seed=9)]
    want, _ = decode_mtp(lm.make_cache(k=2, max_tokens=64), p, 14, use_graph=False)
    cache = lm.make_cache(k=2, max_tokens=64)
    cache.reset()
    S = cache.S
    # prompt in verify-sized steps; the MTP sees the pairs (h[i], token[i+1])
    hs = []
    for i in range(0, len(p), S):
        chunk = p[i:i + S]
        logits, h, hn = backbone(lm, chunk, cache)
        hs.append(h[0])
    h_all = torch.cat(hs)
    t = int(torch.argmax(logits[0, -1]).item())
    out = [t]
    nxt = torch.tensor(list(p[1:]) + [t], dtype=torch.int32)
    drafts = None
    for i in range(0, len(p), S):
        n = min(S, len(p) - i)
        drafts = draft_chain(lm, lm.mtp, h_all[i:i + n][None], nxt[i:i + n][None], cache, 2)
    while len(out) < 14:
        toks = [t] + drafts[0].tolist()
        logits, h, hn = backbone(lm, toks, cache)
        a = torch.argmax(logits[0].float(), dim=-1).tolist()
        n_acc = 0
        while n_acc < 2 and a[n_acc] == toks[1 + n_acc]:
            n_acc += 1
        keep = n_acc + 1
        out += a[:keep]
        if keep < S:
            restore(cache, keep)
        t = a[keep - 1]
        drafts = draft_chain(lm, lm.mtp, h[:, :keep], torch.tensor(a[:keep], dtype=torch.int32)[None], cache, 2)
    assert out[:14] == want
