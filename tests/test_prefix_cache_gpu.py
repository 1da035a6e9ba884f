"""Prompt-prefix state cache (engine.py:52-88, 160-172) of the B200 decoder: a prompt that resumes
from a kept prefix decodes the same stream as a fresh prefill of the whole prompt (GPU)."""
import numpy as np
import pytest

from oracle import model as om
from tests.test_model_oracle import prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    from qmtp import model as qm

    Wn = om.synthetic_weights(om.SMALL, seed=0)
    return om.OracleModel(om.SMALL, Wn), qm.from_numpy(Wn)


def _fresh(W, sampling=None):
    from qmtp import model as qm
    from qmtp.mtp import MTPDecoder

    return MTPDecoder(qm.SMALL, W, k=2, max_tokens=400, sampling=sampling)


@pytest.mark.parametrize("sampled", [False, True])
def test_prefix_reuse_matches_fresh_prefill(small, sampled):
    from qmtp.mtp import Sampling, decode_mtp

    orc, W = small
    sp = Sampling(temperature=0.9, top_p=0.95, seed=21) if sampled else None
    rng = np.random.default_rng(5)
    base = [int(v) for v in prompt(31, seed=6)]
    ext = [int(v) for v in rng.integers(0, om.SMALL.vocab, 7)]
    tails = [[int(v) for v in rng.integers(0, om.SMALL.vocab, n)] for n in (5, 1, 8, 4)]
    dec = _fresh(W, sp)
    cases = [(base + tails[0], 31, 0),            # keeps the 31-token prefix
             (base + tails[1], 31, 31),           # resumes from it
             (base + ext + tails[2], 38, 31),     # resumes and extends it to 38
             (base + ext + tails[3], 38, 38),     # resumes from the extended prefix
             (base[:20] + tails[0], 20, 0)]       # shares less than the kept prefix: fresh prefill
    for i, (p, pl, cached) in enumerate(cases):
        out, st = decode_mtp(dec, p, 24, prefix_len=pl, use_graph=i % 2 == 0)
        assert st["cached_tokens"] == cached, (i, st["cached_tokens"])
        ref, _ = decode_mtp(_fresh(W, sp), p, 24)
        assert out == ref, i
        if i == 1:
            want, _ = orc.generate_mtp(p, 24, sampling=sp)
            assert out == want
