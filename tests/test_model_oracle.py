"""Oracle model (CPU): the MTP speculative stream equals plain greedy decoding (the reference's own
equivalence check, mtp.py:351-369), with and without accepted drafts."""
import numpy as np
import pytest

from oracle import model as om


@pytest.fixture(scope="module")
def small():
    W = om.synthetic_weights(om.SMALL, seed=0)
    return om.OracleModel(om.SMALL, W)


def prompt(n, seed=1):
    return np.random.default_rng(seed).integers(0, om.SMALL.vocab, n).astype(np.int32)


def greedy_overrides(g, vocab):
    """draft_override for generate_mtp: cycle 3j gets the right continuation (keep 3), 3j+1 a wrong
    second draft (keep 2), 3j+2 a wrong first draft (keep 1)."""
    pos = {"n": 1}

    def fn(cycle):
        n = pos["n"]
        if n + 1 >= len(g):
            return None
        d = [g[n], g[n + 1]]
        kind = cycle % 3
        if kind == 1:
            d[1] = (d[1] + 1) % vocab
            pos["n"] = n + 2
        elif kind == 2:
            d[0] = (d[0] + 1) % vocab
            pos["n"] = n + 1
        else:
            pos["n"] = n + 3
        return d

    return fn


def test_mtp_equals_greedy(small):
    p = prompt(40)
    g = small.generate_greedy(p, 24)
    out, st = small.generate_mtp(p, 24)
    assert out == g
    assert st["tok_ciclo"] >= 1.0


def test_mtp_with_accepted_drafts_equals_greedy(small):
    p = prompt(33, seed=2)
    g = small.generate_greedy(p, 40)
    out, st = small.generate_mtp(p, 40, draft_override=greedy_overrides(g, om.SMALL.vocab))
    assert out == g
    assert st["acept"][0] > 0.3 and st["tok_ciclo"] > 1.5
