"""The B200 MTP engine (qmtp.mtp) against the oracle model: identical greedy token streams (GPU).

Small Qwen3.5-shaped model (4 layers: 3 GatedDeltaNet + 1 gated attention, hidden 1024) so the
oracle finishes in seconds; the full-size configuration is exercised by bench.py and
test_config4_gpu.py."""
import numpy as np
import pytest

from oracle import model as om
from tests.test_model_oracle import greedy_overrides, prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_pair():
    from qmtp import model as qm

    Wn = om.synthetic_weights(om.SMALL, seed=0)
    return om.OracleModel(om.SMALL, Wn), qm.from_numpy(Wn)


def _decoder(W, max_tokens=300):
    from qmtp import model as qm
    from qmtp.mtp import MTPDecoder

    return MTPDecoder(qm.SMALL, W, k=2, max_tokens=max_tokens)


@pytest.mark.parametrize("use_graph", [False, True])
def test_stream_matches_oracle(small_pair, use_graph):
    from qmtp.mtp import decode_mtp

    orc, W = small_pair
    p = prompt(40)
    ref, _ = orc.generate_mtp(p, 30)
    out, st = decode_mtp(_decoder(W), p, 30, use_graph=use_graph)
    assert out == ref
    assert st["cycles"] >= 1


def test_rollback_paths_match_oracle(small_pair):
    from qmtp.mtp import decode_mtp

    orc, W = small_pair
    p = prompt(34, seed=2)
    g = orc.generate_greedy(p, 45)
    ref, rst = orc.generate_mtp(p, 45, draft_override=greedy_overrides(g, om.SMALL.vocab))
    out, st = decode_mtp(_decoder(W), p, 45, use_graph=True, draft_override=greedy_overrides(g, om.SMALL.vocab))
    assert ref == g and out == ref
    assert st["acept"] == rst["acept"]


def test_config4_loop_shape_on_small_model(small_pair):
    """512-token prompt, 256 generated tokens, k = 2 (the config-4 loop) on the small model."""
    from qmtp.mtp import decode_mtp

    orc, W = small_pair
    p = prompt(512, seed=5)
    ref, _ = orc.generate_mtp(p, 256)
    out, st = decode_mtp(_decoder(W), p, 256, use_graph=True)
    assert len(out) == 256 and out == ref


@pytest.mark.parametrize("tau,override", [(0.0, True), (3e-7, True), (3e-7, False), (0.5, True), (0.999, False)])
def test_adaptive_draft_count_matches_oracle(small_pair, tau, override):
    """Adaptive k (mtp.py:229-238): drafts accepted only up to n_drafts(probs, tau), probs being the
    draft head's argmax probabilities.  The token stream equals plain greedy decoding, and the
    acceptance statistics and drafts verified per cycle equal the oracle's adaptive loop."""
    from qmtp.mtp import decode_mtp

    orc, W = small_pair
    p = prompt(33, seed=8)
    ov = greedy_overrides(orc.generate_greedy(p, 40), om.SMALL.vocab) if override else None
    ref, rst = orc.generate_mtp(p, 40, draft_override=ov, tau=tau)
    assert ref == orc.generate_greedy(p, 40)
    dec = _decoder(W)
    dec.set_tau(tau)
    ov2 = greedy_overrides(orc.generate_greedy(p, 40), om.SMALL.vocab) if override else None
    out, st = decode_mtp(dec, p, 40, use_graph=True, draft_override=ov2)
    assert out == ref
    assert st["acept"] == rst["acept"] and st["cycles"] == rst["cycles"]
    assert st["borradores_ciclo"] == rst["borradores_ciclo"]
    if tau == 0.999:
        assert st["borradores_ciclo"] == 1.0  # random weights: no draft is that likely
    if tau == 0.0:
        assert st["borradores_ciclo"] == 2.0  # every draft is verified


def test_draft_prob_matches_oracle(dev):
    """The draft head's argmax probability (qmtp_draft_prob) equals the oracle's bit for bit."""
    import torch

    from oracle import ops
    from qmtp import _lib
    from tests._util import randn_bf16, to_torch

    for V, scale in ((248320, 3.0), (16384, 0.5), (1000, 20.0)):
        lg = randn_bf16((V,), V, scale)
        t = int(ops.argmax_bf16(lg[None])[0])
        pr = torch.empty(1, dtype=torch.float32, device=dev)
        tok = torch.tensor([t], dtype=torch.int32, device=dev)
        _lib.check(_lib.lib().qmtp_draft_prob(to_torch(lg, dev).data_ptr(), V, tok.data_ptr(), pr.data_ptr(),
                                              _lib.stream()), "draft_prob")
        assert float(pr.item()) == ops.draft_prob(lg, t), V


@pytest.mark.parametrize("mode,tau", [("first", 3e-6), ("freq", 6e-6)])  # taus giving 1.3 and 1.6 drafts a cycle
def test_draft_head_subset_matches_oracle(small_pair, mode, tau):
    """A draft head over a vocabulary subset (mtp.py:156-196 DraftHead with ids, load_draft_head): the
    first drafts after the prompt, the adaptive draft count's statistics (which read the subset head's
    argmax probabilities every cycle) and the stream equal the oracle's with the same subset, and the
    stream still equals plain greedy decoding."""
    from qmtp import model as qm
    from qmtp.mtp import decode_mtp, load_draft_head

    orc, W = small_pair
    lm = qm.Model(qm.SMALL, W)
    V = om.SMALL.vocab
    if mode == "first":
        head = load_draft_head(5000, {"bits": 4, "group_size": 64}, lm=lm)
        assert head.ids is None and head.proj.out_features == 5000
        orc.set_draft_head(5000)
    else:
        counts = np.random.default_rng(3).integers(0, 1000, V)  # many equal counts
        head = load_draft_head(3000, None, True, (7, V - 1), lm=lm, counts=counts)
        orc.set_draft_head(3000, counts, (7, V - 1))
        assert head.ids.tolist() == orc.draft_ids.tolist()
        assert 7 in orc.draft_ids and V - 1 in orc.draft_ids
    try:
        p = prompt(33, seed=8)
        _, _, t, drafts = orc.prefill(p, 2)
        dec = _decoder(W)
        dec.set_draft_head(head)
        dec.prefill(p)
        assert dec.tokens_in.tolist() == [int(t)] + [int(d) for d in drafts]
        if mode == "freq":
            assert set(int(d) for d in drafts) <= set(orc.draft_ids.tolist())
        ref, rst = orc.generate_mtp(p, 40, tau=tau)
        assert ref == orc.generate_greedy(p, 40)
        assert 1.0 < rst["borradores_ciclo"] < 2.0
        dec = _decoder(W)
        dec.set_draft_head(head)
        dec.set_tau(tau)
        out, st = decode_mtp(dec, p, 40, use_graph=True)
        assert out == ref
        assert st["acept"] == rst["acept"] and st["cycles"] == rst["cycles"]
        assert st["borradores_ciclo"] == rst["borradores_ciclo"]
    finally:
        orc.set_draft_head(None)
