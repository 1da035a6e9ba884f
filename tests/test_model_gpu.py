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
