"""Draft head over a vocabulary subset (mtp.py:170-196 load_draft_head) in the oracle (CPU): the head's
4-bit g64 quantization is per row and group, so quantizing the subset's bf16 rows equals taking those
rows of the full quantized head (what both the oracle and qmtp.mtp.load_draft_head do)."""
import numpy as np

from oracle import model as om
from oracle import ops
from tests._util import randn_bf16


def test_subset_quantization_is_a_row_gather():
    W = randn_bf16((300, 256), 5, 0.02)
    full = ops.quantize_affine(W)
    rows = np.array([0, 3, 17, 18, 150, 299])
    sub = ops.quantize_affine(np.ascontiguousarray(W[rows]))
    for a, b in zip(full, sub):
        assert np.array_equal(np.asarray(a)[rows], np.asarray(b))


def test_set_draft_head_ids():
    args = om.SMALL
    W = om.synthetic_weights(args, seed=0)
    m = om.OracleModel(args, W)
    V = args.vocab
    m.set_draft_head(100)                       # the first ids: no id map
    assert m.draft_ids is None and m.draft_W[0].shape[0] == 100
    assert np.array_equal(m.draft_W[0], np.asarray(W["lm_head_q"][0])[:100])
    counts = np.zeros(V, np.int64)
    counts[[5, 9, 400]] = [3, 7, 5]
    m.set_draft_head(2, counts, extra_ids=(11,))  # the 2 most frequent (9, 400) plus 11, ascending
    assert m.draft_ids.tolist() == [9, 11, 400]
    assert np.array_equal(m.draft_W[1], np.asarray(W["lm_head_q"][1])[[9, 11, 400]])
    m.set_draft_head(None)
    assert m.draft_ids is None and m.draft_W is None  # the full head again


def test_load_draft_head_selects_the_oracles_rows():
    """qmtp.mtp.load_draft_head (host code, no kernel runs here) picks the same ids and rows as the
    oracle's set_draft_head, for the first-ids and the frequency forms."""
    import torch
    from types import SimpleNamespace

    from qmtp.mtp import load_draft_head
    from qmtp.qmv_kernel import QuantizedLinear

    args = om.SMALL
    W = om.synthetic_weights(args, seed=0)
    wq, s, b = (torch.from_numpy(np.asarray(t).view(np.int32 if t.dtype == np.uint32 else np.int16)) for t in
                W["lm_head_q"])
    lm = SimpleNamespace(weights={"lm_head_q": QuantizedLinear(wq, s, b)})
    m = om.OracleModel(args, W)
    V = args.vocab
    counts = np.random.default_rng(3).integers(0, 1000, V)
    head = load_draft_head(3000, None, True, (7, V - 1), lm=lm, counts=counts)
    m.set_draft_head(3000, counts, (7, V - 1))
    assert head.ids.tolist() == m.draft_ids.tolist()
    assert np.array_equal(head.proj.weight.numpy().view(np.uint32), m.draft_W[0])
    first = load_draft_head(500, {"bits": 4, "group_size": 64}, lm=lm)
    assert first.ids is None and first.proj.out_features == 500
    assert load_draft_head(V, None, lm=lm).proj is lm.weights["lm_head_q"]


def test_draft_head_argument_checks():
    """Host-side refusals of load_draft_head / DraftHead (no kernel runs)."""
    import pytest
    import torch
    from types import SimpleNamespace

    from qmtp.mtp import DraftHead, load_draft_head
    from qmtp.qmv_kernel import QuantizedLinear

    W = om.synthetic_weights(om.SMALL, seed=0)
    wq, s, b = (torch.from_numpy(np.asarray(t).view(np.int32 if t.dtype == np.uint32 else np.int16)) for t in
                W["lm_head_q"])
    full = QuantizedLinear(wq, s, b)
    lm = SimpleNamespace(weights={"lm_head_q": full})
    with pytest.raises(ValueError):
        load_draft_head(100, None, True, lm=lm)                     # freq needs the corpus counts
    with pytest.raises(NotImplementedError):
        load_draft_head(100, {"bits": 8, "group_size": 64}, lm=lm)  # draft heads are 4-bit g64
    with pytest.raises(ValueError):
        DraftHead(QuantizedLinear(wq[:10], s[:10], b[:10]), torch.arange(9))  # one id per row
    h = DraftHead(QuantizedLinear(wq[:3], s[:3], b[:3]), torch.tensor([5, 9, 2]))
    assert h.token(torch.tensor([[0.1, 0.7, 0.7]])).tolist() == [9]  # first maximum, mapped through ids
