"""BASELINE config 4 at full size: the B200 decoder's greedy MTP stream for a 512-token prompt and 256
generated tokens (k = 2, Qwen3.5-9B-shaped hybrid decoder, affine g64) equals the oracle's, token for
token (GPU).

The expected stream is the committed fixture tests/golden/config4_stream.json, made on the CPU by
tests/golden/make_config4.py with the C oracle.  The weights are regenerated here from the same seed
(oracle.model.synthetic_weights_seeded: numpy draws and the oracle quantizer, identical bits on any
machine) and uploaded, so nothing large is shipped.  This is the end-to-end check of
mtp.py:351-369 (the MTP stream equals plain greedy decoding) at the benchmark's own configuration."""
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
FIXTURE = Path(__file__).resolve().parent / "golden" / "config4_stream.json"


def test_config4_full_size_stream_matches_oracle():
    import torch

    from oracle import model as om
    from qmtp import model as qm
    from qmtp.mtp import MTPDecoder, decode_mtp
    from tests.golden import make_config4 as mk

    want = json.loads(FIXTURE.read_text())
    assert want["weight_seed"] == mk.WEIGHT_SEED and want["prompt_seed"] == mk.PROMPT_SEED
    oargs = mk.config()
    Wn = om.synthetic_weights_seeded(oargs, seed=want["weight_seed"])
    args = qm.ModelArgs(max_pos=oargs.max_pos)
    W = qm.from_numpy(Wn)
    del Wn
    prompt = mk.prompt_ids(oargs)
    assert len(prompt) == want["prompt_len"]
    dec = MTPDecoder(args, W, k=want["k"], max_tokens=want["max_tokens"] + 16)
    out, st = decode_mtp(dec, prompt, want["max_tokens"], use_graph=True)
    torch.cuda.synchronize()
    first_diff = next((i for i, (a, b) in enumerate(zip(out, want["tokens"])) if a != b), None)
    print(f"config 4: {len(out)} tokens, {st['cycles']} cycles, smallest oracle logit margin "
          f"{want['min_margin']:.4g} over {want['rows_checked']} verified rows")
    assert first_diff is None and len(out) == len(want["tokens"]), f"streams differ from token {first_diff}"
    from qmtp import _lib

    assert _lib.device_error() == 0
