"""Generates tests/golden/config4_stream.json: the oracle's greedy MTP token stream for BASELINE.json
config 4 at full size (Qwen3.5-9B-shaped hybrid decoder, affine g64, 512-token prompt, 256 generated
tokens, k = 2, batch 1), the fixture tests/test_config4_gpu.py decodes against.

    python tests/golden/make_config4.py      (about half an hour on 8 cores)

Weights: oracle.model.synthetic_weights_seeded(CONFIG4, WEIGHT_SEED) -- reproducible on any machine,
so the GPU test regenerates the same bits instead of shipping ~6 GB.  Prompt: 512 ids drawn uniformly
from the vocabulary by numpy.random.default_rng(PROMPT_SEED).  Besides the tokens the file keeps the
smallest margin between the best and second-best exact logit the head saw on any verified row, which
says how close the stream came to a tie.
"""
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import model as om  # noqa: E402
from oracle import ops  # noqa: E402

WEIGHT_SEED, PROMPT_SEED, PROMPT_LEN, MAX_TOKENS, K = 4, 1000, 512, 256, 2
OUT = HERE / "config4_stream.json"


def config():
    return om.ModelArgs(max_pos=1024)


def prompt_ids(args):
    return np.random.default_rng(PROMPT_SEED).integers(0, args.vocab, PROMPT_LEN).tolist()


def main():
    t0 = time.time()
    args = config()
    W = om.synthetic_weights_seeded(args, seed=WEIGHT_SEED)
    t1 = time.time()
    orc = om.OracleModel(args, W)
    margins = []

    def head(hn, k=64):
        wq, s, b = orc.W["lm_head_q"]
        _, idx, fine, amax = ops.two_stage_head(hn, wq, s, b, orc.W["lm_head"], k)
        f = np.sort(ops.bf16_to_f32(fine).astype(np.float64), axis=1)
        margins.extend((f[:, -1] - f[:, -2]).tolist())
        return amax

    orc.head = head
    p = prompt_ids(args)
    tokens, st = orc.generate_mtp(p, MAX_TOKENS, k=K)
    t2 = time.time()
    rec = {"weight_seed": WEIGHT_SEED, "prompt_seed": PROMPT_SEED, "prompt_len": PROMPT_LEN,
           "max_tokens": MAX_TOKENS, "k": K, "tokens": [int(t) for t in tokens],
           "cycles": int(st.get("cycles", 0)), "min_margin": float(min(margins)),
           "rows_checked": len(margins), "weights_s": round(t1 - t0, 1), "decode_s": round(t2 - t1, 1)}
    OUT.write_text(json.dumps(rec, indent=1) + "\n")
    print(json.dumps({k: v for k, v in rec.items() if k != "tokens"}))


if __name__ == "__main__":
    main()
