"""The oracle reproduces the committed golden fixtures bit for bit (CPU)."""
from pathlib import Path

import numpy as np

from oracle import ops

from tests.golden.make_golden import bf16

G = Path(__file__).resolve().parent / "golden"


def test_qmv_golden():
    d = np.load(G / "qmv.npz")
    wq, s, b = ops.quantize_affine(bf16((256, 2048), 100, 0.02))
    assert np.array_equal(wq, d["wq"]) and np.array_equal(s, d["s"]) and np.array_equal(b, d["b"])
    assert np.array_equal(ops.qmv_affine(d["x"], d["wq"], d["s"], d["b"]), d["y"])
    assert np.array_equal(ops.qmv_nvfp4(d["x"], d["nq"], d["ns"]), d["ny"])
