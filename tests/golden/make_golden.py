"""Generates the committed golden fixtures of tests/golden/ from seeded inputs with the C oracle.

    python tests/golden/make_golden.py

The reference (aulafy/qwen-mtp-mac) commits no golden vectors and cannot run here (MLX + Metal), so
these fixtures pin the ORACLE against drift and give the GPU tests a fixed expected output.  Every
input is regenerated from numpy.random.default_rng(seed); only outputs and quantized weights are
stored.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import ops  # noqa: E402


def bf16(shape, seed, scale=1.0):
    return ops.f32_to_bf16(np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))


def make_qmv():
    N, K = 256, 2048
    w = bf16((N, K), 100, 0.02)
    wq, s, b = ops.quantize_affine(w)
    x = bf16((4, K), 101)
    y = ops.qmv_affine(x, wq, s, b)
    r = np.random.default_rng(102)
    nq = r.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
    ns = r.integers(54, 70, (N, K // 16), dtype=np.int64).astype(np.uint8)
    ny = ops.qmv_nvfp4(x, nq, ns)
    np.savez_compressed(HERE / "qmv.npz", x=x, wq=wq, s=s, b=b, y=y, nq=nq, ns=ns, ny=ny)


def main(which=("qmv",)):
    for name in which:
        globals()["make_" + name]()
        print("wrote", name)


if __name__ == "__main__":
    main(tuple(sys.argv[1:]) or ("qmv",))
