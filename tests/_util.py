"""Shared helpers for the tests (seeded inputs, torch <-> numpy bf16 bit views)."""
import numpy as np

from oracle import ops


def rng(seed=0):
    return np.random.default_rng(seed)


def randn_bf16(shape, seed=0, scale=1.0):
    return ops.f32_to_bf16(rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))


def to_torch(a, dev):
    """numpy bits -> torch tensor of the matching dtype on `dev` (uint16 -> bf16, uint32 -> int32)."""
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(dev)
    return torch.from_numpy(a).to(dev)


def to_np(t):
    """torch tensor -> numpy bits (bf16 -> uint16, int32 -> uint32)."""
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def affine_layer(N, K, seed=0, std=0.02):
    """Seeded N(0, std) bf16 weights quantized by the oracle: (w_bf16, wq, scales, biases)."""
    w = randn_bf16((N, K), seed, std)
    wq, s, b = ops.quantize_affine(w)
    return w, wq, s, b
