"""Synthetic Qwen3.5-9B-shaped hybrid decoder for the B200 engine: configuration and weights.

Structure (mlx-lm qwen3_5 as patched by the reference, cross-checked with transformers' Qwen3.5):
32 layers, layer i is gated full attention when (i+1) % 4 == 0 and GatedDeltaNet otherwise; hidden
4096, SwiGLU MLP 12288, 16 query / 4 KV heads of dim 256 with partial (64-dim) rotate-half RoPE,
q/k RMS norms and a sigmoid output gate; GatedDeltaNet with 16 key / 32 value heads of dim 128 and a
4-tap causal conv; vocab 248320; plus the 1-layer MTP head of mtp.py:35-70.

Every linear layer is 4-bit affine group 64 (uint32 nibbles + bf16 scales/biases).  Projections
that read the same input are stored concatenated along the output rows, which changes nothing in
the per-row arithmetic: GatedDeltaNet in_proj = [qkv | z | b | a], attention qkv_proj =
[per head (query, gate) | k | v], MLP gate_up = [gate | up].  The lm_head is kept in bf16 (exact
stage of the two-stage head) and as an affine g64 copy (coarse stage and draft head).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .qmv_kernel import QuantizedLinear, quantize


@dataclass
class ModelArgs:
    hidden: int = 4096
    layers: int = 32
    intermediate: int = 12288
    n_heads: int = 16
    n_kv: int = 4
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 10_000_000.0
    vocab: int = 248320
    lin_hk: int = 16
    lin_hv: int = 32
    lin_dk: int = 128
    lin_dv: int = 128
    conv_k: int = 4
    eps: float = 1e-6
    full_attention_interval: int = 4
    max_pos: int = 1024

    def is_linear(self, i: int) -> bool:
        return (i + 1) % self.full_attention_interval != 0

    @property
    def conv_dim(self) -> int:
        return 2 * self.lin_hk * self.lin_dk + self.lin_hv * self.lin_dv

    @property
    def gdn_proj(self) -> int:
        return self.conv_dim + self.lin_hv * self.lin_dv + 2 * self.lin_hv

    @property
    def attn_proj(self) -> int:
        return self.n_heads * 2 * self.head_dim + 2 * self.n_kv * self.head_dim

    def param_count(self) -> int:
        h, i = self.hidden, self.intermediate
        n = self.vocab * h  # embedding
        for l in range(self.layers):
            n += 3 * h * i
            n += self.gdn_proj * h + self.lin_hv * self.lin_dv * h if self.is_linear(l) else \
                self.attn_proj * h + self.n_heads * self.head_dim * h
        return n


CONFIG4 = ModelArgs()
SMALL = ModelArgs(hidden=1024, layers=4, intermediate=2048, n_heads=4, n_kv=2, head_dim=256, vocab=16384,
                  lin_hk=4, lin_hv=8, max_pos=1024)


def rope_tables(args: ModelArgs, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_pos, rotary/2] fp32, computed in float64 on the host (inv_freq_i = theta^(-2i/R))."""
    half = args.rotary_dim // 2
    inv = 1.0 / (args.rope_theta ** (np.arange(0, args.rotary_dim, 2, dtype=np.float64) / args.rotary_dim))
    ang = np.arange(args.max_pos, dtype=np.float64)[:, None] * inv[None, :half]
    return (torch.from_numpy(np.cos(ang).astype(np.float32)).to(device),
            torch.from_numpy(np.sin(ang).astype(np.float32)).to(device))


class Weights(dict):
    """Nested dict of device tensors / QuantizedLinear layers, same key names as the oracle's."""


class Model:
    """The language model handle the reference's loop functions take as ``lm`` (mtp.py:143-303):
    configuration, weights, the two-stage head (``lm_head``, lm_head2.py:14-29) and its MTP weights
    (``mtp``, mtp.py:35-70).  ``make_cache`` returns the device state of a decoding session (an
    ``MTPDecoder``), which stands for the reference's trunk cache and MTP cache together."""

    def __init__(self, args: ModelArgs, weights: Weights):
        from .lm_head2 import TwoStageHead

        self.args, self.weights = args, weights
        self.mtp = weights["mtp"]
        self.lm_head = TwoStageHead(weights["lm_head"], 64, weights["lm_head_q"])
        self._caches: dict = {}

    def make_cache(self, k: int = 2, max_tokens: int = 1024, sampling=None):
        from .mtp import MTPDecoder

        return MTPDecoder(self.args, self.weights, k=k, max_tokens=max_tokens,
                          device=self.weights["norm"].device, sampling=sampling)

    def session(self, k: int = 2, max_tokens: int = 1024):
        """A decoder for k drafts kept on the model (reused by generate_mtp calls with the same k while
        it has room for max_tokens)."""
        dec = self._caches.get(k)
        if dec is None or dec.out_cap < max_tokens + dec.S + 8:
            dec = self.make_cache(k=k, max_tokens=max(max_tokens, 1024))
            self._caches[k] = dec
        return dec


def _randn_bf16(shape, gen, std, device):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def synthetic_weights(args: ModelArgs, seed: int = 0, std: float = 0.02, device="cuda", fmt: str = "affine") -> Weights:
    """Random-init weights generated and quantized on the GPU (torch CUDA RNG, libqmtp quantizer).
    Linear weights N(0, std); norm weights 1; conv N(0, 1/KC); A_log = log U(1, 16); dt_bias N(0, 1).
    fmt "nvfp4": the linears and the embedding in NVFP4 g16 (the Ollama checkpoint's format); the
    lm_head stays bf16 with its affine g64 coarse copy."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    a = args
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)

    def lin(n, k):
        w = _randn_bf16((n, k), g, std, device)
        if fmt == "nvfp4":
            from .moe import quantize as quantize_fp4

            wq, sc = quantize_fp4(w[None], "nvfp4")
            q = QuantizedLinear(wq[0], sc[0], None, group_size=16, mode="nvfp4")
        else:
            q = QuantizedLinear.from_linear(w)
        del w
        return q

    W = Weights()
    W["embed"] = lin(a.vocab, a.hidden)
    for i in range(a.layers):
        L = {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden), "gate_up": lin(2 * a.intermediate, a.hidden),
             "down": lin(a.hidden, a.intermediate)}
        if a.is_linear(i):
            L.update(in_proj=lin(a.gdn_proj, a.hidden),
                     conv1d=_randn_bf16((a.conv_dim, a.conv_k), g, 1.0 / np.sqrt(a.conv_k), device),
                     A_log=torch.log(torch.rand(a.lin_hv, generator=g, device=device) * 15 + 1),
                     dt_bias=_randn_bf16((a.lin_hv,), g, 1.0, device), norm=ones(a.lin_dv),
                     out_proj=lin(a.hidden, a.lin_hv * a.lin_dv))
        else:
            L.update(qkv_proj=lin(a.attn_proj, a.hidden), q_norm=ones(a.head_dim), k_norm=ones(a.head_dim),
                     o_proj=lin(a.hidden, a.n_heads * a.head_dim))
        W[f"layers.{i}"] = L
    W["norm"] = ones(a.hidden)
    W["lm_head"] = _randn_bf16((a.vocab, a.hidden), g, std, device)
    W["lm_head_q"] = QuantizedLinear(*quantize(W["lm_head"]))
    W["mtp"] = {"pre_fc_norm_embedding": ones(a.hidden), "pre_fc_norm_hidden": ones(a.hidden),
                "fc": lin(a.hidden, 2 * a.hidden), "norm": ones(a.hidden),
                "layer": {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden),
                          "qkv_proj": lin(a.attn_proj, a.hidden), "q_norm": ones(a.head_dim),
                          "k_norm": ones(a.head_dim), "o_proj": lin(a.hidden, a.n_heads * a.head_dim),
                          "gate_up": lin(2 * a.intermediate, a.hidden), "down": lin(a.hidden, a.intermediate)}}
    return W


def from_numpy(Wn: dict, device="cuda") -> Weights:
    """Device weights from the oracle's numpy bit arrays (uint16 = bf16, uint32 = packed nibbles)."""
    device = torch.device(device)

    def t(x):
        x = np.ascontiguousarray(x)
        if x.dtype == np.uint16:
            return torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(device)
        if x.dtype == np.uint32:
            return torch.from_numpy(x.view(np.int32)).to(device)
        return torch.from_numpy(x).to(device)

    def conv(v):
        if isinstance(v, dict):
            return {k: conv(x) for k, x in v.items()}
        if isinstance(v, tuple) and len(v) == 2:  # NVFP4: (uint32 nibbles, uint8 e4m3 scales per 16)
            return QuantizedLinear(t(v[0]), t(v[1]), None, group_size=16, mode="nvfp4")
        if isinstance(v, tuple):
            return QuantizedLinear(*(t(x) for x in v))
        return t(v)

    return Weights({k: conv(v) for k, v in Wn.items()})


def to_numpy(W: dict) -> dict:
    """The oracle's layout (numpy bit arrays) of device weights (e.g. GPU-generated full-size ones)."""

    def n(x: torch.Tensor):
        x = x.detach().contiguous().cpu()
        if x.dtype == torch.bfloat16:
            return x.view(torch.int16).numpy().view(np.uint16)
        if x.dtype == torch.int32:
            return x.numpy().view(np.uint32)
        return x.numpy()

    def conv(v):
        if isinstance(v, dict):
            return {k: conv(x) for k, x in v.items()}
        if isinstance(v, QuantizedLinear):
            if v.mode == "nvfp4":
                return (n(v.weight), n(v.scales))
            return (n(v.weight), n(v.scales), n(v.biases))
        return n(v)

    return {k: conv(v) for k, v in W.items()}
