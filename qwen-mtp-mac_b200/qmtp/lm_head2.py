"""Two-stage lm_head -- the lm_head2.py surface of qwen-mtp-mac on B200.

Reference: lm_head2.py:14-29 ``TwoStageHead(weight, k=64)`` (coarse quantized full-vocab logits,
argpartition top-k, exact rescoring of the k rows with the original bf16 weights, full-size logits
with -inf elsewhere) and lm_head2.py:32-36 ``k_for(sampling)``.

The coarse stage here is the affine 4-bit group-64 format (the reference builds NVFP4 group-16;
the B200 build is judged on affine g64).  ``__call__`` keeps the reference's output contract;
``select`` is the engine's path: candidates, exact logits and the greedy token without
materialising [.., V] logits.  Ties are resolved as (value descending, vocab index ascending).
"""
from __future__ import annotations

import torch

from . import _lib
from .qmv_kernel import QuantizedLinear


class TwoStageHead:
    def __init__(self, weight: torch.Tensor, k: int = 64, coarse: QuantizedLinear | None = None):
        """weight: bf16 [V, D] (kept resident, only k rows per position are read)."""
        if weight.dtype != torch.bfloat16 or weight.dim() != 2:
            raise ValueError("TwoStageHead expects a bf16 [V, D] weight")
        self.weight = weight
        self.coarse = coarse if coarse is not None else QuantizedLinear.from_linear(weight, group_size=64, bits=4)
        self.k = k
        self._ws: dict = {}

    @property
    def vocab(self) -> int:
        return self.weight.shape[0]

    def _workspace(self, M: int, k: int) -> torch.Tensor:
        key = (M, k)
        if key not in self._ws:
            n = _lib.lib().qmtp_lmhead2_workspace(M, self.vocab, k)
            self._ws[key] = torch.empty(n, dtype=torch.uint8, device=self.weight.device)
        return self._ws[key]

    def select(self, h: torch.Tensor, k: int | None = None, coarse_out: torch.Tensor | None = None,
               out=None):
        """h bf16 [..., D] -> (idx int32 [M, k], fine bf16 [M, k], argmax int32 [M])."""
        k = self.k if k is None else k
        D = h.shape[-1]
        h2 = h.reshape(-1, D)
        if h2.stride(0) != D:
            h2 = h2.contiguous()
        M = h2.shape[0]
        _lib.require_cuda(h2)
        if out is None:
            idx = torch.empty((M, k), dtype=torch.int32, device=h.device)
            fine = torch.empty((M, k), dtype=torch.bfloat16, device=h.device)
            amax = torch.empty((M,), dtype=torch.int32, device=h.device)
        else:
            idx, fine, amax = out
        ws = self._workspace(M, k)
        c = self.coarse
        _lib.check(_lib.lib().qmtp_lmhead2(
            h2.data_ptr(), c.weight.data_ptr(), c.scales.data_ptr(), c.biases.data_ptr(), self.weight.data_ptr(),
            M, self.vocab, D, k, idx.data_ptr(), fine.data_ptr(), amax.data_ptr(),
            None if coarse_out is None else coarse_out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream()),
            "TwoStageHead")
        return idx, fine, amax

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        """Reference contract (lm_head2.py:23-29): full-size logits, -inf outside the candidates."""
        idx, fine, _ = self.select(h)
        out = torch.full((idx.shape[0], self.vocab), float("-inf"), dtype=torch.bfloat16, device=h.device)
        out.scatter_(1, idx.long(), fine)
        return out.reshape(*h.shape[:-1], self.vocab)


def k_for(sampling) -> int:
    """lm_head2.py:32-36: 64 for greedy or top_k <= 32; else 4*top_k (top_k = 0 -> 256), max 2048.
    This build's selection kernel supports k <= 256."""
    if sampling is None or sampling.temperature <= 0 or 0 < sampling.top_k <= 32:
        return 64
    return 256 if sampling.top_k <= 0 else min(4 * sampling.top_k, 2048)


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None):
    """Greedy token of bf16 logits [..., V] (ties -> lowest index), int32 [M]."""
    V = logits.shape[-1]
    l2 = logits.reshape(-1, V)
    M = l2.shape[0]
    _lib.require_cuda(l2)
    if out is None:
        out = torch.empty((M,), dtype=torch.int32, device=logits.device)
    n = _lib.lib().qmtp_argmax_workspace(M, V)
    if workspace is None or workspace.numel() < n:
        workspace = torch.empty(n, dtype=torch.uint8, device=logits.device)
    _lib.check(_lib.lib().qmtp_argmax_bf16(l2.data_ptr(), l2.stride(0), M, V, out.data_ptr(), workspace.data_ptr(),
                                           workspace.numel(), _lib.stream()), "argmax")
    return out
