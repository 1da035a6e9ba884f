"""Two-stage lm_head -- the lm_head2.py surface of qwen-mtp-mac on B200.

Reference: lm_head2.py:14-29 ``TwoStageHead(weight, k=64)`` (coarse quantized full-vocab logits,
argpartition top-k, exact rescoring of the k rows with the original bf16 weights, full-size logits
with -inf elsewhere) and lm_head2.py:32-36 ``k_for(sampling)``.

The coarse stage is the affine 4-bit group-64 format by default or, with
``mode="nvfp4"``, the reference's own NVFP4 group-16 format (lm_head2.py:19).  ``__call__`` keeps the reference's output contract;
``select`` is the engine's path: candidates, exact logits and the greedy token without
materialising [.., V] logits.  Ties are resolved as (value descending, vocab index ascending).
"""
from __future__ import annotations

import torch

from . import _lib
from .qmv_kernel import QuantizedLinear


class TwoStageHead:
    def __init__(self, weight: torch.Tensor, k: int = 64, coarse: QuantizedLinear | None = None,
                 mode: str = "affine"):
        """weight: bf16 [V, D] (kept resident, only k rows per position are read).  coarse: a 4-bit copy
        (affine g64 or NVFP4 g16); built from weight in `mode` ("affine" or "nvfp4") when not given."""
        if weight.dtype != torch.bfloat16 or weight.dim() != 2:
            raise ValueError("TwoStageHead expects a bf16 [V, D] weight")
        self.weight = weight
        if coarse is None:
            if mode == "nvfp4":
                from .moe import quantize as quantize_fp4

                wq, sc = quantize_fp4(weight[None], "nvfp4")
                coarse = QuantizedLinear(wq[0], sc[0], None, group_size=16, mode="nvfp4")
            elif mode == "affine":
                coarse = QuantizedLinear.from_linear(weight, group_size=64, bits=4)
            else:
                raise ValueError(f"unknown coarse mode {mode!r}")
        self.coarse = coarse
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
        if c.mode == "nvfp4":
            rc = _lib.lib().qmtp_lmhead2_nvfp4(
                h2.data_ptr(), c.weight.data_ptr(), c.scales.data_ptr(), self.weight.data_ptr(), M, self.vocab, D, k,
                idx.data_ptr(), fine.data_ptr(), amax.data_ptr(), None if coarse_out is None else coarse_out.data_ptr(),
                ws.data_ptr(), ws.numel(), _lib.stream())
        else:
            rc = _lib.lib().qmtp_lmhead2(
                h2.data_ptr(), c.weight.data_ptr(), c.scales.data_ptr(), c.biases.data_ptr(), self.weight.data_ptr(),
                M, self.vocab, D, k, idx.data_ptr(), fine.data_ptr(), amax.data_ptr(),
                None if coarse_out is None else coarse_out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream())
        _lib.check(rc, "TwoStageHead")
        return idx, fine, amax

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        """Reference contract (lm_head2.py:23-29): full-size logits, -inf outside the candidates."""
        idx, fine, _ = self.select(h)
        out = torch.full((idx.shape[0], self.vocab), float("-inf"), dtype=torch.bfloat16, device=h.device)
        out.scatter_(1, idx.long(), fine)
        return out.reshape(*h.shape[:-1], self.vocab)


class ShardedTwoStageHead:
    """The two-stage head sharded by vocabulary over the ranks of a process group: lm_head2.py:111-117
    with the output rows split, so each GPU streams only its share of the coarse weight.  Rank r holds
    rows [v0, v0 + Vs) of the bf16 weight and of its 4-bit coarse copy (``split`` gives the even
    split).  One call:

      1. local: the shard's coarse logits, its best k (value descending, index ascending) and their
         exact logits, as uint64 candidate words carrying global indices (qmtp_lmhead2_shard);
      2. exchange: all-gather of the M x k words and fine logits over the group (NCCL on GPUs);
      3. merge: the best k words of the G lists in order, their fine logits and the argmax
         (qmtp_lmhead2_merge) -- the same on every rank and the same, bit for bit, as TwoStageHead on
         the whole vocabulary, because each shard's list holds that shard's best k under the same order.

    ``local(h, k) -> (words int64 [M, k], fine bf16 [M, k])`` and ``merge(words [G, M, k], fine [G, M,
    k], k) -> (idx, fine, argmax)`` are the library calls by default and pluggable, so the exchange is
    tested with the CPU oracle on gloo ranks."""

    def __init__(self, weight_shard: torch.Tensor | None, v0: int, vocab: int, k: int = 64,
                 coarse: QuantizedLinear | None = None, group=None, local=None, merge=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.v0, self.vocab_total, self.k = int(v0), int(vocab), k
        self.weight = weight_shard
        if local is None:
            if weight_shard is None or weight_shard.dtype != torch.bfloat16 or weight_shard.dim() != 2:
                raise ValueError("ShardedTwoStageHead expects a bf16 [Vs, D] weight shard")
            if coarse is not None and coarse.mode != "affine":
                raise NotImplementedError("the sharded head's coarse stage is affine g64")
            self.coarse = coarse if coarse is not None else QuantizedLinear.from_linear(weight_shard)
        self._local = local or self._local_lib
        self._merge = merge or self._merge_lib
        self._ws: dict = {}

    @staticmethod
    def split(vocab: int, world: int, rank: int) -> tuple[int, int]:
        """(first row, rows) of rank's shard: the first vocab % world ranks hold one row more."""
        base, extra = divmod(vocab, world)
        return rank * base + min(rank, extra), base + (1 if rank < extra else 0)

    @classmethod
    def from_full(cls, weight: torch.Tensor, k: int = 64, group=None, coarse: QuantizedLinear | None = None):
        """This rank's shard of a full [V, D] head (rows copied; a full coarse copy is sliced by rows)."""
        import torch.distributed as dist

        V = weight.shape[0]
        v0, vs = cls.split(V, dist.get_world_size(group), dist.get_rank(group))
        cq = None
        if coarse is not None:
            cq = QuantizedLinear(coarse.weight[v0:v0 + vs].contiguous(), coarse.scales[v0:v0 + vs].contiguous(),
                                 coarse.biases[v0:v0 + vs].contiguous())
        return cls(weight[v0:v0 + vs].contiguous(), v0, V, k, cq, group)

    def _local_lib(self, h2: torch.Tensor, k: int):
        M, D = h2.shape
        Vs = self.weight.shape[0]
        key = ("local", M, k)
        if key not in self._ws:
            n = _lib.lib().qmtp_lmhead2_shard_workspace(M, Vs, k)
            self._ws[key] = (torch.empty(n, dtype=torch.uint8, device=h2.device),
                             torch.empty((M, k), dtype=torch.int64, device=h2.device),
                             torch.empty((M, k), dtype=torch.bfloat16, device=h2.device))
        ws, words, fine = self._ws[key]
        c = self.coarse
        _lib.check(_lib.lib().qmtp_lmhead2_shard(
            h2.data_ptr(), c.weight.data_ptr(), c.scales.data_ptr(), c.biases.data_ptr(), self.weight.data_ptr(),
            M, Vs, D, k, self.v0, words.data_ptr(), fine.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream()),
            "ShardedTwoStageHead.local")
        return words, fine

    def _merge_lib(self, words: torch.Tensor, fine: torch.Tensor, k: int, out=None):
        G, M, _ = words.shape
        if out is None:
            out = (torch.empty((M, k), dtype=torch.int32, device=words.device),
                   torch.empty((M, k), dtype=torch.bfloat16, device=words.device),
                   torch.empty((M,), dtype=torch.int32, device=words.device))
        idx, fv, amax = out
        _lib.check(_lib.lib().qmtp_lmhead2_merge(words.data_ptr(), fine.data_ptr(), G, M, k, idx.data_ptr(),
                                                 fv.data_ptr(), amax.data_ptr(), _lib.stream()),
                   "ShardedTwoStageHead.merge")
        return idx, fv, amax

    def select(self, h: torch.Tensor, k: int | None = None, out=None):
        """h [..., D] (the same on every rank) -> (idx int32 [M, k], fine bf16 [M, k], argmax int32 [M])."""
        import torch.distributed as dist

        k = self.k if k is None else k
        D = h.shape[-1]
        h2 = h.reshape(-1, D)
        if h2.stride(0) != D:
            h2 = h2.contiguous()
        M = h2.shape[0]
        words, fine = self._local(h2, k)
        G = self.world
        key = ("gather", M, k, words.device)
        if key not in self._ws:
            self._ws[key] = (torch.empty((G * M, k), dtype=torch.int64, device=words.device),
                             torch.empty((G * M, k), dtype=fine.dtype, device=words.device))
        all_w, all_f = self._ws[key]
        dist.all_gather_into_tensor(all_w, words.contiguous(), group=self.group)
        dist.all_gather_into_tensor(all_f, fine.contiguous(), group=self.group)
        if out is None:
            return self._merge(all_w.view(G, M, k), all_f.view(G, M, k), k)
        return self._merge(all_w.view(G, M, k), all_f.view(G, M, k), k, out)


def k_for(sampling) -> int:
    """lm_head2.py:32-36: 64 for greedy or top_k <= 32; else 4*top_k (top_k = 0 -> 256), max 2048."""
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
