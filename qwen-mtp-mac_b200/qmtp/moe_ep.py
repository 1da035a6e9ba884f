"""Expert-parallel MoE decode over G ranks (torch.distributed; NCCL on B200, gloo for the CPU tests).

The reference's MoE experiment is single-device, batch 1 (experiments/deepseek_moe/kernels.py:133-155);
config 5 asks for the 64 routed experts sharded over 1/2/4/8 GPUs with all-to-all dispatch and combine.
Layout: rank r owns routed experts [r*E/G, (r+1)*E/G) and a copy of every shared expert; every rank holds
its own T tokens (weak scaling).  One layer:

  1. dispatch plan: each (token, slot) entry of a routed expert goes to the owner rank; entries are
     ordered by (destination rank, token, slot), which fixes the order of everything that follows;
  2. all-to-all of the per-peer counts, then of the token rows (bf16) and their local expert ids;
  3. the owner computes one fp32 partial per received row (qmtp_moe_experts);
  4. all-to-all of the partials back to the token's rank (same split sizes, reversed);
  5. shared experts run locally on the rank's own tokens;
  6. y[t] = sum_j scores[t, j] * partial(t, j) in slot order (qmtp_moe_combine) -- the same sum, in
     the same order, as the single-GPU kernel's combine.

The expert computation and the combine are pluggable (`compute`, `combine_fn`) so the identical
dispatch logic runs with the CUDA kernels on GPUs and with the C oracle in the gloo tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def plan_dispatch(idx: torch.Tensor, n_routed: int, world: int):
    """idx int [T, S] -> (order, dest, counts): routed entries (flat t*S + j) in (dest, t, j) order."""
    T, S = idx.shape
    flat = idx.reshape(-1).to(torch.int64)
    per = n_routed // world
    routed = flat < n_routed
    ent = torch.nonzero(routed, as_tuple=False).reshape(-1)  # ascending = (t, j) order
    dest = torch.div(flat[ent], per, rounding_mode="floor")
    key = dest * (T * S) + ent
    order = ent[torch.argsort(key)]
    dest_sorted = torch.div(flat[order], per, rounding_mode="floor")
    counts = torch.bincount(dest_sorted, minlength=world)
    return order, dest_sorted, counts


class ExpertParallelMoE:
    """One MoE layer sharded expert-parallel over the default process group (or `group`).

    compute(x_rows, local_expert_ids) -> fp32 partials [n, H]: routed experts owned by this rank use
    local ids 0 .. E/G-1; shared expert s uses local id E/G + s.
    combine_fn(partials, row_of [T, S], scores [T, S]) -> y [T, H]."""

    def __init__(self, n_routed: int, n_shared: int, compute, combine_fn, group=None):
        self.n_routed, self.n_shared = n_routed, n_shared
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_routed % self.world:
            raise ValueError(f"{n_routed} routed experts do not split over {self.world} ranks")
        self.per = n_routed // self.world
        self.compute, self.combine_fn = compute, combine_fn

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        T, S = idx.shape
        H = x.shape[-1]
        dev = x.device
        order, dest, counts = plan_dispatch(idx, self.n_routed, self.world)
        tok = torch.div(order, S, rounding_mode="floor")
        send_x = x.index_select(0, tok).contiguous()
        send_e = (idx.reshape(-1)[order].to(torch.int64) - dest * self.per).to(torch.int32).contiguous()
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        sc = counts.tolist()
        rc = recv_counts.tolist()
        recv_x = torch.empty((sum(rc), H), dtype=x.dtype, device=dev)
        recv_e = torch.empty((sum(rc),), dtype=torch.int32, device=dev)
        # 16-bit rows travel as int32 pairs (gloo has no 16-bit all-to-all; NCCL moves bytes either way)
        wide = x.element_size() == 2 and H % 2 == 0
        dist.all_to_all_single(recv_x.view(torch.int32) if wide else recv_x,
                               send_x.view(torch.int32) if wide else send_x,
                               output_split_sizes=rc, input_split_sizes=sc, group=self.group)
        dist.all_to_all_single(recv_e, send_e, output_split_sizes=rc, input_split_sizes=sc, group=self.group)
        part = self.compute(recv_x, recv_e).contiguous()
        back = torch.empty((len(order), H), dtype=part.dtype, device=dev)
        dist.all_to_all_single(back, part, output_split_sizes=sc, input_split_sizes=rc, group=self.group)
        # shared experts on this rank's own tokens
        flat = idx.reshape(-1).to(torch.int64)
        sh = torch.nonzero(flat >= self.n_routed, as_tuple=False).reshape(-1)
        sh_x = x.index_select(0, torch.div(sh, S, rounding_mode="floor")).contiguous()
        sh_e = (flat[sh] - self.n_routed + self.per).to(torch.int32).contiguous()
        sh_part = self.compute(sh_x, sh_e).contiguous()
        # row of every (t, j) entry in the table [back ; sh_part]
        row_of = torch.full((T * S,), -1, dtype=torch.int64, device=dev)
        row_of[order] = torch.arange(len(order), device=dev)
        row_of[sh] = len(order) + torch.arange(len(sh), device=dev)
        table = torch.cat([back, sh_part], 0)
        return self.combine_fn(table, row_of.reshape(T, S), scores)


def local_expert_table(wg, sg, wu, su, wd, sd, n_routed: int, n_shared: int, rank: int, world: int):
    """This rank's weight table: its routed shard followed by all shared experts (same layout as the
    single-GPU tensors, [E_local, N, K/8] / [E_local, N, K/G])."""
    per = n_routed // world
    sel = list(range(rank * per, (rank + 1) * per)) + list(range(n_routed, n_routed + n_shared))
    ix = torch.tensor(sel, device=wg.device)
    return tuple(t.index_select(0, ix).contiguous() for t in (wg, sg, wu, su, wd, sd))
