"""Expert-parallel MoE decode over G ranks (torch.distributed; NCCL on B200, gloo for the CPU tests).

The reference's MoE experiment is single-device, batch 1 (experiments/deepseek_moe/kernels.py:133-155);
config 5 asks for the 64 routed experts sharded over 1/2/4/8 GPUs with all-to-all dispatch and combine.
Layout: rank r owns routed experts [r*E/G, (r+1)*E/G) and a copy of every shared expert; every rank holds
its own T tokens (weak scaling).  One layer:

  1. dispatch plan: each (token, slot) entry of a routed expert goes to the owner rank; entries are
     ordered by (destination rank, token, slot), which fixes the order of everything that follows;
  2. all-to-all of the per-peer counts (the layer's only host synchronisation: NCCL needs the split
     sizes), then of the token rows (bf16) and their local expert ids;
  3. one expert pass (qmtp_moe_experts) over the received rows followed by the rank's own
     shared-expert rows: one fp32 partial per row;
  4. all-to-all of the received rows' partials back to the token's rank (split sizes reversed);
  5. y[t] = sum_j scores[t, j] * partial(t, j) in slot order (qmtp_moe_combine) -- the same sum, in
     the same order, as the single-GPU kernel's combine.

With a fixed capacity per peer (`capacity=`) the layer makes no host synchronisation: the dispatch
kernel (qmtp_moe_dispatch) lays the rows out in equal slots of `capacity` rows per peer (empty slots
carry expert id -1), the all-to-alls use equal splits, and the combine reads every partial through a
position table computed on the device.  The whole layer can then be captured in one CUDA graph.

The expert computation, the combine and the fixed-capacity planner are pluggable (`compute`,
`combine_fn`, `dispatch`) so the identical dispatch logic runs with the CUDA kernels on GPUs and with
the C oracle in the gloo tests.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    """One MoE layer sharded expert-parallel over the default process group (or `group`).

    compute(x_rows, local_expert_ids, out=None) -> fp32 partials [n, H] (written into `out` when given):
    routed experts owned by this rank use local ids 0 .. E/G-1, shared expert s uses local id E/G + s,
    id -1 marks an empty row (its partial is not needed).
    combine_fn(partials, row_of [T, S], scores [T, S]) -> y [T, H]."""

    def __init__(self, n_routed: int, n_shared: int, compute, combine_fn, group=None, capacity=None, dispatch=None):
        self.n_routed, self.n_shared = n_routed, n_shared
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_routed % self.world:
            raise ValueError(f"{n_routed} routed experts do not split over {self.world} ranks")
        self.per = n_routed // self.world
        self.compute, self.combine_fn = compute, combine_fn
        # capacity=None: exact split sizes, one host synchronisation per layer.  capacity = int or
        # callable(T, S) -> int: fixed-capacity dispatch, no host synchronisation (the layer can be
        # captured in a CUDA graph together with its NCCL calls); it must cover the routed entries a
        # rank sends to any one rank (T * S always does).
        self.capacity = capacity
        self.dispatch = dispatch  # fixed-capacity planner; None = the CUDA kernel (qmtp.moe.dispatch)
        self._bufs = {}

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        if self.capacity is not None:
            return self._call_fixed(x, idx, scores)
        return self._call_exact(x, idx, scores)

    def _call_fixed(self, x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        T, S = idx.shape
        H = x.shape[-1]
        G, n, dev = self.world, T * S, x.device
        cap = int(self.capacity(T, S) if callable(self.capacity) else self.capacity)
        key = (T, S, H, cap, x.dtype, dev)
        b = self._bufs.get(key)
        if b is None:
            b = dict(send_x=torch.empty((G * cap, H), dtype=x.dtype, device=dev),
                     send_e=torch.empty((G * cap,), dtype=torch.int32, device=dev),
                     rows_x=torch.empty((G * cap + n, H), dtype=x.dtype, device=dev),
                     rows_e=torch.empty((G * cap + n,), dtype=torch.int32, device=dev),
                     pos=torch.empty((n,), dtype=torch.int32, device=dev),
                     counts=torch.empty((G + 1,), dtype=torch.int32, device=dev),
                     # [partials back from the ranks ; this rank's pass: received rows, shared rows]
                     table=torch.empty((2 * G * cap + n, H), dtype=torch.float32, device=dev))
            self._bufs = {key: b}
        plan = self.dispatch
        if plan is None:
            from .moe import dispatch as plan
        plan(idx, x, self.n_routed, self.n_shared, G, cap, b["send_x"], b["send_e"], b["rows_x"][G * cap:],
             b["rows_e"][G * cap:], b["pos"], b["counts"])
        wide = x.element_size() == 2 and H % 2 == 0
        rx, sx = b["rows_x"][:G * cap], b["send_x"]
        dist.all_to_all_single(rx.view(torch.int32) if wide else rx, sx.view(torch.int32) if wide else sx,
                               group=self.group)
        dist.all_to_all_single(b["rows_e"][:G * cap], b["send_e"], group=self.group)
        tab = b["table"]
        self.compute(b["rows_x"], b["rows_e"], out=tab[G * cap:])
        dist.all_to_all_single(tab[:G * cap], tab[G * cap:2 * G * cap], group=self.group)
        return self.combine_fn(tab, b["pos"].view(T, S), scores)

    def _call_exact(self, x: torch.Tensor, idx: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        T, S = idx.shape
        H = x.shape[-1]
        dev = x.device
        G, n_ent = self.world, T * S
        flat = idx.reshape(-1).to(torch.int64)
        # destination of every (t, j) entry: the owner rank of a routed expert, G for a shared one.
        # One stable order (dest, t, j) serves the dispatch (dest < G) and the local shared rows.
        dest = torch.where(flat < self.n_routed, torch.div(flat, self.per, rounding_mode="floor"),
                           torch.full_like(flat, G))
        order_all = torch.argsort(dest * n_ent + torch.arange(n_ent, device=dev))
        counts_all = torch.zeros(G + 1, dtype=torch.int64, device=dev).scatter_add_(0, dest, torch.ones_like(dest))
        recv_counts = torch.empty(G, dtype=torch.int64, device=dev)
        dist.all_to_all_single(recv_counts, counts_all[:G].contiguous(), group=self.group)
        host = torch.cat([counts_all, recv_counts]).tolist()  # the layer's one host synchronisation
        sc, n_sh, rc = host[:G], host[G], host[G + 1:]
        n_send, n_recv = sum(sc), sum(rc)
        order, sh = order_all[:n_send], order_all[n_send:]
        tok_all = torch.div(order_all, S, rounding_mode="floor")
        send_x = x.index_select(0, tok_all[:n_send]).contiguous()
        send_e = (flat[order] - dest[order] * self.per).to(torch.int32).contiguous()
        # the rows this rank computes: the routed rows it receives, then its own shared-expert rows
        rows_x = torch.empty((n_recv + n_sh, H), dtype=x.dtype, device=dev)
        rows_e = torch.empty((n_recv + n_sh,), dtype=torch.int32, device=dev)
        # 16-bit rows travel as int32 pairs (gloo has no 16-bit all-to-all; NCCL moves bytes either way)
        wide = x.element_size() == 2 and H % 2 == 0
        rx = rows_x[:n_recv]
        dist.all_to_all_single(rx.view(torch.int32) if wide else rx, send_x.view(torch.int32) if wide else send_x,
                               output_split_sizes=rc, input_split_sizes=sc, group=self.group)
        dist.all_to_all_single(rows_e[:n_recv], send_e, output_split_sizes=rc, input_split_sizes=sc,
                               group=self.group)
        rows_x[n_recv:] = x.index_select(0, tok_all[n_send:])
        rows_e[n_recv:] = (flat[sh] - self.n_routed + self.per).to(torch.int32)
        part = self.compute(rows_x, rows_e).contiguous()
        back = torch.empty((n_send, H), dtype=part.dtype, device=dev)
        dist.all_to_all_single(back, part[:n_recv], output_split_sizes=sc, input_split_sizes=rc, group=self.group)
        # row of every (t, j) entry in the table [back ; own shared rows]
        row_of = torch.empty((n_ent,), dtype=torch.int64, device=dev)
        row_of[order_all] = torch.arange(n_ent, device=dev)
        table = torch.cat([back, part[n_recv:]], 0)
        return self.combine_fn(table, row_of.reshape(T, S), scores)


def local_expert_table(wg, sg, wu, su, wd, sd, n_routed: int, n_shared: int, rank: int, world: int):
    """This rank's weight table: its routed shard followed by all shared experts (same layout as the
    single-GPU tensors, [E_local, N, K/8] / [E_local, N, K/G])."""
    per = n_routed // world
    sel = list(range(rank * per, (rank + 1) * per)) + list(range(n_routed, n_routed + n_shared))
    ix = torch.tensor(sel, device=wg.device)
    return tuple(t.index_select(0, ix).contiguous() for t in (wg, sg, wu, su, wd, sd))
