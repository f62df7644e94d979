"""Expert parallelism for batched tokens (prefill) over G ranks of one node.

Experts [g*E/G, (g+1)*E/G) are computed on rank g; tokens are data-parallel (each rank routes its
own T tokens). One MoE layer on one rank:

    route (local)  ->  ep_pack: (token, j) entries counting-sorted by destination rank, their
    Q8_K-quantised f16 rows gathered  ->  all-to-all of the per-destination counts, then of the rows
    and their expert ids  ->  ep_experts on the received rows (the tensor-core grouped GEMM)  ->
    all-to-all of the f16 outputs back (reverse splits)  ->  ep_combine: x[t] += sum_j w_j y_(t,j),
    j ascending.

The arithmetic of every row is independent of which rows share its tile and the outputs travel in the
f16 form the single-rank tensor-core path stores too, so G ranks reproduce it bit for bit. The exchange uses torch.distributed
(NCCL on GPUs, gloo in the CPU tests): plain all-to-all collectives; no kernel reads peer memory.

hoard has no multi-GPU path; this is the sharded form of its batched mul_mat_id
(src/run_specloop.cpp:125-140).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallel:
    """Drives ctx (a MoEContext, or any object with the same route / ep_* methods) over a process group.

    slot_base: pool slot of this rank's first expert. 0 when the context holds only the rank's own
    experts in slots 0..E/G-1; rank*E/G when every expert is resident (slot = expert id).
    """

    def __init__(self, ctx, group=None, experts_per_rank: int | None = None, slot_base: int | None = None,
                 max_rows: int | None = None):
        self.ctx = ctx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E = ctx.E
        self.epr = experts_per_rank or (E + self.world - 1) // self.world
        if self.epr * self.world < E:
            raise ValueError("experts_per_rank * world must cover every expert")
        self.slot_base = 0 if slot_base is None else slot_base
        if max_rows is not None and hasattr(ctx, "ep_reserve"):
            ctx.ep_reserve(max_rows)
        self.last_recv_rows = 0

    def _exchange(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def layer(self, layer: int, x: torch.Tensor, sel_out: torch.Tensor | None = None,
              w_out: torch.Tensor | None = None):
        """One MoE layer on this rank's tokens x [T, H] (updated in place). Returns (x, sel, w)."""
        ctx = self.ctx
        T, H, k = x.shape[0], ctx.H, ctx.k
        sel, w = ctx.route(layer, x, sel_out, w_out)
        counts, pos, expert, rows = ctx.ep_pack(layer, sel, self.world, self.epr)
        recv_counts = torch.empty_like(counts)
        self._exchange(recv_counts, counts, None, None)
        send_splits = counts.tolist()
        recv_splits = recv_counts.tolist()
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        self.last_recv_rows = n_recv
        recv_rows = torch.empty(n_recv, H, dtype=rows.dtype, device=rows.device)
        recv_expert = torch.empty(n_recv, dtype=torch.int32, device=rows.device)
        self._exchange(recv_rows, rows[:n_send], recv_splits, send_splits)
        self._exchange(recv_expert, expert[:n_send], recv_splits, send_splits)
        slot = (recv_expert - self.rank * self.epr + self.slot_base).to(torch.int32)
        y = ctx.ep_experts(layer, recv_rows, slot)
        y_back = torch.empty(T * k, H, dtype=y.dtype, device=rows.device)
        self._exchange(y_back[:n_send], y, send_splits, recv_splits)
        ctx.ep_combine(w, pos, y_back, x)
        return x, sel, w

    def layers(self, layer0: int, n_layers: int, x: torch.Tensor):
        for layer in range(layer0, layer0 + n_layers):
            self.layer(layer, x)
        return x
