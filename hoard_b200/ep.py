"""Expert parallelism for batched tokens (prefill) over G ranks of one node.

Experts [g*E/G, (g+1)*E/G) are computed on rank g; tokens are data-parallel (each rank routes its
own T tokens). One MoE layer on one rank:

    route (local)  ->  ep_pack: (token, j) entries counting-sorted by destination rank, their
    Q8_K-quantised f16 rows gathered  ->  all-to-all of the per-destination counts, then of the rows
    and their expert ids  ->  ep_experts on the received rows (the tensor-core grouped GEMM)  ->
    all-to-all of the f16 outputs back (reverse splits)  ->  ep_combine: x[t] += sum_j w_j y_(t,j),
    j ascending.

The arithmetic of every row is independent of which rows share its tile and the outputs travel in the
f16 form the single-rank tensor-core path stores too, so G ranks reproduce it bit for bit.

Two transports:
  "nccl"  the exchange is torch.distributed all-to-all (NCCL on GPUs, gloo in the CPU tests), with a
          host read of the per-destination counts each layer;
  "p2p"   the library's own kernels over NVLink peer memory (hoard_moe_p2p_*): the pack kernel stores
          rows straight into the destination ranks' receive regions, the down-GEMM epilogue stores
          each output row straight into its source rank's y_back, and two bounded device barriers per
          layer order the steps; no host synchronisation and no collective library on the data path.
          torch.distributed only all-gathers the CUDA IPC handles once.

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
                 max_rows: int | None = None, chunks: int = 1, transport: str = "nccl"):
        self.ctx = ctx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E = ctx.E
        self.epr = experts_per_rank or (E + self.world - 1) // self.world
        if self.epr * self.world < E:
            raise ValueError("experts_per_rank * world must cover every expert")
        self.slot_base = 0 if slot_base is None else slot_base
        self.chunks = max(1, chunks)
        if transport not in ("nccl", "p2p"):
            raise ValueError("transport must be 'nccl' or 'p2p'")
        self.transport = transport
        self.last_recv_rows = 0
        if transport == "p2p":
            ctx.p2p_init(self.world, self.rank, self.epr, self.slot_base)
            ctx.p2p_open(self._all_gather_bytes(ctx.p2p_handle()))
        elif max_rows is not None and hasattr(ctx, "ep_reserve"):
            ctx.ep_reserve(max_rows)

    def _all_gather_bytes(self, blob: bytes):
        if dist.get_backend(self.group) == "nccl":
            dev = torch.device("cuda", torch.cuda.current_device())
        else:
            dev = torch.device("cpu")
        mine = torch.tensor(list(blob), dtype=torch.uint8, device=dev)
        out = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(out, mine, group=self.group)
        return [bytes(t.cpu().tolist()) for t in out]

    def close(self):
        """Unmaps the peers' blocks (p2p): every rank's kernels are done before any rank unmaps."""
        if self.transport == "p2p":
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self.ctx.p2p_close()
            dist.barrier(group=self.group)

    def _exchange(self, out, inp, out_splits, in_splits, async_op=False):
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=async_op)

    def layer(self, layer: int, x: torch.Tensor, sel_out: torch.Tensor | None = None,
              w_out: torch.Tensor | None = None):
        """One MoE layer on this rank's tokens x [T, H] (updated in place). Returns (x, sel, w)."""
        ctx = self.ctx
        T, H, k = x.shape[0], ctx.H, ctx.k
        if self.transport == "p2p":
            sel = sel_out if sel_out is not None else torch.empty(T, k, dtype=torch.int32, device=x.device)
            w = w_out if w_out is not None else torch.empty(T, k, dtype=torch.float32, device=x.device)
            ctx.p2p_layers(layer, 1, x, sel, w)
            return x, sel, w
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

    def layer_pipelined(self, layer: int, x: torch.Tensor):
        """The same layer with the tokens in `chunks` micro-batches whose exchanges are asynchronous:
        micro-batch i's expert GEMMs run while i+1's rows and i-1's outputs are in flight (the
        collectives run on the process group's own stream). Routing, rows and outputs are those of
        layer(), so the result is identical."""
        ctx = self.ctx
        T, H, G = x.shape[0], ctx.H, self.world
        n = self.chunks if T >= 2 * self.chunks else 1
        if n == 1:
            return self.layer(layer, x)[0]
        edges = [T * i // n for i in range(n + 1)]
        parts = []
        for i in range(n):
            xs = x[edges[i]:edges[i + 1]]
            sel, w = ctx.route(layer, xs)
            counts, pos, expert, rows = ctx.ep_pack(layer, sel, G, self.epr)
            parts.append({"x": xs, "w": w, "counts": counts, "pos": pos, "expert": expert, "rows": rows})
        # one exchange of every micro-batch's per-destination counts: send [G][n], receive [G][n]
        send_c = torch.stack([p["counts"] for p in parts], 1).contiguous()
        recv_c = torch.empty_like(send_c)
        self._exchange(recv_c, send_c, None, None)
        send_h, recv_h = send_c.cpu().tolist(), recv_c.cpu().tolist()
        total = 0
        for i, p in enumerate(parts):
            p["ss"] = [send_h[g][i] for g in range(G)]
            p["rs"] = [recv_h[g][i] for g in range(G)]
            ns, nr = sum(p["ss"]), sum(p["rs"])
            total += nr
            p["rrows"] = torch.empty(nr, H, dtype=p["rows"].dtype, device=x.device)
            p["rexp"] = torch.empty(nr, dtype=torch.int32, device=x.device)
            p["w_rows"] = self._exchange(p["rrows"], p["rows"][:ns], p["rs"], p["ss"], async_op=True)
            p["w_exp"] = self._exchange(p["rexp"], p["expert"][:ns], p["rs"], p["ss"], async_op=True)
        self.last_recv_rows = total
        for p in parts:
            p["w_rows"].wait()
            p["w_exp"].wait()
            slot = (p["rexp"] - self.rank * self.epr + self.slot_base).to(torch.int32)
            y = ctx.ep_experts(layer, p["rrows"], slot)
            p["yback"] = torch.empty(p["x"].shape[0] * ctx.k, H, dtype=y.dtype, device=x.device)
            p["w_y"] = self._exchange(p["yback"][:sum(p["ss"])], y, p["ss"], p["rs"], async_op=True)
            p["y"] = y                                    # alive until its exchange has run
        for p in parts:
            p["w_y"].wait()
            ctx.ep_combine(p["w"], p["pos"], p["yback"], p["x"])
        return x

    def layers(self, layer0: int, n_layers: int, x: torch.Tensor):
        if self.transport == "p2p":
            return self.ctx.p2p_layers(layer0, n_layers, x)
        for layer in range(layer0, layer0 + n_layers):
            if self.chunks > 1:
                self.layer_pipelined(layer, x)
            else:
                self.layer(layer, x)
        return x
