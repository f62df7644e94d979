"""A CPU stand-in for the MoEContext methods that hoard_b200.ep.ExpertParallel drives (route, ep_pack,
ep_experts, ep_combine), written with numpy over dequantised weights. It tests the expert-parallel
orchestration (partitioning, split sizes, the send-order map, combine order) on gloo ranks without
a GPU; the kernels themselves are tested on the GPU against the single-rank path.

Each row's arithmetic is a fixed sequence of float32 operations, so the expert-parallel result over
any number of ranks must equal the single-process result bit for bit, as on the GPU.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as orc
from tests.moe_fixtures import LayerData


def _silu(v):
    return v / (np.float32(1.0) + np.exp(-v))


class FakeContext:
    def __init__(self, L: LayerData, shuffle_seed: int = 0):
        s = L.spec
        self.H, self.E, self.k, self.I = s.H, s.E, s.k, s.I
        self.L = L
        self.gate = np.stack([orc.dequant(s.types[0], L.gate[e]).reshape(s.I, s.H) for e in range(s.E)])
        self.up = np.stack([orc.dequant(s.types[1], L.up[e]).reshape(s.I, s.H) for e in range(s.E)])
        self.down = np.stack([orc.dequant(s.types[2], L.down[e]).reshape(s.H, s.I) for e in range(s.E)])
        self.rng = np.random.default_rng(shuffle_seed)
        self.fx = None

    # graph A: RMSNorm, router, softmax over all experts, top-k (descending, ties to the lower id), renorm
    def route(self, layer, x, sel=None, w=None):
        s = self.L.spec
        xn = x.numpy().astype(np.float32)
        ms = (xn.astype(np.float64) ** 2).mean(-1, keepdims=True)
        fx = (xn / np.sqrt(ms + s.eps)).astype(np.float32) * self.L.w_norm
        self.fx = fx.astype(np.float32)
        logits = self.fx.astype(np.float64) @ self.L.w_router.astype(np.float64).T
        p = np.exp(logits - logits.max(-1, keepdims=True))
        p = p / p.sum(-1, keepdims=True)
        order = np.lexsort((np.arange(self.E)[None, :].repeat(len(p), 0), -p), axis=-1)[:, :self.k]
        ws = np.take_along_axis(p, order, -1).astype(np.float32)
        if s.renorm:
            ws = ws / np.maximum(ws.sum(-1, keepdims=True), np.float32(6.103515625e-5))
        return torch.from_numpy(order.astype(np.int32)), torch.from_numpy(ws.astype(np.float32))

    def ep_pack(self, layer, sel, n_ranks, experts_per_rank):
        sel_n = sel.numpy().reshape(-1)
        n = sel_n.size
        dest = sel_n // experts_per_rank
        counts = np.bincount(dest, minlength=n_ranks).astype(np.int32)
        starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
        pos = np.empty(n, np.int32)
        for r in range(n_ranks):                      # arbitrary order within a destination, as on the GPU
            idx = np.nonzero(dest == r)[0]
            pos[self.rng.permutation(idx)] = starts[r] + np.arange(idx.size)
        expert = np.empty(n, np.int32)
        rows = np.empty((n, self.H), np.float32)
        expert[pos] = sel_n
        rows[pos] = self.fx[np.arange(n) // self.k]
        return (torch.from_numpy(counts), torch.from_numpy(pos), torch.from_numpy(expert), torch.from_numpy(rows))

    def expert_row(self, e, row):
        h = (_silu(self.gate[e] @ row) * (self.up[e] @ row)).astype(np.float32)
        return (self.down[e] @ h).astype(np.float32)

    def ep_experts(self, layer, rows, slot_of_row, y_out=None):
        r = rows.numpy()
        s = slot_of_row.numpy()
        y = np.stack([self.expert_row(int(s[i]), r[i]) for i in range(len(s))]) if len(s) else np.zeros((0, self.H), np.float32)
        return torch.from_numpy(y.astype(np.float32))

    def ep_combine(self, w, pos, y_back, x):
        wn, pn, yb = w.numpy(), pos.numpy(), y_back.numpy()
        xn = x.numpy()
        T = xn.shape[0]
        for t in range(T):
            acc = np.zeros(self.H, np.float32)
            for j in range(self.k):
                acc = acc + wn[t, j] * yb[pn[t * self.k + j]]
            xn[t] = acc + xn[t]
        return x

    def reference_layer(self, x):
        """Single process: every entry's expert output in (t, j) order, the same combine."""
        sel, w = self.route(0, x)
        sn = sel.numpy()
        T = x.shape[0]
        y = np.stack([self.expert_row(int(sn[t, j]), self.fx[t]) for t in range(T) for j in range(self.k)])
        pos = torch.arange(T * self.k, dtype=torch.int32)
        return self.ep_combine(w, pos, torch.from_numpy(y), x), sel, w
