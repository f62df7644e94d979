"""Seeded MoE layers shared by the tests: weights, GGUF-layout expert bytes, and a loader that
puts one layer into a MoEContext. Sizes follow the benchmark configurations (Qwen3-30B-A3B shape:
H 2048, E 128, k 8, I 768, renorm, down Q6_K) or smaller stand-ins of the same structure."""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from hoard_b200 import quant

Q4_K, Q6_K = quant.Q4_K, quant.Q6_K


@dataclass
class LayerSpec:
    H: int
    E: int
    k: int
    I: int
    types: tuple = (Q4_K, Q4_K, Q6_K)
    renorm: bool = True
    eps: float = 1e-6
    shared: bool = False
    sh_types: tuple = (Q4_K, Q4_K, Q6_K)


@dataclass
class LayerData:
    spec: LayerSpec
    w_router: np.ndarray          # f32 [E, H]
    w_norm: np.ndarray            # f32 [H]
    gate: np.ndarray              # uint8 [E, I, rowbytes(H)]
    up: np.ndarray
    down: np.ndarray              # uint8 [E, H, rowbytes(I)]
    shared: dict | None = field(default=None)


def make_layer(spec: LayerSpec, seed: int, device: str = "cpu") -> LayerData:
    """Seeded weights drawn and quantised on `device` (a GPU draws and quantises the 128-expert
    layers of the benchmark shape in seconds); the bytes come back as numpy arrays either way."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, E, I = spec.H, spec.E, spec.I
    w_router = (torch.randn(E, H, generator=g, device=device) * 0.02).cpu().numpy()
    w_norm = (1.0 + 0.1 * torch.randn(H, generator=g, device=device)).cpu().numpy()

    def q(n_out, k_in, qt, n_exp):
        out = np.empty((n_exp, n_out, quant.row_bytes(qt, k_in)), np.uint8)
        for e0 in range(0, n_exp, 16):
            e1 = min(n_exp, e0 + 16)
            out[e0:e1] = quant.quantize(torch.randn(e1 - e0, n_out, k_in, generator=g, device=device) * 0.02,
                                        qt).cpu().numpy()
        return out

    gate = q(I, H, spec.types[0], E)
    up = q(I, H, spec.types[1], E)
    down = q(H, I, spec.types[2], E)
    shared = None
    if spec.shared:
        shared = dict(I=I, gate_type=spec.sh_types[0], up_type=spec.sh_types[1], down_type=spec.sh_types[2],
                      gate=q(I, H, spec.sh_types[0], 1)[0], up=q(I, H, spec.sh_types[1], 1)[0],
                      down=q(H, I, spec.sh_types[2], 1)[0],
                      gate_inp=(torch.randn(H, generator=g, device=device) * 0.02).cpu().numpy())
    return LayerData(spec, w_router, w_norm, gate, up, down, shared)


def make_x(T: int, H: int, seed: int) -> np.ndarray:
    """Residual input: N(0,1) rows, RMS-normalised (the benchmark's activation distribution)."""
    g = torch.Generator().manual_seed(seed + 1_000_003)
    x = torch.randn(T, H, generator=g)
    x = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)
    return x.numpy().astype(np.float32)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_layer(L: LayerData, x: np.ndarray, mode: int, nthreads: int = 0):
    from oracle import oracle as orc
    s = L.spec
    return orc.moe_layer(x, L.w_norm, L.w_router, L.gate, L.up, L.down, H=s.H, E=s.E, k=s.k, I=s.I,
                         types=s.types, renorm=s.renorm, eps=s.eps, mode=mode, nthreads=nthreads, shared=L.shared)


def load_context(ctx, layer: int, L: LayerData, slot_of_expert=None):
    """Uploads one layer into a MoEContext (router, experts into slots, shared expert)."""
    dev = torch.device("cuda", ctx.device)
    ctx.set_router(layer, torch.from_numpy(L.w_router).to(dev), torch.from_numpy(L.w_norm).to(dev))
    gate = torch.from_numpy(L.gate).to(dev)
    up = torch.from_numpy(L.up).to(dev)
    down = torch.from_numpy(L.down).to(dev)
    experts = range(L.spec.E) if slot_of_expert is None else slot_of_expert.keys()
    for e in experts:
        slot = e if slot_of_expert is None else slot_of_expert[e]
        ctx.upload_expert(layer, slot, gate[e], up[e], down[e])
    if L.shared is not None:
        sh = L.shared
        ctx.set_shared(layer, torch.from_numpy(sh["gate"]).to(dev), torch.from_numpy(sh["up"]).to(dev),
                       torch.from_numpy(sh["down"]).to(dev), torch.from_numpy(sh["gate_inp"]).to(dev))
    torch.cuda.synchronize(dev)


def near_tie_mask(probs: np.ndarray, sel: np.ndarray, k: int, gap: float = 1e-3) -> np.ndarray:
    """Tokens whose k-th and (k+1)-th routing scores differ by less than `gap` (selection ambiguous)."""
    srt = -np.sort(-probs, axis=1)
    if probs.shape[1] <= k:
        return np.zeros(probs.shape[0], bool)
    lp = np.log(np.maximum(srt, 1e-30))
    return (lp[:, k - 1] - lp[:, k]) < gap
