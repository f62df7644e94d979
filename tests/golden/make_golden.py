"""Generates tests/golden/kquant_golden.npz: Q4_K / Q6_K blocks and their decoded values.

The decoded values come from `gguf.quants` (gguf-py 0.19.0, MIT, the Python package of the
ggml / llama.cpp project whose Q4_K / Q6_K formats hoard's Q4_K_M models use). It is not vendored
in the hoard tree; it is installed in this image and used here, offline, only to produce these
vectors. The blocks are a mix of
  * blocks encoded by hoard_b200.quant from seeded N(0, 0.02) rows (the benchmark's weights),
  * random bytes with hand-picked fp16 scale words: zero, negative, subnormal, max-normal-ish,
    and all-ones 6-bit scales/mins,
so that every bit field of both formats is exercised.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def main():
    import torch
    import gguf.quants as gq
    from gguf import GGMLQuantizationType as QT

    from hoard_b200 import quant

    rng = np.random.default_rng(20241201)
    out = {}
    g = torch.Generator().manual_seed(7)
    w = torch.randn(8, 1024, generator=g) * 0.02
    for name, qt, gt, bb in (("q4k", quant.Q4_K, QT.Q4_K, 144), ("q6k", quant.Q6_K, QT.Q6_K, 210)):
        enc = quant.quantize(w, qt).numpy().reshape(-1, bb)
        rnd = rng.integers(0, 256, size=(24, bb), dtype=np.uint8)
        special = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x8123, 0x7BFF, 0x3C00, 0xBC00], dtype=np.uint16)
        for i, h in enumerate(special):
            hb = np.frombuffer(h.tobytes(), dtype=np.uint8)
            if qt == quant.Q4_K:
                rnd[i, 0:2] = hb           # d
                rnd[i + 8, 2:4] = hb       # dmin
            else:
                rnd[i, 208:210] = hb       # d
        # avoid inf/nan scale words elsewhere (exponent field 31)
        if qt == quant.Q4_K:
            for off in (0, 2):
                hi = rnd[:, off + 1]
                rnd[:, off + 1] = np.where((hi & 0x7C) == 0x7C, hi & 0xBF, hi)
            rnd[16, 4:16] = 0xFF           # all 6-bit scales and mins at 63
        else:
            hi = rnd[:, 209]
            rnd[:, 209] = np.where((hi & 0x7C) == 0x7C, hi & 0xBF, hi)
            rnd[16, 192:208] = 0x80        # int8 scales at -128
        blocks = np.concatenate([enc, rnd], axis=0)
        vals = gq.dequantize(blocks.reshape(-1), gt).reshape(-1, 256).astype(np.float32)
        out[f"{name}_blocks"] = blocks
        out[f"{name}_values"] = vals
        out[f"{name}_source_row"] = w.numpy()
    np.savez_compressed(os.path.join(HERE, "kquant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "kquant_golden.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
