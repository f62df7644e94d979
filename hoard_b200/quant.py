"""Q4_K / Q6_K block encoders and seeded synthetic MoE weights.

hoard itself never quantizes: it reads Q4_K_M GGUF files produced elsewhere
(notes/model_url.txt in the hoard project). The seeded models used by the tests and the
benchmark are therefore quantized here by an encoder written from the GGUF block format:

* Q4_K, 256 weights in 144 bytes: fp16 d, fp16 dmin, 12 bytes of packed 6-bit
  (scale, min) pairs for 8 sub-blocks of 32, then 128 bytes of 4-bit quants where byte
  32*g + l holds element 64*g + l in its low nibble and element 64*g + 32 + l in its high
  nibble.  Decoded value = (d*sc) * q - (dmin*m).
* Q6_K, 256 weights in 210 bytes: 128 bytes of low 4 bits, 64 bytes of high 2 bits,
  16 int8 sub-block scales (one per 16 weights), fp16 d.  Decoded value = d*sc*(q - 32).

The encoder is a plain min/max fit (not ggml's iterative search); both the CPU oracle and the
CUDA kernels consume the same bytes, so the choice of encoder does not affect parity.
All functions accept CPU or CUDA tensors and return uint8 tensors on the same device, laid out
as GGUF stores a weight with ne = [K_in, N_out(, E)]: N_out rows of K_in/256 blocks.
"""
from __future__ import annotations

import torch

QK = 256
Q4_K, Q6_K = 12, 14  # GGUF / ggml type ids
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}


def row_bytes(qtype: int, k: int) -> int:
    """Bytes of one quantized row of k weights."""
    if k % QK:
        raise ValueError(f"row length {k} is not a multiple of {QK}")
    return (k // QK) * BLOCK_BYTES[qtype]


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    return v.to(torch.float16).contiguous().view(torch.uint8).reshape(*v.shape, 2)


def quantize_q4k(w: torch.Tensor) -> torch.Tensor:
    """Encodes w[..., K] (K % 256 == 0) into Q4_K blocks; returns uint8 [..., K/256*144]."""
    *lead, k = w.shape
    nb = k // QK
    if k % QK:
        raise ValueError("K must be a multiple of 256")
    x = w.reshape(-1, nb, 8, 32).float()
    r = x.shape[0]
    mn = x.amin(-1).clamp(max=0.0)
    mneg = -mn
    scale = (x.amax(-1) - mn) / 15.0
    d16 = (scale.amax(-1) / 63.0).to(torch.float16)
    dmin16 = (mneg.amax(-1) / 63.0).to(torch.float16)
    df, dminf = d16.float()[..., None], dmin16.float()[..., None]
    zero = torch.zeros((), device=x.device)
    sc = torch.where(df > 0, torch.round(scale / torch.where(df > 0, df, 1.0)), zero).clamp(0, 63)
    mq = torch.where(dminf > 0, torch.round(mneg / torch.where(dminf > 0, dminf, 1.0)), zero).clamp(0, 63)
    step = (df * sc)[..., None]
    off = (dminf * mq)[..., None]
    q = torch.where(step > 0, torch.round((x + off) / torch.where(step > 0, step, 1.0)), zero)
    q = q.clamp(0, 15).to(torch.uint8)
    sc8, mq8 = sc.to(torch.uint8), mq.to(torch.uint8)
    scales = torch.empty(r, nb, 12, dtype=torch.uint8, device=x.device)
    scales[..., 0:4] = sc8[..., 0:4] | ((sc8[..., 4:8] >> 4) << 6)
    scales[..., 4:8] = mq8[..., 0:4] | ((mq8[..., 4:8] >> 4) << 6)
    scales[..., 8:12] = (sc8[..., 4:8] & 0xF) | ((mq8[..., 4:8] & 0xF) << 4)
    qv = q.reshape(r, nb, 4, 2, 32)
    qs = (qv[..., 0, :] | (qv[..., 1, :] << 4)).reshape(r, nb, 128)
    blk = torch.cat([_f16_bytes(d16), _f16_bytes(dmin16), scales, qs], dim=-1)
    return blk.reshape(*lead, nb * 144)


def quantize_q6k(w: torch.Tensor) -> torch.Tensor:
    """Encodes w[..., K] (K % 256 == 0) into Q6_K blocks; returns uint8 [..., K/256*210]."""
    *lead, k = w.shape
    nb = k // QK
    if k % QK:
        raise ValueError("K must be a multiple of 256")
    x = w.reshape(-1, nb, 16, 16).float()
    r = x.shape[0]
    scale = x.abs().amax(-1) / 31.0
    d16 = (scale.amax(-1) / 127.0).to(torch.float16)
    df = d16.float()[..., None]
    zero = torch.zeros((), device=x.device)
    sc = torch.where(df > 0, torch.round(scale / torch.where(df > 0, df, 1.0)), zero).clamp(-128, 127)
    step = (df * sc)[..., None]
    q = torch.where(step != 0, torch.round(x / torch.where(step != 0, step, 1.0)), zero)
    q = (q.clamp(-32, 31) + 32).to(torch.uint8).reshape(r, nb, 2, 4, 32)
    ql = torch.empty(r, nb, 2, 64, dtype=torch.uint8, device=x.device)
    ql[..., 0:32] = (q[:, :, :, 0] & 0xF) | ((q[:, :, :, 2] & 0xF) << 4)
    ql[..., 32:64] = (q[:, :, :, 1] & 0xF) | ((q[:, :, :, 3] & 0xF) << 4)
    qh = ((q[:, :, :, 0] >> 4) | ((q[:, :, :, 1] >> 4) << 2) | ((q[:, :, :, 2] >> 4) << 4)
          | ((q[:, :, :, 3] >> 4) << 6))
    sc8 = sc.to(torch.int8).view(torch.uint8)
    blk = torch.cat([ql.reshape(r, nb, 128), qh.reshape(r, nb, 64), sc8, _f16_bytes(d16)], dim=-1)
    return blk.reshape(*lead, nb * 210)


def quantize(w: torch.Tensor, qtype: int) -> torch.Tensor:
    if qtype == Q4_K:
        return quantize_q4k(w)
    if qtype == Q6_K:
        return quantize_q6k(w)
    raise ValueError(f"unsupported quant type {qtype}")


def _normal(shape, std: float, gen: torch.Generator, device) -> torch.Tensor:
    return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std


def synth_experts(E: int, n_out: int, k_in: int, qtype: int, seed: int, device="cpu",
                  std: float = 0.02, chunk: int = 16) -> torch.Tensor:
    """E experts of an [n_out x k_in] weight drawn N(0, std) and quantized; uint8 [E, n_out, rowbytes].

    Generated in chunks of experts so that full-size layers fit comfortably on the device.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = torch.empty(E, n_out, row_bytes(qtype, k_in), dtype=torch.uint8, device=device)
    for e0 in range(0, E, chunk):
        e1 = min(E, e0 + chunk)
        out[e0:e1] = quantize(_normal((e1 - e0, n_out, k_in), std, gen, device), qtype)
    return out
