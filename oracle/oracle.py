"""ctypes loader for the CPU oracle (oracle/_build/liboracle.so) -- TEST INFRASTRUCTURE ONLY.

The oracle is the parity checker and the timed CPU baseline. Only tests/,
__graft_entry__.smoke() and bench.py's CPU legs import this module; the product library never
does. See moe_oracle.cpp for the reference call sites each function restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

MODE_GGML = 0   # activations quantized to Q8_K before each quantized matmul (ggml CPU backend)
MODE_EXACT = 1  # dequantized weights . f32 activations, double sums

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.orc_fp16_to_fp32.restype = ctypes.c_float
        _lib.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def fp16_to_fp32(h: int) -> float:
    return lib().orc_fp16_to_fp32(h)


def dequant(qtype: int, blocks: np.ndarray) -> np.ndarray:
    b = _u8(blocks).reshape(-1)
    bb = {12: 144, 14: 210}[qtype]
    nb = b.size // bb
    out = np.empty(nb * 256, np.float32)
    rc = lib().orc_dequant(ctypes.c_int(qtype), _p(b), ctypes.c_int64(nb), _p(out))
    if rc:
        raise ValueError(f"orc_dequant rc={rc}")
    return out


def quantize_q8k(x: np.ndarray):
    x = _f32(x).reshape(-1)
    n = x.size
    d = np.empty(n // 256, np.float32)
    qs = np.empty(n, np.int8)
    bs = np.empty(n // 16, np.int16)
    lib().orc_quantize_q8k_flat(_p(x), ctypes.c_int64(n), _p(d), _p(qs), _p(bs))
    return d, qs, bs


def matvec(qtype: int, W: np.ndarray, N: int, K: int, x: np.ndarray, mode: int = MODE_GGML):
    W = _u8(W) if qtype != 0 else _f32(W)
    x = _f32(x)
    y = np.empty(N, np.float32)
    rc = lib().orc_matvec(ctypes.c_int(qtype), _p(W), ctypes.c_int(N), ctypes.c_int(K), _p(x), _p(y),
                          ctypes.c_int(mode))
    if rc:
        raise ValueError(f"orc_matvec rc={rc}")
    return y


def route(x, w_norm, w_router, k: int, renorm: bool, eps: float, nthreads: int = 0):
    """Returns (fx [T,H], probs [T,E], sel [T,k] int32, w [T,k])."""
    x = _f32(x)
    T, H = x.shape
    E = w_router.shape[0]
    fx = np.empty((T, H), np.float32)
    probs = np.empty((T, E), np.float32)
    sel = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().orc_route(_p(x), ctypes.c_int(T), ctypes.c_int(H), ctypes.c_int(E), ctypes.c_int(k),
                    ctypes.c_int(int(renorm)), ctypes.c_float(eps), _p(_f32(w_norm)), _p(_f32(w_router)),
                    _p(fx), _p(probs), _p(sel), _p(w), ctypes.c_int(nthreads))
    return fx, probs, sel, w


def _shared_args(shared):
    if shared is None:
        return [ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), None, None, None, None], []
    keep = [_u8(shared["gate"]), _u8(shared["up"]), _u8(shared["down"]), _f32(shared["gate_inp"])]
    return [ctypes.c_int(shared["I"]), ctypes.c_int(shared["gate_type"]), ctypes.c_int(shared["up_type"]),
            ctypes.c_int(shared["down_type"]), _p(keep[0]), _p(keep[1]), _p(keep[2]), _p(keep[3])], keep


def experts(H, E, k, I, types, gate, up, down, fx, resid, sel, w, mode=MODE_GGML, nthreads=0, shared=None):
    """out[T,H] = (sum_j w_j * FFN_{sel_j}(fx) + shared) + resid."""
    fx, resid = _f32(fx), _f32(resid)
    T = fx.shape[0]
    sel = np.ascontiguousarray(sel, np.int32)
    w = _f32(w)
    out = np.empty((T, H), np.float32)
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    sh, keep = _shared_args(shared)
    rc = lib().orc_moe_experts(ctypes.c_int(H), ctypes.c_int(E), ctypes.c_int(k), ctypes.c_int(I),
                               ctypes.c_int(types[0]), ctypes.c_int(types[1]), ctypes.c_int(types[2]),
                               _p(gate), _p(up), _p(down), *sh, _p(fx), _p(resid), ctypes.c_int(T),
                               _p(sel), _p(w), ctypes.c_int(mode), ctypes.c_int(nthreads), _p(out))
    if rc:
        raise ValueError(f"orc_moe_experts rc={rc}")
    return out


def moe_layer(x, w_norm, w_router, gate, up, down, *, H, E, k, I, types, renorm, eps,
              mode=MODE_GGML, nthreads=0, shared=None):
    """Whole layer; returns (out [T,H], sel [T,k], w [T,k], fx [T,H], probs [T,E])."""
    x = _f32(x)
    T = x.shape[0]
    out = np.empty((T, H), np.float32)
    sel = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    fx = np.empty((T, H), np.float32)
    probs = np.empty((T, E), np.float32)
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    sh, keep = _shared_args(shared)
    rc = lib().orc_moe_layer(ctypes.c_int(H), ctypes.c_int(E), ctypes.c_int(k), ctypes.c_int(I),
                             ctypes.c_int(int(renorm)), ctypes.c_float(eps),
                             ctypes.c_int(types[0]), ctypes.c_int(types[1]), ctypes.c_int(types[2]),
                             _p(_f32(w_norm)), _p(_f32(w_router)), _p(gate), _p(up), _p(down), *sh,
                             _p(x), ctypes.c_int(T), ctypes.c_int(mode), ctypes.c_int(nthreads),
                             _p(out), _p(sel), _p(w), _p(fx), _p(probs))
    if rc:
        raise ValueError(f"orc_moe_layer rc={rc}")
    return out, sel, w, fx, probs


def max_threads() -> int:
    return lib().orc_max_threads()
