"""Python host mirror of the C ABI in include/hoard_moe.h.

`MoEContext` wraps one hoard_moe_ctx. Its methods keep the C names (route, experts, layer,
upload_expert, set_router, set_shared) and their argument meaning; a non-zero status raises
`HoardError` carrying the status code and the context's last error message. Tensors are torch
CUDA tensors (torch is used for device memory and streams only; the arithmetic runs in the
library's own kernels). The library is loaded from this package directory and there is no
fallback: if it is missing, `lib()` raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

from .quant import Q4_K, Q6_K, row_bytes

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libhoard_moe.so")

HOARD_OK = 0
HOARD_EINVAL = -1
HOARD_ENOMEM = -2
HOARD_ECUDA = -3
HOARD_ETIMEOUT = -4
HOARD_ENCCL = -5
HOARD_ESTATE = -6

TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_BF16 = 0, 12, 14, 30

EXPORTED = [
    "hoard_moe_create", "hoard_moe_destroy", "hoard_moe_set_router", "hoard_moe_upload_expert",
    "hoard_moe_set_shared", "hoard_moe_route", "hoard_moe_experts", "hoard_moe_layer", "hoard_moe_layers",
    "hoard_moe_sync_status", "hoard_moe_expert_bytes", "hoard_moe_launch_count", "hoard_moe_set_decode_impl",
    "hoard_moe_set_trace", "hoard_moe_trace_layout", "hoard_moe_decode_noalloc", "hoard_moe_decode_noalloc_status",
    "hoard_moe_set_gemm_min_tokens", "hoard_moe_set_gemm_ctas", "hoard_moe_set_top_k", "hoard_moe_ep_reserve", "hoard_moe_ep_pack", "hoard_moe_ep_experts",
    "hoard_moe_ep_combine", "hoard_moe_ram_tier", "hoard_moe_ensure", "hoard_moe_residency_stats",
    "hoard_moe_p2p_init", "hoard_moe_p2p_handle", "hoard_moe_p2p_open", "hoard_moe_p2p_attach", "hoard_moe_p2p_close",
    "hoard_moe_p2p_set_timeout", "hoard_moe_p2p_send", "hoard_moe_p2p_compute", "hoard_moe_p2p_finish",
    "hoard_moe_p2p_layers", "hoard_moe_last_error", "hoard_strerror",
]

P2P_HANDLE_BYTES = 128


class Desc(ctypes.Structure):
    _fields_ = [
        ("n_embd", ctypes.c_int), ("n_expert", ctypes.c_int), ("n_expert_used", ctypes.c_int),
        ("n_ff", ctypes.c_int), ("n_layer", ctypes.c_int), ("n_slots", ctypes.c_int),
        ("norm_topk", ctypes.c_int), ("eps", ctypes.c_float), ("resid_type", ctypes.c_int),
        ("gate_types", ctypes.POINTER(ctypes.c_int)), ("up_types", ctypes.POINTER(ctypes.c_int)),
        ("down_types", ctypes.POINTER(ctypes.c_int)), ("n_ff_shexp", ctypes.c_int),
        ("shexp_gate_type", ctypes.c_int), ("shexp_up_type", ctypes.c_int), ("shexp_down_type", ctypes.c_int),
        ("max_tokens", ctypes.c_int), ("device", ctypes.c_int),
    ]


class HoardError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"hoard status {status}: {msg}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libhoard_moe.so; raises if it has not been built (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m hoard_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.hoard_moe_create.argtypes = [ctypes.POINTER(Desc), ctypes.POINTER(vp)]
        L.hoard_moe_destroy.argtypes = [vp]
        L.hoard_moe_set_router.argtypes = [vp, i32, vp, vp]
        L.hoard_moe_upload_expert.argtypes = [vp, i32, i32, vp, vp, vp, vp]
        L.hoard_moe_set_shared.argtypes = [vp, i32, vp, vp, vp, vp]
        L.hoard_moe_route.argtypes = [vp, i32, vp, i32, vp, vp, vp]
        L.hoard_moe_experts.argtypes = [vp, i32, vp, vp, vp, vp, vp, i32, vp]
        L.hoard_moe_layer.argtypes = [vp, i32, vp, i32, vp, vp, vp]
        L.hoard_moe_layers.argtypes = [vp, i32, i32, vp, i32, vp, vp, vp]
        L.hoard_moe_sync_status.argtypes = [vp, vp]
        L.hoard_moe_expert_bytes.argtypes = [vp, i32]
        L.hoard_moe_expert_bytes.restype = i64
        L.hoard_moe_launch_count.argtypes = [vp]
        L.hoard_moe_launch_count.restype = i64
        L.hoard_moe_set_decode_impl.argtypes = [vp, i32]
        L.hoard_moe_set_gemm_min_tokens.argtypes = [vp, i32]
        L.hoard_moe_set_gemm_ctas.argtypes = [vp, i32]
        L.hoard_moe_set_top_k.argtypes = [vp, i32]
        L.hoard_moe_ram_tier.argtypes = [vp, i32, i32, vp, vp, vp]
        L.hoard_moe_ensure.argtypes = [vp, i32, vp, i32, vp, vp]
        L.hoard_moe_residency_stats.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.hoard_moe_ep_reserve.argtypes = [vp, i64]
        L.hoard_moe_ep_pack.argtypes = [vp, i32, vp, i32, i32, i32, vp, vp, vp, vp, vp]
        L.hoard_moe_ep_experts.argtypes = [vp, i32, vp, vp, i32, vp, vp]
        L.hoard_moe_ep_combine.argtypes = [vp, vp, vp, vp, vp, i32, vp]
        L.hoard_moe_p2p_init.argtypes = [vp, i32, i32, i32, i32]
        L.hoard_moe_p2p_handle.argtypes = [vp, vp]
        L.hoard_moe_p2p_open.argtypes = [vp, vp]
        L.hoard_moe_p2p_attach.argtypes = [vp, vp]
        L.hoard_moe_p2p_close.argtypes = [vp]
        L.hoard_moe_p2p_set_timeout.argtypes = [vp, ctypes.c_double]
        L.hoard_moe_p2p_send.argtypes = [vp, i32, vp, i32, vp, vp, vp]
        L.hoard_moe_p2p_compute.argtypes = [vp, vp]
        L.hoard_moe_p2p_finish.argtypes = [vp, vp, vp]
        L.hoard_moe_p2p_layers.argtypes = [vp, i32, i32, vp, i32, vp, vp, vp]
        L.hoard_moe_set_trace.argtypes = [vp, vp, i64]
        L.hoard_moe_decode_noalloc.argtypes = [vp, i32, i32, vp, vp, vp, vp]
        L.hoard_moe_decode_noalloc_status.argtypes = [vp, vp]
        L.hoard_moe_trace_layout.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        L.hoard_moe_last_error.argtypes = [vp]
        L.hoard_moe_last_error.restype = ctypes.c_char_p
        L.hoard_strerror.argtypes = [i32]
        L.hoard_strerror.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


class MoEContext:
    """One MoE layer stack on one GPU: HBM expert pool [n_layer][n_slots], router weights, scratch."""

    def __init__(self, *, n_embd: int, n_expert: int, n_expert_used: int, n_ff: int, n_layer: int = 1,
                 n_slots: int | None = None, norm_topk: bool = True, eps: float = 1e-6,
                 resid_dtype: torch.dtype = torch.float32, gate_types=None, up_types=None, down_types=None,
                 n_ff_shexp: int = 0, shexp_types=(Q4_K, Q4_K, Q6_K), max_tokens: int = 16, device: int = 0):
        self.H, self.E, self.k, self.I, self.n_layer = n_embd, n_expert, n_expert_used, n_ff, n_layer
        self.n_slots = n_expert if n_slots is None else n_slots
        self.resid_dtype = resid_dtype
        self.device = device
        self.max_tokens = max_tokens
        self.gate_types = list(gate_types) if gate_types is not None else [Q4_K] * n_layer
        self.up_types = list(up_types) if up_types is not None else [Q4_K] * n_layer
        self.down_types = list(down_types) if down_types is not None else [Q6_K] * n_layer
        self.n_ff_shexp = n_ff_shexp
        self.shexp_types = tuple(shexp_types)
        arr = ctypes.c_int * n_layer
        self._types = (arr(*self.gate_types), arr(*self.up_types), arr(*self.down_types))
        d = Desc(n_embd, n_expert, n_expert_used, n_ff, n_layer, self.n_slots, int(norm_topk), eps,
                 TYPE_BF16 if resid_dtype == torch.bfloat16 else TYPE_F32,
                 self._types[0], self._types[1], self._types[2], n_ff_shexp,
                 self.shexp_types[0], self.shexp_types[1], self.shexp_types[2], max_tokens, device)
        h = ctypes.c_void_p()
        rc = lib().hoard_moe_create(ctypes.byref(d), ctypes.byref(h))
        if rc != HOARD_OK:
            raise HoardError(rc, "hoard_moe_create: " + lib().hoard_strerror(rc).decode())
        self._h = h

    # -- plumbing ----------------------------------------------------------------------------
    def _check(self, rc: int, what: str):
        if rc != HOARD_OK:
            msg = lib().hoard_moe_last_error(self._h).decode()
            raise HoardError(rc, f"{what}: {msg}")

    def close(self):
        if getattr(self, "_h", None):
            lib().hoard_moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def launch_count(self) -> int:
        return lib().hoard_moe_launch_count(self._h)

    def expert_bytes(self, layer: int) -> int:
        return lib().hoard_moe_expert_bytes(self._h, layer)

    def set_decode_impl(self, impl: int):
        self._check(lib().hoard_moe_set_decode_impl(self._h, impl), "set_decode_impl")

    # ---- residency: LRU slot pool over a host RAM tier ----
    def ram_tier(self, layer: int, expert: int, gate, up, down):
        """Registers host copies (raw GGUF bytes: CPU tensors, ideally pinned; kept alive by the caller)."""
        self._check(lib().hoard_moe_ram_tier(self._h, layer, expert, _ptr(gate), _ptr(up), _ptr(down)), "ram_tier")

    def ensure(self, layer: int, sel, stream=None):
        """Slots for the expert ids in sel (host int32 array); misses are uploaded from the RAM tier."""
        import numpy as np
        sel_h = np.ascontiguousarray(np.asarray(sel, dtype=np.int32).reshape(-1))
        out = np.empty_like(sel_h)
        self._check(lib().hoard_moe_ensure(self._h, layer, sel_h.ctypes.data, sel_h.size, out.ctypes.data,
                                           _stream(stream)), "ensure")
        return out

    def residency_stats(self):
        h, m, b = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        self._check(lib().hoard_moe_residency_stats(self._h, ctypes.byref(h), ctypes.byref(m), ctypes.byref(b)),
                    "residency_stats")
        return {"hits": h.value, "misses": m.value, "bytes_uploaded": b.value}

    # ---- expert parallelism (the exchange between these calls is the caller's; see hoard_b200.ep) ----
    def ep_reserve(self, max_rows: int):
        """Receive-side scratch for up to max_rows rows per ep_experts call."""
        self._check(lib().hoard_moe_ep_reserve(self._h, max_rows), "ep_reserve")

    def ep_pack(self, layer: int, sel: torch.Tensor, n_ranks: int, experts_per_rank: int, stream=None):
        """After route(layer, x): entries sorted by destination rank. Returns (send_counts [n_ranks],
        pos_of_entry [T*k], send_expert [T*k], send_rows [T*k][H] f16) on the device."""
        T = sel.shape[0]
        dev = sel.device
        n = T * self.k
        counts = torch.empty(n_ranks, dtype=torch.int32, device=dev)
        pos = torch.empty(n, dtype=torch.int32, device=dev)
        expert = torch.empty(n, dtype=torch.int32, device=dev)
        rows = torch.empty(n, self.H, dtype=torch.float16, device=dev)
        self._check(lib().hoard_moe_ep_pack(self._h, layer, _ptr(sel), T, n_ranks, experts_per_rank, _ptr(counts),
                                            _ptr(pos), _ptr(expert), _ptr(rows), _stream(stream)), "ep_pack")
        return counts, pos, expert, rows

    def ep_experts(self, layer: int, rows: torch.Tensor, slot_of_row: torch.Tensor, y_out: torch.Tensor | None = None,
                   stream=None):
        """Expert FFN of received f16 rows [R][H] bound to slots [R] -> y [R][H] f16."""
        R = rows.shape[0]
        if y_out is None:
            y_out = torch.empty(R, self.H, dtype=torch.float16, device=rows.device)
        self._check(lib().hoard_moe_ep_experts(self._h, layer, _ptr(rows), _ptr(slot_of_row), R, _ptr(y_out),
                                               _stream(stream)), "ep_experts")
        return y_out

    def ep_combine(self, w: torch.Tensor, pos_of_entry: torch.Tensor, y_back: torch.Tensor, x_inout: torch.Tensor,
                   stream=None):
        T = x_inout.shape[0]
        self._check(lib().hoard_moe_ep_combine(self._h, _ptr(w), _ptr(pos_of_entry), _ptr(y_back), _ptr(x_inout), T,
                                               _stream(stream)), "ep_combine")
        return x_inout

    # ---- expert parallelism over NVLink peer memory ----
    def p2p_init(self, n_ranks: int, rank: int, experts_per_rank: int, slot_base: int):
        self._check(lib().hoard_moe_p2p_init(self._h, n_ranks, rank, experts_per_rank, slot_base), "p2p_init")

    def p2p_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(P2P_HANDLE_BYTES)
        self._check(lib().hoard_moe_p2p_handle(self._h, buf), "p2p_handle")
        return buf.raw

    def p2p_open(self, handles):
        """handles: every rank's p2p_handle() bytes in rank order."""
        blob = b"".join(handles)
        if len(blob) != P2P_HANDLE_BYTES * len(handles):
            raise ValueError("each handle must be P2P_HANDLE_BYTES long")
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._check(lib().hoard_moe_p2p_open(self._h, buf), "p2p_open")

    def p2p_attach(self, peers):
        """peers: the group's contexts of this process in rank order (this one included)."""
        arr = (ctypes.c_void_p * len(peers))(*[p._h for p in peers])
        self._check(lib().hoard_moe_p2p_attach(self._h, arr), "p2p_attach")

    def p2p_close(self):
        self._check(lib().hoard_moe_p2p_close(self._h), "p2p_close")

    def p2p_set_timeout(self, seconds: float):
        self._check(lib().hoard_moe_p2p_set_timeout(self._h, float(seconds)), "p2p_set_timeout")

    def p2p_send(self, layer: int, x: torch.Tensor, sel_out=None, w_out=None, stream=None):
        self._check(lib().hoard_moe_p2p_send(self._h, layer, _ptr(x), x.shape[0], _ptr(sel_out), _ptr(w_out),
                                             _stream(stream)), "p2p_send")

    def p2p_compute(self, stream=None):
        self._check(lib().hoard_moe_p2p_compute(self._h, _stream(stream)), "p2p_compute")

    def p2p_finish(self, x_inout: torch.Tensor, stream=None):
        self._check(lib().hoard_moe_p2p_finish(self._h, _ptr(x_inout), _stream(stream)), "p2p_finish")
        return x_inout

    def p2p_layers(self, layer0: int, n_layers: int, x_inout: torch.Tensor, sel_out=None, w_out=None, stream=None):
        self._check(lib().hoard_moe_p2p_layers(self._h, layer0, n_layers, _ptr(x_inout), x_inout.shape[0],
                                               _ptr(sel_out), _ptr(w_out), _stream(stream)), "p2p_layers")
        return x_inout

    def set_gemm_min_tokens(self, min_tokens: int):
        """T at or above which the expert FFN runs as the tensor-core grouped GEMM (0 = never)."""
        self._check(lib().hoard_moe_set_gemm_min_tokens(self._h, min_tokens), "set_gemm_min_tokens")

    def set_top_k(self, k: int):
        """Top-k override: 1 <= k <= n_expert_used (the value the context was created with)."""
        self._check(lib().hoard_moe_set_top_k(self._h, k), "set_top_k")
        self.k = k

    def set_gemm_ctas(self, ctas: int):
        """CTAs of the tensor-core GEMMs (0 = one per SM)."""
        self._check(lib().hoard_moe_set_gemm_ctas(self._h, ctas), "set_gemm_ctas")

    def set_trace(self, buf: torch.Tensor | None):
        """Enables %globaltimer stamps into an int64 CUDA tensor (None turns them off): the persistent
        decode kernel's phases ([cta][layer][phase], see trace_layout), the tensor-core GEMMs' stages
        (capacity >= 4096), and for the small-batch layer path words 0-5 = {first start, last end} of
        the fused route, gate/up and down kernels (set the starts to -1 and the ends to 0 first)."""
        if buf is None:
            self._check(lib().hoard_moe_set_trace(self._h, None, 0), "set_trace")
        else:
            self._check(lib().hoard_moe_set_trace(self._h, _ptr(buf), buf.numel()), "set_trace")

    def trace_layout(self):
        ctas, phases = ctypes.c_int(), ctypes.c_int()
        self._check(lib().hoard_moe_trace_layout(self._h, ctypes.byref(ctas), ctypes.byref(phases)), "trace_layout")
        return ctas.value, phases.value

    def sync_status(self, stream=None):
        self._check(lib().hoard_moe_sync_status(self._h, _stream(stream)), "sync_status")

    # -- weights -------------------------------------------------------------------------------
    def set_router(self, layer: int, w_router: torch.Tensor, w_norm: torch.Tensor):
        w_router = w_router.contiguous().float()
        w_norm = w_norm.contiguous().float()
        assert w_router.shape == (self.E, self.H) and w_norm.shape == (self.H,)
        self._check(lib().hoard_moe_set_router(self._h, layer, _ptr(w_router), _ptr(w_norm)), "set_router")

    def upload_expert(self, layer: int, slot: int, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                      stream=None):
        """Raw GGUF bytes of one expert (uint8 tensors, host or device)."""
        for t, (typ, n, kk) in zip((gate, up, down), ((self.gate_types[layer], self.I, self.H),
                                                      (self.up_types[layer], self.I, self.H),
                                                      (self.down_types[layer], self.H, self.I))):
            assert t.dtype == torch.uint8 and t.is_contiguous() and t.numel() == n * row_bytes(typ, kk)
        self._check(lib().hoard_moe_upload_expert(self._h, layer, slot, _ptr(gate), _ptr(up), _ptr(down),
                                                  _stream(stream)), "upload_expert")

    def set_shared(self, layer: int, gate, up, down, gate_inp: torch.Tensor):
        gate_inp = gate_inp.contiguous().float()
        self._check(lib().hoard_moe_set_shared(self._h, layer, _ptr(gate), _ptr(up), _ptr(down), _ptr(gate_inp)),
                    "set_shared")

    # -- the hot path ------------------------------------------------------------------------
    def route(self, layer: int, x: torch.Tensor, sel: torch.Tensor | None = None, w: torch.Tensor | None = None,
              stream=None):
        T = x.shape[0]
        dev = x.device
        if sel is None:
            sel = torch.empty(T, self.k, dtype=torch.int32, device=dev)
        if w is None:
            w = torch.empty(T, self.k, dtype=torch.float32, device=dev)
        self._check(lib().hoard_moe_route(self._h, layer, _ptr(x), T, _ptr(sel), _ptr(w), _stream(stream)), "route")
        return sel, w

    def experts(self, layer: int, sel: torch.Tensor, w: torch.Tensor, x_inout: torch.Tensor, fx=None,
                slot_of_sel=None, stream=None):
        T = x_inout.shape[0]
        self._check(lib().hoard_moe_experts(self._h, layer, _ptr(fx), _ptr(sel), _ptr(slot_of_sel), _ptr(w),
                                            _ptr(x_inout), T, _stream(stream)), "experts")
        return x_inout

    def layer(self, layer: int, x_inout: torch.Tensor, sel_out=None, w_out=None, stream=None):
        T = x_inout.shape[0]
        self._check(lib().hoard_moe_layer(self._h, layer, _ptr(x_inout), T, _ptr(sel_out), _ptr(w_out),
                                          _stream(stream)), "layer")
        return x_inout

    def decode_noalloc(self, layer0: int, n_layers: int, x_inout: torch.Tensor, sel_out=None, w_out=None,
                       stream=None):
        """T = 1 decode over n_layers layers with the library's static scratch (no device allocation)."""
        self._check(lib().hoard_moe_decode_noalloc(self._h, layer0, n_layers, _ptr(x_inout), _ptr(sel_out),
                                                   _ptr(w_out), _stream(stream)), "decode_noalloc")
        return x_inout

    def decode_noalloc_status(self, stream=None):
        """Waits for the stream; raises HoardError for errors recorded in the static scratch's error word."""
        self._check(lib().hoard_moe_decode_noalloc_status(self._h, _stream(stream)), "decode_noalloc_status")

    def layers(self, layer0: int, n_layers: int, x_inout: torch.Tensor, sel_out=None, w_out=None, stream=None):
        T = x_inout.shape[0]
        self._check(lib().hoard_moe_layers(self._h, layer0, n_layers, _ptr(x_inout), T, _ptr(sel_out), _ptr(w_out),
                                           _stream(stream)), "layers")
        return x_inout
