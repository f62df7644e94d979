"""hoard_b200: a B200-native (sm_100a) implementation of hoard's per-layer MoE hot path.

router (RMSNorm -> f32 router GEMV -> softmax -> top-k, optional renorm) -> expert dispatch ->
SwiGLU expert FFN on GGUF Q4_K/Q6_K weights -> weighted combine into the residual, behind the C
ABI of include/hoard_moe.h (built as hoard_b200/libhoard_moe.so).
"""
from .quant import Q4_K, Q6_K, quantize, quantize_q4k, quantize_q6k, row_bytes, synth_experts  # noqa: F401

__all__ = ["Q4_K", "Q6_K", "quantize", "quantize_q4k", "quantize_q6k", "row_bytes", "synth_experts"]
