/* hoard_harness.h -- the per-token operations of a decode step around the MoE layers.
 *
 * hoard runs these as ggml graphs on its single backend thread: graph E (embedding row,
 * src/run_moe_stream.cpp:302-312), graph A's attention part (:320-351: attn RMSNorm, q/k/v
 * projections, QK RMSNorm over the full projection (OLMoE) or per head (Qwen3), NEOX RoPE, KV-cache
 * store, single-query attention with softmax scale 1/sqrt(head_dim), output projection plus the
 * residual) and the head (:452-472: output RMSNorm, lm-head, argmax). These entry points are the
 * same steps as stateless device operations, so a decode driver keeps hoard's schedule
 * (graph E -> per layer: attention, then hoard_moe_layer -> head) with every buffer on the device.
 *
 * Quantised weights (Q4_K = 12, Q6_K = 14) are used in the plane layout that hoard_hx_repack
 * produces from raw GGUF blocks; projections quantise the activation to Q8_K first
 * (hoard_hx_quant_q8) and form exact integer block dots, the semantics of ggml's CPU mul_mat. The KV
 * cache is [max_ctx][n_head_kv][head_dim] per layer of f16 or bf16 (kv_type HOARD_TYPE_F16 /
 * HOARD_TYPE_BF16; hoard keeps an f32 cache, src/run_moe_stream.cpp:239). All pointers are device pointers; every
 * call is asynchronous on `stream`. Status codes are those of hoard_moe.h. */
#ifndef HOARD_HARNESS_H
#define HOARD_HARNESS_H

#include <stdint.h>
#include "hoard_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Raw GGUF Q4_K / Q6_K blocks (n_blocks of them, rows back to back) -> plane layout (same size). */
int hoard_hx_repack(int type, const void* src, void* dst, int64_t n_blocks, hoard_stream stream);

/* x_out[n_embd] = row *token of an embedding table (raw GGUF Q4_K / Q6_K blocks, or f32 = 0 / f16 = 1);
 * token is a device int32 (ggml_get_rows). */
int hoard_hx_embed(int type, const void* table, int n_embd, int64_t n_vocab, const int32_t* token, float* x_out,
                   hoard_stream stream);

/* out[r] = x[r] / sqrt(mean(x[r]^2) + eps) * w, rows of `cols` values (cols <= 8192). */
int hoard_hx_rmsnorm(const float* x, int rows, int cols, float eps, const float* w, float* out, hoard_stream stream);

/* Bytes of the Q8_K workspace of a K-vector: int8 [K] | f32 scales [K/256] | int32 16-sums [K/16]. */
int64_t hoard_hx_q8_bytes(int K);
int hoard_hx_quant_q8(const float* x, int K, void* q8, hoard_stream stream);

/* y[N] = W . x (+ resid, elementwise, when non-null): W plane layout, N rows of K, x as Q8_K. */
int hoard_hx_gemv(int type, const void* w_plane, int N, int K, const void* q8, const float* resid, float* y,
                  hoard_stream stream);

/* NEOX RoPE of q [n_head][head_dim] and k [n_head_kv][head_dim] (in place) at position pos with
 * theta_i = pos * freq_base^(-2i/head_dim); then k and v stored (f16 or bf16, rounded to nearest) at
 * cache row pos. */
int hoard_hx_rope_store(float* q, float* k, const float* v, int n_head, int n_head_kv, int head_dim, int pos,
                        float freq_base, void* k_cache, void* v_cache, int kv_type, hoard_stream stream);

/* out[h] = softmax(scale * q[h] . K[0..n_pos)) . V[0..n_pos) of KV head h / (n_head / n_head_kv). */
int hoard_hx_attention(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                       int head_dim, int n_pos, float scale, float* out, int kv_type, hoard_stream stream);

/* *out = the first index of the maximum of v[0..n). */
int hoard_hx_argmax(const float* v, int n, int32_t* out, hoard_stream stream);

/* ---- the same steps with the position in device memory, so that one captured CUDA graph of a
 * whole decode step can be replayed for every token ----
 * embed_at: token = seq[*pos]. rope_store_at: position *pos (nothing is written when
 * *pos >= max_ctx). attention_at: n_pos = min(*pos + 1, max_ctx). argmax_at: seq[*pos + 1] = the
 * argmax (when *pos + 1 < seq_len), then *pos += 1. */
int hoard_hx_embed_at(int type, const void* table, int n_embd, int64_t n_vocab, const int32_t* seq,
                      const int32_t* pos, float* x_out, hoard_stream stream);
int hoard_hx_rope_store_at(float* q, float* k, const float* v, int n_head, int n_head_kv, int head_dim,
                           const int32_t* pos, int max_ctx, float freq_base, void* k_cache, void* v_cache,
                           int kv_type, hoard_stream stream);
int hoard_hx_attention_at(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                          int head_dim, const int32_t* pos, int max_ctx, float scale, float* out, int kv_type,
                          hoard_stream stream);
int hoard_hx_argmax_at(const float* v, int n, int32_t* seq, int32_t* pos, int seq_len, hoard_stream stream);

/* ---- fused forms of the steps above (fewer launches per layer) ----
 * rmsnorm_q8: RMSNorm(x) * w of one vector (H a power-of-two multiple of 256, <= 8192) straight into
 * a Q8_K workspace. gemv_multi: 1..3 projections of the same Q8_K activation (types, plane-layout
 * weights, row counts, optional residuals and outputs are host arrays of n device pointers/values).
 * qknorm_rope_store: QK RMSNorm (mode 0 none, 1 over the whole projection with weights
 * [n_head*head_dim] / [n_head_kv*head_dim], 2 per head with weights [head_dim]) + NEOX RoPE + KV
 * store; the rotated q is written to q_out (!= q). */
int hoard_hx_rmsnorm_q8(const float* x, int H, float eps, const float* w, void* q8, hoard_stream stream);
int hoard_hx_gemv_multi(int n, const int* types, const void* const* w_planes, const int* N, int K, const void* q8,
                        const float* const* resid, float* const* y, hoard_stream stream);
int hoard_hx_qknorm_rope_store(const float* q, const float* k, const float* v, const float* q_norm,
                               const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                               int pos, float freq_base, float* q_out, void* k_cache, void* v_cache, int kv_type,
                               hoard_stream stream);
int hoard_hx_qknorm_rope_store_at(const float* q, const float* k, const float* v, const float* q_norm,
                                  const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                                  const int32_t* pos, int max_ctx, float freq_base, float* q_out, void* k_cache,
                                  void* v_cache, int kv_type, hoard_stream stream);

/* ---- the hybrid (Qwen3-Next) layer kinds, graph A of src/run_qwen35.cpp:472-553 ----
 * qknorm_rope_store_ex: qknorm_rope_store with q heads q_stride floats apart (2 * head_dim for the
 * fused q + gate projection, whose head h is [q (head_dim) | gate (head_dim)]) and NEOX RoPE on the
 * first rope_dim values of each head only (the rest pass through); pos_dev != NULL reads the
 * position from device memory (bounded by max_ctx), else pos is used.
 * attention_ex: attention with n_pos positions, or min(*pos_dev + 1, n_pos) when pos_dev != NULL,
 * and with gate != NULL the output of head h multiplied by sigmoid(gate[h * gate_stride + i]).
 * gdn_step: one token through a gated delta-net layer (d_state 128): qkv [conv_dim] = [q: Hk*128 |
 * k: Hk*128 | v: Hv*128] projection outputs, z [Hv*128] the output-gate projection, ba [2*Hv] the
 * beta/alpha projection in per-key-head groups [Hv/Hk betas | Hv/Hk alphas], conv_w ne = [d_conv,
 * conv_dim] (f32), conv_ring [d_conv][conv_dim] the last inputs (slot = position % d_conv; any
 * contents at position 0), dt_bias / ssm_a [Hv], norm_w [128], state [Hv][128 key][128 value] f32
 * (zero at the start of a sequence). Writes out [Hv*128] = RMSNorm(S^T q) * norm_w * silu(z) per value
 * head and updates state and the ring. */
int hoard_hx_qknorm_rope_store_ex(const float* q, const float* k, const float* v, const float* q_norm,
                                  const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                                  int q_stride, int rope_dim, int pos, const int32_t* pos_dev, int max_ctx,
                                  float freq_base, float* q_out, void* k_cache, void* v_cache, int kv_type,
                                  hoard_stream stream);
int hoard_hx_attention_ex(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                          int head_dim, int n_pos, const int32_t* pos_dev, float scale, const float* gate,
                          int gate_stride, float* out, int kv_type, hoard_stream stream);
int hoard_hx_gdn_step(const float* qkv, const float* z, const float* ba, const float* conv_w, float* conv_ring,
                      const float* dt_bias, const float* ssm_a, const float* norm_w, float* state, int n_v_heads,
                      int n_k_heads, int d_state, int d_conv, float eps, int pos, const int32_t* pos_dev, float* out,
                      hoard_stream stream);

#ifdef __cplusplus
}
#endif

#endif
