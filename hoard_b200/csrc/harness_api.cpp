// harness_api.cpp -- the C ABI of include/hoard_harness.h: argument checks and launches of the
// per-token decode-step operations (kernels_harness.cu). Stateless; status codes as hoard_moe.h.
#include "../../include/hoard_harness.h"
#include "kernels.h"

#include <cuda_runtime.h>

using namespace hoard;

namespace {

inline int64_t al256(int64_t v) { return (v + 255) / 256 * 256; }
inline bool quant_type(int t) { return t == HOARD_TYPE_Q4_K || t == HOARD_TYPE_Q6_K; }
inline int st(cudaError_t e) {
    if (e == cudaSuccess) return HOARD_OK;
    cudaGetLastError();
    return e == cudaErrorInvalidValue ? HOARD_EINVAL : HOARD_ECUDA;
}

}  // namespace

// KV cache element types: f16 (HOARD_TYPE_F16) or bf16 (HOARD_TYPE_BF16)
static bool kv_ok(int t) { return t == HOARD_TYPE_F16 || t == HOARD_TYPE_BF16; }

extern "C" {

int hoard_hx_repack(int type, const void* src, void* dst, int64_t n_blocks, hoard_stream stream) {
    if (!quant_type(type) || !src || !dst || n_blocks <= 0) return HOARD_EINVAL;
    return st(launch_repack(type, static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), n_blocks,
                            (cudaStream_t)stream));
}

int hoard_hx_embed(int type, const void* table, int n_embd, int64_t n_vocab, const int32_t* token, float* x_out,
                   hoard_stream stream) {
    if (!table || !token || !x_out || n_embd <= 0 || n_vocab <= 0) return HOARD_EINVAL;
    if (!(type == HOARD_TYPE_F32 || type == 1 || quant_type(type))) return HOARD_EINVAL;
    if (quant_type(type) && n_embd % 256) return HOARD_EINVAL;
    return st(launch_embed(type, static_cast<const uint8_t*>(table), n_embd, n_vocab, token, nullptr, x_out,
                           (cudaStream_t)stream));
}

int hoard_hx_embed_at(int type, const void* table, int n_embd, int64_t n_vocab, const int32_t* seq,
                      const int32_t* pos, float* x_out, hoard_stream stream) {
    if (!table || !seq || !pos || !x_out || n_embd <= 0 || n_vocab <= 0) return HOARD_EINVAL;
    if (!(type == HOARD_TYPE_F32 || type == 1 || quant_type(type))) return HOARD_EINVAL;
    if (quant_type(type) && n_embd % 256) return HOARD_EINVAL;
    return st(launch_embed(type, static_cast<const uint8_t*>(table), n_embd, n_vocab, seq, pos, x_out,
                           (cudaStream_t)stream));
}

int hoard_hx_rmsnorm(const float* x, int rows, int cols, float eps, const float* w, float* out, hoard_stream stream) {
    if (!x || !w || !out || rows <= 0 || cols <= 0 || cols > 8192) return HOARD_EINVAL;
    return st(launch_rmsnorm_f32(x, rows, cols, eps, w, out, (cudaStream_t)stream));
}

int64_t hoard_hx_q8_bytes(int K) {
    if (K <= 0 || K % 256) return -1;
    return al256(K) + al256((int64_t)K / 256 * 4) + al256((int64_t)K / 16 * 4);
}

int hoard_hx_quant_q8(const float* x, int K, void* q8, hoard_stream stream) {
    if (!x || !q8 || K <= 0 || K % 256) return HOARD_EINVAL;
    uint8_t* b = static_cast<uint8_t*>(q8);
    return st(launch_quant_q8(x, 1, K, reinterpret_cast<int8_t*>(b), reinterpret_cast<float*>(b + al256(K)),
                              reinterpret_cast<int*>(b + al256(K) + al256((int64_t)K / 256 * 4)),
                              (cudaStream_t)stream));
}

int hoard_hx_gemv(int type, const void* w_plane, int N, int K, const void* q8, const float* resid, float* y,
                  hoard_stream stream) {
    if (!quant_type(type) || !w_plane || !q8 || !y || N <= 0 || K <= 0 || K % 256) return HOARD_EINVAL;
    const uint8_t* b = static_cast<const uint8_t*>(q8);
    return st(launch_qgemv(type, static_cast<const uint8_t*>(w_plane), N, K, reinterpret_cast<const int8_t*>(b),
                           reinterpret_cast<const float*>(b + al256(K)),
                           reinterpret_cast<const int*>(b + al256(K) + al256((int64_t)K / 256 * 4)), resid, y,
                           (cudaStream_t)stream));
}

int hoard_hx_rope_store(float* q, float* k, const float* v, int n_head, int n_head_kv, int head_dim, int pos,
                        float freq_base, void* k_cache, void* v_cache, int kv_type, hoard_stream stream) {
    if (!q || !k || !v || !k_cache || !v_cache || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim % 2 || pos < 0 || !(freq_base > 0) || !kv_ok(kv_type))
        return HOARD_EINVAL;
    return st(launch_rope_store(q, k, v, n_head, n_head_kv, head_dim, pos, nullptr, pos + 1, freq_base, k_cache, v_cache,
                                kv_type == HOARD_TYPE_BF16, (cudaStream_t)stream));
}

int hoard_hx_rope_store_at(float* q, float* k, const float* v, int n_head, int n_head_kv, int head_dim,
                           const int32_t* pos, int max_ctx, float freq_base, void* k_cache, void* v_cache,
                           int kv_type, hoard_stream stream) {
    if (!q || !k || !v || !pos || !k_cache || !v_cache || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim % 2 || max_ctx <= 0 || !(freq_base > 0) || !kv_ok(kv_type))
        return HOARD_EINVAL;
    return st(launch_rope_store(q, k, v, n_head, n_head_kv, head_dim, 0, pos, max_ctx, freq_base, k_cache, v_cache,
                                kv_type == HOARD_TYPE_BF16, (cudaStream_t)stream));
}

int hoard_hx_attention(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                       int head_dim, int n_pos, float scale, float* out, int kv_type, hoard_stream stream) {
    if (!q || !k_cache || !v_cache || !out || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim > 256 || 256 % head_dim || n_pos <= 0 || !kv_ok(kv_type))
        return HOARD_EINVAL;
    if (attention_smem(head_dim, n_pos) > 200 * 1024) return HOARD_EINVAL;
    return st(launch_attention(q, k_cache, v_cache, kv_type == HOARD_TYPE_BF16, n_head, n_head_kv, head_dim, n_pos,
                               nullptr, scale, nullptr, 0, out, (cudaStream_t)stream));
}

int hoard_hx_attention_at(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                          int head_dim, const int32_t* pos, int max_ctx, float scale, float* out, int kv_type,
                          hoard_stream stream) {
    if (!q || !k_cache || !v_cache || !pos || !out || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim > 256 || 256 % head_dim || max_ctx <= 0 || !kv_ok(kv_type))
        return HOARD_EINVAL;
    if (attention_smem(head_dim, max_ctx) > 200 * 1024) return HOARD_EINVAL;
    return st(launch_attention(q, k_cache, v_cache, kv_type == HOARD_TYPE_BF16, n_head, n_head_kv, head_dim, max_ctx,
                               pos, scale, nullptr, 0, out, (cudaStream_t)stream));
}

int hoard_hx_argmax(const float* v, int n, int32_t* out, hoard_stream stream) {
    if (!v || !out || n <= 0) return HOARD_EINVAL;
    return st(launch_argmax(v, n, out, nullptr, 0, (cudaStream_t)stream));
}

int hoard_hx_argmax_at(const float* v, int n, int32_t* seq, int32_t* pos, int seq_len, hoard_stream stream) {
    if (!v || !seq || !pos || n <= 0 || seq_len <= 0) return HOARD_EINVAL;
    return st(launch_argmax(v, n, seq, pos, seq_len, (cudaStream_t)stream));
}

int hoard_hx_rmsnorm_q8(const float* x, int H, float eps, const float* w, void* q8, hoard_stream stream) {
    if (!x || !w || !q8 || H <= 0 || H % 256 || H > 8192 || ((H / 256) & (H / 256 - 1))) return HOARD_EINVAL;
    uint8_t* b = static_cast<uint8_t*>(q8);
    return st(launch_rmsnorm_q8(x, H, eps, w, reinterpret_cast<int8_t*>(b), reinterpret_cast<float*>(b + al256(H)),
                                reinterpret_cast<int*>(b + al256(H) + al256((int64_t)H / 256 * 4)), (cudaStream_t)stream));
}

int hoard_hx_gemv_multi(int n, const int* types, const void* const* w_planes, const int* N, int K, const void* q8,
                        const float* const* resid, float* const* y, hoard_stream stream) {
    if (n < 1 || n > 3 || !types || !w_planes || !N || !q8 || !y || K <= 0 || K % 256) return HOARD_EINVAL;
    for (int m = 0; m < n; ++m)
        if (!quant_type(types[m]) || !w_planes[m] || !y[m] || N[m] <= 0) return HOARD_EINVAL;
    const uint8_t* b = static_cast<const uint8_t*>(q8);
    return st(launch_qgemv_set(n, types, reinterpret_cast<const uint8_t* const*>(w_planes), N, K, resid, y,
                               reinterpret_cast<const int8_t*>(b), reinterpret_cast<const float*>(b + al256(K)),
                               reinterpret_cast<const int*>(b + al256(K) + al256((int64_t)K / 256 * 4)),
                               (cudaStream_t)stream));
}

static int qknorm_check(const float* q, const float* k, const float* v, const float* qn, const float* kn, int mode,
                        int n_head, int n_head_kv, int head_dim, const float* q_out, const void* kc, const void* vc) {
    if (!q || !k || !v || !q_out || !kc || !vc || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim % 2 || head_dim > 256 || mode < 0 || mode > 2 || q_out == q)
        return HOARD_EINVAL;
    if (mode != 0 && (!qn || !kn)) return HOARD_EINVAL;
    return HOARD_OK;
}

int hoard_hx_qknorm_rope_store(const float* q, const float* k, const float* v, const float* q_norm,
                               const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                               int pos, float freq_base, float* q_out, void* k_cache, void* v_cache, int kv_type,
                               hoard_stream stream) {
    int rc = qknorm_check(q, k, v, q_norm, k_norm, mode, n_head, n_head_kv, head_dim, q_out, k_cache, v_cache);
    if (rc || pos < 0 || !(freq_base > 0) || !kv_ok(kv_type)) return rc ? rc : HOARD_EINVAL;
    return st(launch_qknorm_rope_store(q, k, v, q_norm, k_norm, mode, eps, n_head, n_head_kv, head_dim, head_dim,
                                       head_dim, pos, nullptr, pos + 1, freq_base, q_out, k_cache, v_cache, kv_type == HOARD_TYPE_BF16,
                                       (cudaStream_t)stream));
}

int hoard_hx_qknorm_rope_store_at(const float* q, const float* k, const float* v, const float* q_norm,
                                  const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                                  const int32_t* pos, int max_ctx, float freq_base, float* q_out, void* k_cache,
                                  void* v_cache, int kv_type, hoard_stream stream) {
    int rc = qknorm_check(q, k, v, q_norm, k_norm, mode, n_head, n_head_kv, head_dim, q_out, k_cache, v_cache);
    if (rc || !pos || max_ctx <= 0 || !(freq_base > 0) || !kv_ok(kv_type)) return rc ? rc : HOARD_EINVAL;
    return st(launch_qknorm_rope_store(q, k, v, q_norm, k_norm, mode, eps, n_head, n_head_kv, head_dim, head_dim,
                                       head_dim, 0, pos, max_ctx, freq_base, q_out, k_cache, v_cache, kv_type == HOARD_TYPE_BF16,
                                       (cudaStream_t)stream));
}

int hoard_hx_qknorm_rope_store_ex(const float* q, const float* k, const float* v, const float* q_norm,
                                  const float* k_norm, int mode, float eps, int n_head, int n_head_kv, int head_dim,
                                  int q_stride, int rope_dim, int pos, const int32_t* pos_dev, int max_ctx,
                                  float freq_base, float* q_out, void* k_cache, void* v_cache, int kv_type,
                                  hoard_stream stream) {
    int rc = qknorm_check(q, k, v, q_norm, k_norm, mode, n_head, n_head_kv, head_dim, q_out, k_cache, v_cache);
    if (rc) return rc;
    if (q_stride < head_dim || (mode == 1 && q_stride != head_dim) || rope_dim < 2 || rope_dim > head_dim ||
        rope_dim % 2 || max_ctx <= 0 || (!pos_dev && (pos < 0 || pos >= max_ctx)) || !(freq_base > 0) ||
        !kv_ok(kv_type))
        return HOARD_EINVAL;
    return st(launch_qknorm_rope_store(q, k, v, q_norm, k_norm, mode, eps, n_head, n_head_kv, head_dim, q_stride,
                                       rope_dim, pos, pos_dev, max_ctx, freq_base, q_out, k_cache, v_cache,
                                       kv_type == HOARD_TYPE_BF16, (cudaStream_t)stream));
}

int hoard_hx_attention_ex(const float* q, const void* k_cache, const void* v_cache, int n_head, int n_head_kv,
                          int head_dim, int n_pos, const int32_t* pos_dev, float scale, const float* gate,
                          int gate_stride, float* out, int kv_type, hoard_stream stream) {
    if (!q || !k_cache || !v_cache || !out || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv ||
        head_dim <= 0 || head_dim > 256 || 256 % head_dim || n_pos <= 0 || !kv_ok(kv_type) ||
        (gate && gate_stride < head_dim))
        return HOARD_EINVAL;
    if (attention_smem(head_dim, n_pos) > 200 * 1024) return HOARD_EINVAL;
    return st(launch_attention(q, k_cache, v_cache, kv_type == HOARD_TYPE_BF16, n_head, n_head_kv, head_dim, n_pos,
                               pos_dev, scale, gate, gate_stride, out, (cudaStream_t)stream));
}

int hoard_hx_gdn_step(const float* qkv, const float* z, const float* ba, const float* conv_w, float* conv_ring,
                      const float* dt_bias, const float* ssm_a, const float* norm_w, float* state, int n_v_heads,
                      int n_k_heads, int d_state, int d_conv, float eps, int pos, const int32_t* pos_dev, float* out,
                      hoard_stream stream) {
    if (!qkv || !z || !ba || !conv_w || !conv_ring || !dt_bias || !ssm_a || !norm_w || !state || !out ||
        d_state != 128 || n_k_heads <= 0 || n_v_heads <= 0 || n_v_heads % n_k_heads || d_conv < 1 || d_conv > 8 ||
        (!pos_dev && pos < 0))
        return HOARD_EINVAL;
    return st(launch_gdn_step(qkv, z, ba, conv_w, conv_ring, dt_bias, ssm_a, norm_w, state, n_v_heads, n_k_heads,
                              d_state, d_conv, eps, pos, pos_dev, out, (cudaStream_t)stream));
}

}  // extern "C"
