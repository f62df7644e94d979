// kernels_harness.cu -- the per-token operations around the MoE layers of a decode step, i.e. hoard's
// graph E / graph A attention / head (src/run_moe_stream.cpp:302-351, :452-472): embedding row,
// RMSNorm over rows, Q8_K of an activation vector, quantised projection GEMV (the same exact
// Q4_K / Q6_K . Q8_K integer dots as the expert path, on plane-layout weights), NEOX RoPE with the
// KV-cache store, single-query attention over an f16 KV cache, argmax.
#include "common.cuh"
#include "kernels.h"
#include "block_ops.cuh"

#include <cuda_fp16.h>

namespace hoard {

namespace {

// ---- embedding: one row of a raw GGUF table (Q4_K / Q6_K blocks, f32 or f16) to f32 ----
__global__ void __launch_bounds__(256) k_embed(int type, const uint8_t* __restrict__ table, int H, int64_t n_vocab,
                                               const int32_t* __restrict__ tok, const int32_t* __restrict__ pos,
                                               float* __restrict__ out) {
    pdl_enter();
    const int nb = H / QK;
    const int64_t token = tok[pos ? *pos : 0];
    const bool ok = token >= 0 && token < n_vocab;     // an id out of range gives a zero row
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
        float v;
        if (!ok) {
            v = 0.f;
        } else if (type == T_F32) {
            v = reinterpret_cast<const float*>(table)[token * H + i];
        } else if (type == T_F16) {
            v = __half2float(reinterpret_cast<const __half*>(table)[token * H + i]);
        } else if (type == T_Q4K) {
            // block: fp16 d | fp16 dmin | 12 bytes of 6-bit scales/mins | 128 bytes of 4-bit values;
            // value j of a block: 64-value group j/64, low nibble for j%64 < 32, sub-block j/32
            const uint8_t* b = table + (token * nb + i / QK) * 144;
            const int j = i % QK, g = j / 64, l = j % 32, is = j / 32;
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(b)));
            const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(b + 2)));
            const uint8_t* s = b + 4;
            int sc, m;
            if (is < 4) {
                sc = s[is] & 63;
                m = s[is + 4] & 63;
            } else {
                sc = (s[is + 4] & 0xF) | ((s[is - 4] >> 6) << 4);
                m = (s[is + 4] >> 4) | ((s[is] >> 6) << 4);
            }
            const uint8_t qb = b[16 + 32 * g + l];
            const int q = (j % 64) < 32 ? (qb & 0xF) : (qb >> 4);
            v = (d * (float)sc) * (float)q - dmin * (float)m;
        } else {
            // block: 128 bytes low 4 bits | 64 bytes high 2 bits | 16 int8 scales | fp16 d; value j:
            // half n = j/128, within it l = j%32 and quarter a = (j%128)/32
            const uint8_t* b = table + (token * nb + i / QK) * 210;
            const int j = i % QK, n = j / 128, a = (j % 128) / 32, l = j % 32;
            const uint8_t* ql = b + 64 * n;
            const uint8_t* qh = b + 128 + 32 * n;
            const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 8 * n;
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(b + 208)));
            const int lo = (a & 1) ? ql[l + 32] : ql[l];
            const int low4 = (a < 2) ? (lo & 0xF) : (lo >> 4);
            const int hi2 = (qh[l] >> (2 * a)) & 3;
            const int q = (low4 | (hi2 << 4)) - 32;
            v = (d * (float)sc[l / 16 + 2 * a]) * (float)q;
        }
        out[i] = v;
    }
}

// ---- y[n] = W[n] . Q8_K(x) (+ resid[n]): one warp per output row ----
template <int TYPE>
__global__ void __launch_bounds__(256) k_qgemv(const uint8_t* __restrict__ w, int N, int K,
                                               const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                               const int* __restrict__ xbs, const float* __restrict__ resid,
                                               float* __restrict__ y) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (n >= N) return;
    const int nb = K / QK;
    const ActRow a{xq, xd, xbs};
    float v = warp_sum(row_dot_lane<TYPE>(w, (int64_t)N * nb, n, nb, a, lane));
    if (lane == 0) y[n] = resid ? v + resid[n] : v;
}

// KV cache elements: f16 or bf16 (round to nearest even either way)
__device__ __forceinline__ void kv_put(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void kv_put(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ float kv_get(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float kv_get(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// ---- NEOX RoPE of q [n_head][hd] and k [n_kv][hd] in place at position pos, then k and v stored
//      as f16 or bf16 into the caches at [pos][kv head][hd]. theta_i = pos * base^(-2i/hd) formed by
//      repeated multiplication, as ggml's rope cache does ----
template <typename KT>
__global__ void __launch_bounds__(256) k_rope_store(float* __restrict__ q, float* __restrict__ k,
                                                    const float* __restrict__ v, int n_head, int n_kv, int hd,
                                                    int pos, const int32_t* __restrict__ pos_dev, int max_ctx,
                                                    float theta_scale, KT* __restrict__ kc, KT* __restrict__ vc) {
    pdl_enter();
    if (pos_dev) pos = *pos_dev;
    if (pos < 0 || pos >= max_ctx) return;              // outside the cache: nothing is written
    const int half = hd / 2;
    const int n_pairs = (n_head + n_kv) * half;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n_pairs; t += gridDim.x * blockDim.x) {
        const int head = t / half, i = t - head * half;
        float theta = (float)pos;
        for (int s = 0; s < i; ++s) theta *= theta_scale;
        const float c = cosf(theta), sn = sinf(theta);
        float* x = head < n_head ? q + (int64_t)head * hd : k + (int64_t)(head - n_head) * hd;
        const float x0 = x[i], x1 = x[i + half];
        const float r0 = x0 * c - x1 * sn, r1 = x0 * sn + x1 * c;
        x[i] = r0;
        x[i + half] = r1;
        if (head >= n_head) {
            const int64_t o = ((int64_t)pos * n_kv + (head - n_head)) * hd;
            kv_put(kc + o + i, r0);
            kv_put(kc + o + i + half, r1);
        }
    }
    const int nv = n_kv * hd;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < nv; t += gridDim.x * blockDim.x)
        kv_put(vc + (int64_t)pos * nv + t, v[t]);
}

// sum over u = t, t + 128, ... < n of (double)(v[u]^2), in that order, with eight loads issued
// before their squares are added (a plain strided loop waits for each load in turn)
__device__ __forceinline__ double sumsq_stride128(const float* __restrict__ v, int n, int t) {
    double ss = 0.0;
    for (int u0 = t; u0 < n; u0 += 8 * 128) {
        float x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = u0 + k * 128 < n ? v[u0 + k * 128] : 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (u0 + k * 128 < n) ss += (double)(x[k] * x[k]);
    }
    return ss;
}

// ---- single-query attention: one CTA per head; scores over the n_pos cached keys of its KV head
//      (f16 or bf16, products and sums in f32), softmax with the max subtracted and a double sum, then
//      the probability-weighted sum of the cached values ----
constexpr int ATT_THREADS = 256;
template <typename KT>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const float* __restrict__ q, const KT* __restrict__ kc,
                                                          const KT* __restrict__ vc, int n_head, int n_kv, int hd,
                                                          int n_pos, const int32_t* __restrict__ pos_dev,
                                                          float scale, const float* __restrict__ gate, int gstride,
                                                          float* __restrict__ out) {
    pdl_enter();
    extern __shared__ float sm[];
    const int cap = n_pos;                           // positions the shared memory was sized for
    if (pos_dev) n_pos = min(*pos_dev + 1, cap);
    float* sq = sm;                  // [hd]
    float* sp = sm + hd;             // [n_pos] scores, then probabilities
    float* part = sp + cap;          // [ATT_THREADS / hd][hd] partial output sums
    __shared__ float redf[32];
    __shared__ double redd[32];
    const int h = blockIdx.x, kvh = h / (n_head / n_kv);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sq[i] = q[(int64_t)h * hd + i];
    __syncthreads();
    for (int j = warp; j < n_pos; j += nw) {
        const KT* kr = kc + ((int64_t)j * n_kv + kvh) * hd;
        float s = 0.f;
        for (int i = lane; i < hd; i += 32) s += sq[i] * kv_get(kr + i);
        s = warp_sum(s);
        if (lane == 0) sp[j] = s * scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n_pos; j += blockDim.x) mx = fmaxf(mx, sp[j]);
    mx = block_max_f(mx, redf);
    double sum = 0.0;
    for (int j = threadIdx.x; j < n_pos; j += blockDim.x) {
        const float e = expf(sp[j] - mx);
        sp[j] = e;
        sum += (double)e;
    }
    sum = block_sum_d(sum, redd);
    const float inv = (float)(1.0 / sum);
    __syncthreads();
    // thread = (position group g, dimension i); groups take positions j = g, g + G, ...
    const int G = blockDim.x / hd;
    if (threadIdx.x < G * hd) {
        const int g = threadIdx.x / hd, i = threadIdx.x - g * hd;
        float acc = 0.f;
        for (int j = g; j < n_pos; j += G) acc += (sp[j] * inv) * kv_get(vc + ((int64_t)j * n_kv + kvh) * hd + i);
        part[g * hd + i] = acc;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.f;
        for (int g = 0; g < G; ++g) acc += part[g * hd + i];
        if (gate) acc *= sigmoid_f(gate[(int64_t)h * gstride + i]);
        out[(int64_t)h * hd + i] = acc;
    }
}

// ---- the same attention for head dims that are a multiple of 8 (16-byte rows of 8 cache values):
//      one CTA of AV_THREADS per head; a thread takes whole positions for the scores (its key row read
//      with 16-byte loads, q from shared memory), and (position group, 8 dimensions) for the
//      probability-weighted value sum; the groups' partial sums are added in group order ----
constexpr int AV_THREADS = 512;
__device__ __forceinline__ void kv_get8(const __half* p, float* f) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
__device__ __forceinline__ void kv_get8(const __nv_bfloat16* p, float* f) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

template <typename KT>
__global__ void __launch_bounds__(AV_THREADS) k_attention_v8(const float* __restrict__ q, const KT* __restrict__ kc,
                                                             const KT* __restrict__ vc, int n_head, int n_kv, int hd,
                                                             int n_pos, const int32_t* __restrict__ pos_dev,
                                                             float scale, const float* __restrict__ gate, int gstride,
                                                             float* __restrict__ out) {
    pdl_enter();
    extern __shared__ float sm[];
    const int cap = n_pos;
    if (pos_dev) n_pos = min(*pos_dev + 1, cap);
    const int V8 = hd / 8, PG = AV_THREADS / V8;
    float* sq = sm;                  // [hd]
    float* sp = sm + hd;             // [cap] scores, then probabilities
    float* part = sp + cap;          // [PG][hd]
    __shared__ float redf[32];
    __shared__ double redd[32];
    const int h = blockIdx.x, kvh = h / (n_head / n_kv);
    const int64_t rs = (int64_t)n_kv * hd;           // cache row stride (elements)
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sq[i] = q[(int64_t)h * hd + i];
    __syncthreads();
    for (int j = threadIdx.x; j < n_pos; j += blockDim.x) {
        const KT* kr = kc + j * rs + (int64_t)kvh * hd;
        float s = 0.f;
        for (int v = 0; v < V8; v += 2) {            // two 16-byte loads in flight (V8 is even or 1)
            float f0[8], f1[8];
            kv_get8(kr + 8 * v, f0);
            if (v + 1 < V8) kv_get8(kr + 8 * v + 8, f1);
#pragma unroll
            for (int i = 0; i < 8; ++i) s += sq[8 * v + i] * f0[i];
            if (v + 1 < V8) {
#pragma unroll
                for (int i = 0; i < 8; ++i) s += sq[8 * v + 8 + i] * f1[i];
            }
        }
        sp[j] = s * scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n_pos; j += blockDim.x) mx = fmaxf(mx, sp[j]);
    mx = block_max_f(mx, redf);
    double sum = 0.0;
    for (int j = threadIdx.x; j < n_pos; j += blockDim.x) {
        const float e = expf(sp[j] - mx);
        sp[j] = e;
        sum += (double)e;
    }
    sum = block_sum_d(sum, redd);
    const float inv = (float)(1.0 / sum);
    __syncthreads();
    {
        const int g = threadIdx.x / V8, v = threadIdx.x - g * V8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        const KT* vb = vc + (int64_t)kvh * hd + 8 * v;
        int j = g;
        for (; j + PG < n_pos; j += 2 * PG) {        // two rows in flight
            float f0[8], f1[8];
            kv_get8(vb + j * rs, f0);
            kv_get8(vb + (j + PG) * rs, f1);
            const float p0 = sp[j] * inv, p1 = sp[j + PG] * inv;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += p0 * f0[i];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += p1 * f1[i];
        }
        if (j < n_pos) {
            float f0[8];
            kv_get8(vb + j * rs, f0);
            const float p0 = sp[j] * inv;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += p0 * f0[i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) part[g * hd + 8 * v + i] = acc[i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.f;
        for (int g = 0; g < PG; ++g) acc += part[g * hd + i];
        if (gate) acc *= sigmoid_f(gate[(int64_t)h * gstride + i]);
        out[(int64_t)h * hd + i] = acc;
    }
}

// ---- fused: out = RMSNorm(x) * w, quantised to Q8_K (one CTA; thread t holds value 256j + t of
//      every 256-value block j, so a block's maximum is one CTA-wide reduction per j) ----
template <int NB>
__global__ void __launch_bounds__(256) k_rmsnorm_q8(const float* __restrict__ x, int H, float eps,
                                                    const float* __restrict__ w, int8_t* __restrict__ q,
                                                    float* __restrict__ d, int* __restrict__ bs) {
    pdl_enter();
    __shared__ double redd[32];
    __shared__ float samax[8][NB];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float v[NB];
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        v[j] = x[256 * j + t];
        ss += (double)(v[j] * v[j]);
    }
    ss = block_sum_d(ss, redd);
    const float scale = 1.0f / sqrtf((float)(ss / H) + eps);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        v[j] = (v[j] * scale) * w[256 * j + t];
        const float am = warp_max(fabsf(v[j]));
        if (lane == 0) samax[warp][j] = am;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        float am = samax[0][j];
#pragma unroll
        for (int u = 1; u < 8; ++u) am = fmaxf(am, samax[u][j]);
        int qi = 0;
        float dd = 0.f;
        if (am != 0.f) {
            const float iscale = 127.f / am;
            qi = min(127, __float2int_rn(iscale * v[j]));
            dd = 1.f / iscale;
        }
        q[256 * j + t] = (int8_t)qi;
        int sum = qi;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((t & 15) == 0) bs[16 * j + (t >> 4)] = sum;
        if (t == 0) d[j] = dd;
    }
}

// ---- several projections of one Q8_K activation in one launch: rows of the matrices back to back,
//      one warp per row ----
struct GemvSet {
    const uint8_t* w[3];
    float* y[3];
    const float* resid[3];
    int N[3];
    int type[3];
    int n;
};
__global__ void __launch_bounds__(256) k_qgemv_set(GemvSet g, int K, const int8_t* __restrict__ xq,
                                                   const float* __restrict__ xd, const int* __restrict__ xbs) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    int m = 0;
    while (m < g.n && n >= g.N[m]) n -= g.N[m++];
    if (m >= g.n) return;
    const int nb = K / QK;
    const ActRow a{xq, xd, xbs};
    const float v = warp_sum(g.type[m] == T_Q4K ? row_dot_lane<T_Q4K>(g.w[m], (int64_t)g.N[m] * nb, n, nb, a, lane)
                                                : row_dot_lane<T_Q6K>(g.w[m], (int64_t)g.N[m] * nb, n, nb, a, lane));
    if (lane == 0) g.y[m][n] = g.resid[m] ? v + g.resid[m][n] : v;
}

// ---- fused QK RMSNorm (mode 1: over the whole projection, weights [n*hd]; mode 2: per head, weights
//      [hd]; 0: none) + NEOX RoPE + KV store: one CTA per q or k head, one thread per rotated pair.
//      Rotated q goes to q_out (mode 1 reads the whole input vector in every CTA); rotated k and v
//      go to the caches ----
template <typename KT>
__global__ void __launch_bounds__(128) k_qknorm_rope_store(const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v, const float* __restrict__ qn,
                                                           const float* __restrict__ kn, int mode, float eps,
                                                           int n_head, int n_kv, int hd, int q_stride, int rope_dim,
                                                           int pos, const int32_t* __restrict__ pos_dev, int max_ctx,
                                                           float theta_scale, float* __restrict__ q_out,
                                                           KT* __restrict__ kc, KT* __restrict__ vc) {
    pdl_enter();
    __shared__ double redd[32];
    if (pos_dev) pos = *pos_dev;
    if (pos < 0 || pos >= max_ctx) return;
    const int head = blockIdx.x;
    const bool isq = head < n_head;
    const int hh = isq ? head : head - n_head;
    const float* vec = isq ? q : k;
    const int nvec = (isq ? n_head : n_kv) * hd;
    const float* wn = isq ? qn : kn;
    const float* xh = vec + (int64_t)hh * (isq ? q_stride : hd);
    const int rh = rope_dim / 2;
    float scale = 1.f;
    if (mode != 0) {
        const double ss = block_sum_d(mode == 1 ? sumsq_stride128(vec, nvec, threadIdx.x)
                                                : sumsq_stride128(xh, hd, threadIdx.x), redd);
        scale = 1.0f / sqrtf((float)(ss / (mode == 1 ? nvec : hd)) + eps);
    }
    auto normed = [&](int j) {
        const float x = xh[j];
        if (mode == 1) return (x * scale) * wn[hh * hd + j];
        if (mode == 2) return (x * scale) * wn[j];
        return x;
    };
    auto put = [&](int j, float r) {
        if (isq) {
            q_out[(int64_t)hh * hd + j] = r;
        } else {
            const int64_t o = ((int64_t)pos * n_kv + hh) * hd;
            kv_put(kc + o + j, r);
        }
    };
    // NEOX rotation of the first rope_dim values (pairs j, j + rope_dim/2, theta_j = pos * base^(-2j/rope_dim));
    // values past rope_dim pass through
    for (int j = threadIdx.x; j < hd; j += blockDim.x) {
        if (j < rh) {
            const float x0 = normed(j), x1 = normed(j + rh);
            float theta = (float)pos;
            for (int u = 0; u < j; ++u) theta *= theta_scale;
            const float c = cosf(theta), sn = sinf(theta);
            put(j, x0 * c - x1 * sn);
            put(j + rh, x0 * sn + x1 * c);
        } else if (j >= rope_dim) {
            put(j, normed(j));
        }
        if (!isq) {
            const int64_t o = ((int64_t)pos * n_kv + hh) * hd;
            kv_put(vc + o + j, v[(int64_t)hh * hd + j]);
        }
    }
}

// ---- argmax (first index of the maximum) of n floats: one CTA of 1024 threads ----
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ v, int n, int32_t* __restrict__ out,
                                                 int32_t* __restrict__ pos, int seq_len) {
    pdl_enter();
    __shared__ float sv[32];
    __shared__ int si[32];
    float best = -INFINITY;
    int bi = 0x7fffffff;
    auto take = [&](float x, int i) {
        if (x > best || (x == best && i < bi)) { best = x; bi = i; }
    };
    // 16-byte loads, four in flight per thread (v is 16-byte aligned), then the scalar tail
    const int n4 = (reinterpret_cast<uintptr_t>(v) & 15) ? 0 : n / 4;
    const float4* v4 = reinterpret_cast<const float4*>(v);
    for (int q0 = threadIdx.x; q0 < n4; q0 += 4 * blockDim.x) {
        float4 c[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int q = q0 + u * blockDim.x;
            c[u] = q < n4 ? v4[q] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int q = q0 + u * blockDim.x;
            if (q < n4) { take(c[u].x, 4 * q); take(c[u].y, 4 * q + 1); take(c[u].z, 4 * q + 2); take(c[u].w, 4 * q + 3); }
        }
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) take(v[i], i);
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        best = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
        bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) {
            const int r = bi == 0x7fffffff ? 0 : bi;
            if (!pos) {
                *out = r;
            } else {                                 // out[*pos + 1] = r, then the position advances
                const int p = *pos + 1;
                if (p < seq_len) out[p] = r;
                *pos = p;
            }
        }
    }
}

}  // namespace

cudaError_t launch_rmsnorm_q8(const float* x, int H, float eps, const float* w, int8_t* q, float* d, int* bs,
                              cudaStream_t s) {
    switch (H / QK) {
        case 1: return launch_pdl(k_rmsnorm_q8<1>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        case 2: return launch_pdl(k_rmsnorm_q8<2>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        case 4: return launch_pdl(k_rmsnorm_q8<4>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        case 8: return launch_pdl(k_rmsnorm_q8<8>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        case 16: return launch_pdl(k_rmsnorm_q8<16>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        case 32: return launch_pdl(k_rmsnorm_q8<32>, 1, 256, 0, s, x, H, eps, w, q, d, bs);
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_qgemv_set(int n, const int* types, const uint8_t* const* w, const int* N, int K,
                             const float* const* resid, float* const* y, const int8_t* xq, const float* xd,
                             const int* xbs, cudaStream_t s) {
    if (n < 1 || n > 3) return cudaErrorInvalidValue;
    GemvSet g{};
    int64_t rows = 0;
    for (int m = 0; m < n; ++m) {
        g.w[m] = w[m];
        g.y[m] = y[m];
        g.resid[m] = resid ? resid[m] : nullptr;
        g.N[m] = N[m];
        g.type[m] = types[m];
        rows += N[m];
    }
    g.n = n;
    return launch_pdl(k_qgemv_set, (unsigned)((rows + 7) / 8), 256, 0, s, g, K, xq, xd, xbs);
}

cudaError_t launch_qknorm_rope_store(const float* q, const float* k, const float* v, const float* qn, const float* kn,
                                     int mode, float eps, int n_head, int n_kv, int hd, int q_stride, int rope_dim,
                                     int pos, const int32_t* pos_dev, int max_ctx, float freq_base, float* q_out,
                                     void* kc, void* vc, bool kv_bf16, cudaStream_t s) {
    if (rope_dim < 2 || rope_dim > hd || rope_dim % 2 || q_stride < hd || (mode == 1 && q_stride != hd))
        return cudaErrorInvalidValue;
    const float theta_scale = powf(freq_base, -2.0f / (float)rope_dim);
    if (kv_bf16)
        return launch_pdl(k_qknorm_rope_store<__nv_bfloat16>, n_head + n_kv, 128, 0, s, q, k, v, qn, kn, mode, eps,
                          n_head, n_kv, hd, q_stride, rope_dim, pos, pos_dev, max_ctx, theta_scale, q_out,
                          (__nv_bfloat16*)kc, (__nv_bfloat16*)vc);
    return launch_pdl(k_qknorm_rope_store<__half>, n_head + n_kv, 128, 0, s, q, k, v, qn, kn, mode, eps, n_head, n_kv,
                      hd, q_stride, rope_dim, pos, pos_dev, max_ctx, theta_scale, q_out, (__half*)kc, (__half*)vc);
}

cudaError_t launch_embed(int type, const uint8_t* table, int H, int64_t n_vocab, const int32_t* token,
                         const int32_t* pos, float* out, cudaStream_t s) {
    return launch_pdl(k_embed, (H + 255) / 256, 256, 0, s, type, table, H, n_vocab, token, pos, out);
}

cudaError_t launch_rmsnorm_rows(const float* x, int rows, int cols, float eps, const float* w, float* out,
                                cudaStream_t s) {
    return launch_rmsnorm_f32(x, rows, cols, eps, w, out, s);
}

cudaError_t launch_qgemv(int type, const uint8_t* w, int N, int K, const int8_t* xq, const float* xd, const int* xbs,
                         const float* resid, float* y, cudaStream_t s) {
    const unsigned grid = (unsigned)((N + 7) / 8);
    if (type == T_Q4K) return launch_pdl(k_qgemv<T_Q4K>, grid, 256, 0, s, w, N, K, xq, xd, xbs, resid, y);
    return launch_pdl(k_qgemv<T_Q6K>, grid, 256, 0, s, w, N, K, xq, xd, xbs, resid, y);
    return cudaGetLastError();
}

cudaError_t launch_rope_store(float* q, float* k, const float* v, int n_head, int n_kv, int hd, int pos,
                              const int32_t* pos_dev, int max_ctx, float freq_base, void* kc, void* vc, bool kv_bf16,
                              cudaStream_t s) {
    const float theta_scale = powf(freq_base, -2.0f / (float)hd);
    const int n = (n_head + n_kv) * (hd / 2);
    if (kv_bf16)
        k_rope_store<<<(n + 255) / 256, 256, 0, s>>>(q, k, v, n_head, n_kv, hd, pos, pos_dev, max_ctx, theta_scale,
                                                     (__nv_bfloat16*)kc, (__nv_bfloat16*)vc);
    else
        k_rope_store<<<(n + 255) / 256, 256, 0, s>>>(q, k, v, n_head, n_kv, hd, pos, pos_dev, max_ctx, theta_scale,
                                                     (__half*)kc, (__half*)vc);
    return cudaGetLastError();
}

size_t attention_smem(int hd, int n_pos) {
    if (hd % 8 == 0) return (size_t)(hd + n_pos + (AV_THREADS / (hd / 8)) * hd) * sizeof(float);
    return (size_t)(hd + n_pos + (ATT_THREADS / hd) * hd) * sizeof(float);
}

template <typename KT>
static cudaError_t attention_t(const float* q, const void* kc, const void* vc, int n_head, int n_kv, int hd, int n_pos,
                               const int32_t* pos_dev, float scale, const float* gate, int gstride, float* out,
                               cudaStream_t s) {
    const size_t smem = attention_smem(hd, n_pos);
    const bool v8 = hd % 8 == 0;
    const void* fn = v8 ? (const void*)k_attention_v8<KT> : (const void*)k_attention<KT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    if (v8)
        return launch_pdl(k_attention_v8<KT>, n_head, AV_THREADS, smem, s, q, (const KT*)kc, (const KT*)vc, n_head,
                          n_kv, hd, n_pos, pos_dev, scale, gate, gstride, out);
    return launch_pdl(k_attention<KT>, n_head, ATT_THREADS, smem, s, q, (const KT*)kc, (const KT*)vc, n_head, n_kv, hd,
                      n_pos, pos_dev, scale, gate, gstride, out);
}

cudaError_t launch_attention(const float* q, const void* kc, const void* vc, bool kv_bf16, int n_head, int n_kv,
                             int hd, int n_pos, const int32_t* pos_dev, float scale, const float* gate, int gstride,
                             float* out, cudaStream_t s) {
    return kv_bf16 ? attention_t<__nv_bfloat16>(q, kc, vc, n_head, n_kv, hd, n_pos, pos_dev, scale, gate, gstride, out, s)
                   : attention_t<__half>(q, kc, vc, n_head, n_kv, hd, n_pos, pos_dev, scale, gate, gstride, out, s);
}

// ---- gated delta-net decode step (one token), one CTA of GDN_THREADS per value head h ----------------
// qkv [conv_dim] = [q: Hk*D | k: Hk*D | v: Hv*D] projection outputs before the causal conv; the conv
// keeps the last d_conv inputs in a ring (slot = position % d_conv; positions < 0 read as zero), the
// weights ne = [d_conv, conv_dim] (tap t of channel c at c*d_conv + t, tap d_conv-1 = this token).
// Value head h uses key head h / (Hv/Hk). With x = silu(conv): q, k L2-normalised (1/max(|x|, eps)),
// q scaled by 1/sqrt(D); beta = sigmoid(b_h), decay = exp(softplus(a_h + dt_bias_h) * ssm_a_h) with
// (b_h, a_h) from ba's per-key-head groups [Hv/Hk betas | Hv/Hk alphas];
//   S <- decay * S;  delta = beta * (v - S^T k);  S <- S + k delta^T;  o = S^T q
// (S[h] = [D key][D value] f32), then out_h = RMSNorm(o) * norm_w * silu(z_h).
constexpr int GDN_D = 128;
constexpr int GDN_THREADS = 256;
__global__ void __launch_bounds__(GDN_THREADS) k_gdn_step(const float* __restrict__ qkv, const float* __restrict__ z,
                                                          const float* __restrict__ ba, const float* __restrict__ conv_w,
                                                          float* __restrict__ ring, const float* __restrict__ dt_bias,
                                                          const float* __restrict__ ssm_a, const float* __restrict__ norm_w,
                                                          float* __restrict__ state, int Hv, int Hk, int d_conv,
                                                          float eps, int pos, const int32_t* __restrict__ pos_dev,
                                                          float* __restrict__ out) {
    pdl_enter();
    __shared__ float sq[GDN_D], sk[GDN_D], sv[GDN_D], s_red[2][GDN_D];
    __shared__ double redd[32];
    if (pos_dev) pos = *pos_dev;
    const int h = blockIdx.x, vpg = Hv / Hk, g = h / vpg, r = h - g * vpg;
    const int conv_dim = 2 * Hk * GDN_D + Hv * GDN_D;
    const int t = threadIdx.x;
    // causal conv + silu of this head's q, k (threads 0..127) and v (threads 128..255) channels
    auto conv = [&](int c) {
        const float xn = qkv[c];
        float acc = xn * conv_w[(int64_t)c * d_conv + d_conv - 1];
        for (int u = 0; u < d_conv - 1; ++u) {               // tap u: position pos - (d_conv - 1) + u
            const int p = pos - (d_conv - 1) + u;
            if (p >= 0) acc += ring[(int64_t)(p % d_conv) * conv_dim + c] * conv_w[(int64_t)c * d_conv + u];
        }
        ring[(int64_t)(pos % d_conv) * conv_dim + c] = xn;    // read by the next d_conv - 1 positions
        return silu_f(acc);
    };
    if (t < GDN_D) {
        sq[t] = conv(g * GDN_D + t);
        sk[t] = conv(Hk * GDN_D + g * GDN_D + t);
    } else {
        sv[t - GDN_D] = conv(2 * Hk * GDN_D + h * GDN_D + (t - GDN_D));
    }
    __syncthreads();
    // L2 norms of q and k (double sums), q also scaled by 1/sqrt(D)
    const double qq = block_sum_d(t < GDN_D ? (double)(sq[t] * sq[t]) : 0.0, redd);
    const double kk = block_sum_d(t < GDN_D ? (double)(sk[t] * sk[t]) : 0.0, redd);
    const float qs = (1.0f / fmaxf(sqrtf((float)qq), eps)) * (1.0f / sqrtf((float)GDN_D));
    const float ks = 1.0f / fmaxf(sqrtf((float)kk), eps);
    const float beta = sigmoid_f(ba[g * 2 * vpg + r]);
    const float araw = ba[g * 2 * vpg + vpg + r] + dt_bias[h];
    const float sp = araw > 20.f ? araw : log1pf(expf(araw));
    const float decay = expf(sp * ssm_a[h]);
    // thread = (value column j, half of the key rows)
    const int j = t & (GDN_D - 1), half = t >> 7;
    float* S = state + (int64_t)h * GDN_D * GDN_D;
    float sreg[GDN_D / 2];
    float kv = 0.f;
#pragma unroll
    for (int u = 0; u < GDN_D / 2; ++u) {
        const int i = half * (GDN_D / 2) + u;
        sreg[u] = S[(int64_t)i * GDN_D + j] * decay;
        kv += sreg[u] * (sk[i] * ks);
    }
    s_red[half][j] = kv;
    __syncthreads();
    const float delta = beta * (sv[j] - (s_red[0][j] + s_red[1][j]));
    __syncthreads();
    float o = 0.f;
#pragma unroll
    for (int u = 0; u < GDN_D / 2; ++u) {
        const int i = half * (GDN_D / 2) + u;
        sreg[u] += (sk[i] * ks) * delta;
        S[(int64_t)i * GDN_D + j] = sreg[u];
        o += sreg[u] * (sq[i] * qs);
    }
    s_red[half][j] = o;
    __syncthreads();
    o = s_red[0][j] + s_red[1][j];
    // gated RMSNorm over the head's D outputs
    const double oo = block_sum_d(half == 0 ? (double)(o * o) : 0.0, redd);
    if (half == 0) {
        const float rs = 1.0f / sqrtf((float)(oo / GDN_D) + eps);
        out[(int64_t)h * GDN_D + j] = ((o * rs) * norm_w[j]) * silu_f(z[(int64_t)h * GDN_D + j]);
    }
}

cudaError_t launch_gdn_step(const float* qkv, const float* z, const float* ba, const float* conv_w, float* ring,
                            const float* dt_bias, const float* ssm_a, const float* norm_w, float* state, int Hv, int Hk,
                            int d_state, int d_conv, float eps, int pos, const int32_t* pos_dev, float* out,
                            cudaStream_t s) {
    if (d_state != GDN_D || Hk <= 0 || Hv <= 0 || Hv % Hk || d_conv < 1 || d_conv > 8) return cudaErrorInvalidValue;
    return launch_pdl(k_gdn_step, Hv, GDN_THREADS, 0, s, qkv, z, ba, conv_w, ring, dt_bias, ssm_a, norm_w, state, Hv,
                      Hk, d_conv, eps, pos, pos_dev, out);
}

cudaError_t launch_argmax(const float* v, int n, int32_t* out, int32_t* pos, int seq_len, cudaStream_t s) {
    return launch_pdl(k_argmax, 1, 1024, 0, s, v, n, out, pos, seq_len);
}

}  // namespace hoard
