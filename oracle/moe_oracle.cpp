// moe_oracle.cpp -- TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline).
//
// A CPU restatement, in plain C++, of the per-layer Mixture-of-Experts op chain that hoard runs
// through ggml: router (RMSNorm -> f32 router GEMV -> softmax over all experts -> top-k ->
// optional renormalisation with clamp) -> per-expert SwiGLU FFN on Q4_K / Q6_K weights ->
// weighted combine into the residual (+ the gated shared expert of the hybrid models).
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may load this library; the product
// path (hoard_b200/libhoard_moe.so) never links or calls it.
//
// Reference call sites restated here (paths inside the hoard project):
//   src/run_moe_stream.cpp:352   fx = ggml_mul(ggml_rms_norm(ffn_inp, eps), ffn_norm)
//   src/run_moe_stream.cpp:353   rlog = ggml_mul_mat(ffn_gate_inp /*f32 [H,E]*/, fx)
//   src/run_moe_stream.cpp:354   probs = ggml_soft_max(rlog)       -- over ALL experts, before top-k
//   src/run_moe_stream.cpp:355   sel = ggml_top_k(probs, n_used)
//   src/run_moe_stream.cpp:356   w = ggml_get_rows(probs, sel)
//   src/run_moe_stream.cpp:371-373  if wnorm: s = sum w; s = max(s, 6.103515625e-5); w /= s
//   src/run_moe_stream.cpp:432-435  g = gate.fx, u = up.fx, h = silu(g)*u, y = down.h  (per expert)
//   src/run_moe_stream.cpp:447   x[d] = sum_j w_j*y_j[d] + ffn_inp[d]  (j ascending, f32)
//   src/run_specloop.cpp:117-123  batched form: host top-k by std::partial_sort, descending
//   src/run_specloop.cpp:132-140  batched form: mul_mat_id over the slot pool, sum over j, + residual
//   src/run_qwen35.cpp:659-666   shared expert: sigmoid(gate_inp_shexp.fx) * down(silu(gate.fx)*up.fx)
//   src/run_qwen35.cpp:675-676   x[d] = (sum_j w_j*y_j[d] + shex[d]) + ffn_inp[d]
//   notes/olmoe_spec.md:60-74    softmax before top-k; no renorm for OLMoE; silu on the gate branch
//
// The arithmetic of those ops lives in ggml (llama.cpp build b9660, not vendored, not installed).
// Its published algorithms are restated from the GGUF format definition and ggml's CPU backend:
//   * Q4_K block (256 weights, 144 B) and Q6_K block (256 weights, 210 B) decoding;
//   * a quantized mul_mat on the CPU backend first quantizes the f32 activation row to Q8_K
//     (per 256 values: d = 1/(127/amax), q = round-to-nearest-even(x*127/amax) clamped to 127,
//     plus 16-value partial sums), then takes integer dot products per sub-block and scales them
//     by the block's fp16 factors.  Mode ORC_MODE_GGML reproduces that; ORC_MODE_EXACT instead
//     dequantises the weights and dots them with the unquantised f32 activation (double sums).
//   * rms_norm accumulates sum(x*x) in double, then scale = 1/sqrtf(mean + eps);
//   * soft_max accumulates sum(expf(x - max)) in double and scales by (float)(1/sum).
// Ties in top-k are broken towards the lower expert id (ggml does not document its tie order).
#include <cstdint>
#include <cstring>
#include <cmath>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

enum { ORC_F32 = 0, ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_Q8_K = 15 };  // GGUF / ggml type ids
enum { ORC_MODE_GGML = 0, ORC_MODE_EXACT = 1 };
enum { QK = 256 };

struct OrcQ8K {            // ggml block_q8_K: f32 delta, 256 int8, 16 partial sums of 16 values
    float d;
    int8_t qs[QK];
    int16_t bsums[QK / 16];
};

float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {                      // subnormal half: renormalise
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400));
            man &= 0x3FF;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t rd16(const uint8_t* p) { uint16_t v; std::memcpy(&v, p, 2); return v; }

int orc_block_bytes(int type) {
    switch (type) {
        case ORC_Q4_K: return 144;
        case ORC_Q6_K: return 210;
        case ORC_F32: return 4 * QK;
        default: return -1;
    }
}

// Q4_K: 6-bit (scale, min) pair j of the 12 packed bytes (GGUF format definition).
static inline void q4k_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Decodes nblocks Q4_K blocks into nblocks*256 floats: y = (d*sc)*q - (dmin*m).
void orc_dequant_q4k(const uint8_t* blocks, int64_t nblocks, float* out) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 144;
        const float d = orc_fp16_to_fp32(rd16(blk));
        const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        float* y = out + b * QK;
        for (int g = 0; g < 4; ++g) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(2 * g, scales, &sc0, &m0);
            q4k_scale_min(2 * g + 1, scales, &sc1, &m1);
            const float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
            const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            for (int l = 0; l < 32; ++l) y[64 * g + l] = d0 * (float)(qs[32 * g + l] & 0xF) - mm0;
            for (int l = 0; l < 32; ++l) y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - mm1;
        }
    }
}

// Q6_K: element e of a block -> signed 6-bit value (q - 32) and its int8 scale index (e/16).
static inline int q6k_value(const uint8_t* blk, int e) {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int half = e >> 7;          // 128-element halves
    const int r = e & 127;
    const int a = r >> 5;             // which of the 4 interleaved 32-runs
    const int l = r & 31;
    const uint8_t lo = ql[64 * half + l + 32 * (a & 1)];
    const int low4 = (a < 2) ? (lo & 0xF) : (lo >> 4);
    const int hi2 = (qh[32 * half + l] >> (2 * a)) & 3;
    return (low4 | (hi2 << 4)) - 32;
}

// Decodes nblocks Q6_K blocks: y = d * sc[e/16] * (q - 32).
void orc_dequant_q6k(const uint8_t* blocks, int64_t nblocks, float* out) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 210;
        const int8_t* sc = (const int8_t*)(blk + 192);
        const float d = orc_fp16_to_fp32(rd16(blk + 208));
        float* y = out + b * QK;
        for (int e = 0; e < QK; ++e) y[e] = d * (float)sc[e >> 4] * (float)q6k_value(blk, e);
    }
}

int orc_dequant(int type, const uint8_t* blocks, int64_t nblocks, float* out) {
    if (type == ORC_Q4_K) { orc_dequant_q4k(blocks, nblocks, out); return 0; }
    if (type == ORC_Q6_K) { orc_dequant_q6k(blocks, nblocks, out); return 0; }
    if (type == ORC_F32) { std::memcpy(out, blocks, (size_t)nblocks * QK * 4); return 0; }
    return -1;
}

// ggml's nearest_int: round to nearest, ties to even (default FP environment).
static inline int nearest_int(float fval) {
    float val = fval + 12582912.f;
    int i;
    std::memcpy(&i, &val, 4);
    return (i & 0x007fffff) - 0x00400000;
}

// Q8_K activation quantisation of n (multiple of 256) floats.
void orc_quantize_q8k(const float* x, int64_t n, OrcQ8K* y) {
    for (int64_t b = 0; b < n / QK; ++b) {
        const float* xb = x + b * QK;
        float amax = 0.f, mx = 0.f;
        for (int j = 0; j < QK; ++j) {
            const float ax = std::fabs(xb[j]);
            if (ax > amax) { amax = ax; mx = xb[j]; }
        }
        if (amax == 0.f) {
            y[b].d = 0.f;
            std::memset(y[b].qs, 0, QK);
            std::memset(y[b].bsums, 0, sizeof(y[b].bsums));
            continue;
        }
        const float iscale = -127.f / mx;
        for (int j = 0; j < QK; ++j) {
            const int v = nearest_int(iscale * xb[j]);
            y[b].qs[j] = (int8_t)std::min(127, v);
        }
        for (int j = 0; j < QK / 16; ++j) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += y[b].qs[16 * j + i];
            y[b].bsums[j] = (int16_t)s;
        }
        y[b].d = 1.f / iscale;
    }
}

// Flat export of the Q8_K quantiser for tests: d[n/256], qs[n], bsums[n/16].
void orc_quantize_q8k_flat(const float* x, int64_t n, float* d, int8_t* qs, int16_t* bsums) {
    std::vector<OrcQ8K> tmp((size_t)(n / QK));
    orc_quantize_q8k(x, n, tmp.data());
    for (int64_t b = 0; b < n / QK; ++b) {
        d[b] = tmp[b].d;
        std::memcpy(qs + b * QK, tmp[b].qs, QK);
        std::memcpy(bsums + b * 16, tmp[b].bsums, 32);
    }
}

// Q4_K row . Q8_K activation: per block, d8*d*sum_sb(sc*isum_sb) - d8*dmin*sum_sb(m*bsum_sb).
static float dot_q4k_q8k(const uint8_t* row, const OrcQ8K* a, int nb) {
    float sumf = 0.f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = row + (size_t)b * 144;
        const float d = orc_fp16_to_fp32(rd16(blk));
        const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        int32_t isum = 0, msum = 0;
        for (int g = 0; g < 4; ++g) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(2 * g, scales, &sc0, &m0);
            q4k_scale_min(2 * g + 1, scales, &sc1, &m1);
            int32_t s0 = 0, s1 = 0;
            for (int l = 0; l < 32; ++l) {
                s0 += (int32_t)(qs[32 * g + l] & 0xF) * a[b].qs[64 * g + l];
                s1 += (int32_t)(qs[32 * g + l] >> 4) * a[b].qs[64 * g + 32 + l];
            }
            isum += sc0 * s0 + sc1 * s1;
            msum += m0 * (a[b].bsums[4 * g] + a[b].bsums[4 * g + 1]) +
                    m1 * (a[b].bsums[4 * g + 2] + a[b].bsums[4 * g + 3]);
        }
        sumf += a[b].d * d * (float)isum - a[b].d * dmin * (float)msum;
    }
    return sumf;
}

// Q6_K row . Q8_K activation: per block, d8*d*sum_i(sc_i * sum(q6*q8)) over 16-value groups.
static float dot_q6k_q8k(const uint8_t* row, const OrcQ8K* a, int nb) {
    float sumf = 0.f;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = row + (size_t)b * 210;
        const int8_t* sc = (const int8_t*)(blk + 192);
        const float d = orc_fp16_to_fp32(rd16(blk + 208));
        int32_t isum = 0;
        for (int grp = 0; grp < 16; ++grp) {
            int32_t s = 0;
            for (int i = 0; i < 16; ++i) s += q6k_value(blk, 16 * grp + i) * a[b].qs[16 * grp + i];
            isum += (int32_t)sc[grp] * s;
        }
        sumf += a[b].d * d * (float)isum;
    }
    return sumf;
}

// y[N] = W[N rows of K] . x[K], W in GGUF row layout (rows of K/256 blocks).
static void matvec(int type, const uint8_t* W, int N, int K, const float* x, float* y, int mode) {
    const int nb = K / QK;
    const int bb = orc_block_bytes(type);
    if (type == ORC_F32) {
        const float* Wf = (const float*)W;
        for (int n = 0; n < N; ++n) {
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += (double)Wf[(size_t)n * K + k] * (double)x[k];
            y[n] = (float)s;
        }
        return;
    }
    if (mode == ORC_MODE_GGML) {
        std::vector<OrcQ8K> a((size_t)nb);
        orc_quantize_q8k(x, K, a.data());
        // rows in parallel when the caller is not already parallel over tokens (ggml's CPU
        // backend also splits a mul_mat's rows across its threads)
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && N >= 64)
#endif
        for (int n = 0; n < N; ++n) {
            const uint8_t* row = W + (size_t)n * nb * bb;
            y[n] = (type == ORC_Q4_K) ? dot_q4k_q8k(row, a.data(), nb) : dot_q6k_q8k(row, a.data(), nb);
        }
    } else {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && N >= 64)
#endif
        for (int n = 0; n < N; ++n) {
            std::vector<float> wrow((size_t)K);
            orc_dequant(type, W + (size_t)n * nb * bb, nb, wrow.data());
            double s = 0.0;
            for (int k = 0; k < K; ++k) s += (double)wrow[k] * (double)x[k];
            y[n] = (float)s;
        }
    }
}

int orc_matvec(int type, const uint8_t* W, int N, int K, const float* x, float* y, int mode) {
    if (K % QK != 0 || orc_block_bytes(type) < 0) return -1;
    matvec(type, W, N, K, x, y, mode);
    return 0;
}

// rms_norm(x) * w over rows of H.
void orc_rms_norm(const float* x, const float* w, int T, int H, float eps, float* out) {
    for (int t = 0; t < T; ++t) {
        const float* xr = x + (size_t)t * H;
        double sum = 0.0;
        for (int i = 0; i < H; ++i) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / H);
        const float scale = 1.0f / std::sqrt(mean + eps);
        for (int i = 0; i < H; ++i) out[(size_t)t * H + i] = (xr[i] * scale) * w[i];
    }
}

// softmax over E logits (max-subtracted, double sum, scaled by (float)(1/sum)).
void orc_softmax(const float* logits, int E, float* p) {
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = std::max(mx, logits[e]);
    double sum = 0.0;
    for (int e = 0; e < E; ++e) {
        const float v = std::exp(logits[e] - mx);
        p[e] = v;
        sum += (double)v;
    }
    const float inv = (float)(1.0 / sum);
    for (int e = 0; e < E; ++e) p[e] *= inv;
}

// top-k of probabilities, descending, ties to the lower expert id; optional renorm with clamp.
void orc_topk(const float* p, int E, int k, int renorm, int32_t* sel, float* w) {
    std::vector<int> idx((size_t)E);
    for (int e = 0; e < E; ++e) idx[e] = e;
    std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), [&](int a, int b) {
        return p[a] > p[b] || (p[a] == p[b] && a < b);
    });
    for (int j = 0; j < k; ++j) { sel[j] = idx[j]; w[j] = p[idx[j]]; }
    if (renorm) {
        float s = 0.f;
        for (int j = 0; j < k; ++j) s += w[j];
        if (s < 6.103515625e-5f) s = 6.103515625e-5f;
        for (int j = 0; j < k; ++j) w[j] /= s;
    }
}

static inline float silu(float x) { return x / (1.0f + std::exp(-x)); }
static inline float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// Router for T tokens: fx = rms_norm(x)*w_norm; probs = softmax(W_r . fx); top-k (+renorm).
// W_r is the GGUF f32 tensor ffn_gate_inp with ne = [H, E]: E rows of H floats.
void orc_route(const float* x, int T, int H, int E, int k, int renorm, float eps,
               const float* w_norm, const float* w_router,
               float* fx, float* probs, int32_t* sel, float* w, int nthreads) {
    orc_rms_norm(x, w_norm, T, H, eps, fx);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int t = 0; t < T; ++t) {
        std::vector<float> logits((size_t)E);
        matvec(ORC_F32, (const uint8_t*)w_router, E, H, fx + (size_t)t * H, logits.data(), ORC_MODE_EXACT);
        orc_softmax(logits.data(), E, probs + (size_t)t * E);
        orc_topk(probs + (size_t)t * E, E, k, renorm, sel + (size_t)t * k, w + (size_t)t * k);
    }
}

// One SwiGLU expert on one activation row: y[H] = down . (silu(gate.fx) * (up.fx)).
static void expert_ffn(int H, int I, int gt, int ut, int dt,
                       const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                       const float* fx, float* y, int mode) {
    std::vector<float> g((size_t)I), u((size_t)I), h((size_t)I);
    matvec(gt, gate, I, H, fx, g.data(), mode);
    matvec(ut, up, I, H, fx, u.data(), mode);
    for (int i = 0; i < I; ++i) h[i] = silu(g[i]) * u[i];
    matvec(dt, down, H, I, h.data(), y, mode);
}

int orc_expert_ffn(int H, int I, int gt, int ut, int dt,
                   const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                   const float* fx, float* y, int mode) {
    if (H % QK || I % QK) return -1;
    expert_ffn(H, I, gt, ut, dt, gate, up, down, fx, y, mode);
    return 0;
}

static size_t mat_bytes(int type, int N, int K) { return (size_t)N * (K / QK) * orc_block_bytes(type); }

// Experts + combine for T tokens given the routing (sel, w) and the normed activations fx.
// gate/up/down hold E experts back to back in GGUF layout ([K_in, N_out, E], per-expert stride
// = nbytes/E). Shared expert (I_sh > 0) adds sigmoid(sh_gate_inp . fx) * FFN_sh(fx) unweighted.
// out = (sum_j w_j*y_j + shex) + resid.
int orc_moe_experts(int H, int E, int k, int I, int gt, int ut, int dt,
                    const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                    int I_sh, int sgt, int sut, int sdt,
                    const uint8_t* sh_gate, const uint8_t* sh_up, const uint8_t* sh_down,
                    const float* sh_gate_inp,
                    const float* fx, const float* resid, int T, const int32_t* sel, const float* w,
                    int mode, int nthreads, float* out) {
    if (H % QK || I % QK || (I_sh > 0 && I_sh % QK)) return -1;
    for (int64_t i = 0; i < (int64_t)T * k; ++i)
        if (sel[i] < 0 || sel[i] >= E) return -2;          // invalid expert id
    const size_t gs = mat_bytes(gt, I, H), us = mat_bytes(ut, I, H), ds = mat_bytes(dt, H, I);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) if (T > 1)
#endif
    for (int t = 0; t < T; ++t) {
        std::vector<float> ys((size_t)k * H), shex((size_t)H, 0.f);
        const float* f = fx + (size_t)t * H;
        for (int j = 0; j < k; ++j) {
            const int e = sel[(size_t)t * k + j];
            expert_ffn(H, I, gt, ut, dt, gate + (size_t)e * gs, up + (size_t)e * us, down + (size_t)e * ds,
                       f, ys.data() + (size_t)j * H, mode);
        }
        if (I_sh > 0) {
            expert_ffn(H, I_sh, sgt, sut, sdt, sh_gate, sh_up, sh_down, f, shex.data(), mode);
            double gs_dot = 0.0;
            for (int i = 0; i < H; ++i) gs_dot += (double)sh_gate_inp[i] * (double)f[i];
            const float sg = sigmoid((float)gs_dot);
            for (int i = 0; i < H; ++i) shex[i] = shex[i] * sg;
        }
        for (int d = 0; d < H; ++d) {
            float acc = 0.f;
            for (int j = 0; j < k; ++j) acc += w[(size_t)t * k + j] * ys[(size_t)j * H + d];
            out[(size_t)t * H + d] = (acc + shex[d]) + resid[(size_t)t * H + d];
        }
    }
    return 0;
}

// The whole layer: route then experts + combine. x is the residual ffn_inp [T, H].
int orc_moe_layer(int H, int E, int k, int I, int renorm, float eps,
                  int gt, int ut, int dt,
                  const float* w_norm, const float* w_router,
                  const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                  int I_sh, int sgt, int sut, int sdt,
                  const uint8_t* sh_gate, const uint8_t* sh_up, const uint8_t* sh_down,
                  const float* sh_gate_inp,
                  const float* x, int T, int mode, int nthreads,
                  float* out, int32_t* sel, float* w, float* fx_out, float* probs_out) {
    if (k <= 0 || k > E) return -1;
    std::vector<float> fx((size_t)T * H), probs((size_t)T * E);
    orc_route(x, T, H, E, k, renorm, eps, w_norm, w_router, fx.data(), probs.data(), sel, w, nthreads);
    if (fx_out) std::memcpy(fx_out, fx.data(), fx.size() * 4);
    if (probs_out) std::memcpy(probs_out, probs.data(), probs.size() * 4);
    return orc_moe_experts(H, E, k, I, gt, ut, dt, gate, up, down, I_sh, sgt, sut, sdt,
                           sh_gate, sh_up, sh_down, sh_gate_inp, fx.data(), x, T, sel, w, mode,
                           nthreads, out);
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

}  // extern "C"
