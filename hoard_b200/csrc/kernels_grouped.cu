// kernels_grouped.cu -- the router and the token-grouped expert path, valid for any T.
//
// One MoE layer for T tokens runs as:
//   k_route         RMSNorm -> f32 router GEMV -> softmax over all E -> top-k (+renorm), per token
//   k_quant_q8      Q8_K quantisation of the normed activations fx
//   k_dispatch      group the (token, j) pairs by pool slot (counting sort, one CTA)
//   k_gateup        per slot and row tile: h = silu(gate . fx) * (up . fx) for the slot's tokens
//   k_quant_q8      Q8_K quantisation of h
//   k_down          per slot and row tile: y = down . h for the slot's tokens
//   k_combine       x = (sum_j w_j * y_j + sigmoid(g_sh . fx) * y_sh) + x, j ascending
// which restates graph A's router tail and graph B of hoard (src/run_moe_stream.cpp:352-373,
// :425-447) and the batched mul_mat_id form (src/run_specloop.cpp:115-140).
#include "common.cuh"
#include "kernels.h"
#include "block_ops.cuh"

namespace hoard {

// ---------------------------------------------------------------------------------------------
// repack: GGUF blocks -> plane layout (one thread per source byte; coalesced reads)
// ---------------------------------------------------------------------------------------------
__global__ void k_repack(int type, const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t nblk) {
    const int bb = block_bytes(type);
    const int64_t total = nblk * bb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / bb;
        const int o = (int)(i - b * bb);
        int64_t off;
        if (type == T_Q4K) {
            off = (o < 16) ? nblk * 128 + b * 16 + o : b * 128 + (o - 16);
        } else {
            if (o < 128) off = b * 128 + o;
            else if (o < 192) off = nblk * 128 + b * 64 + (o - 128);
            else if (o < 208) off = nblk * 192 + b * 16 + (o - 192);
            else off = nblk * 208 + b * 2 + (o - 208);
        }
        dst[off] = src[i];
    }
}

cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int64_t nblk, cudaStream_t s) {
    if (type != T_Q4K && type != T_Q6K) return cudaErrorInvalidValue;
    const int64_t total = nblk * block_bytes(type);
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    k_repack<<<(unsigned)(blocks < 65535 * 8 ? blocks : 65535 * 8), threads, 0, s>>>(type, src, dst, nblk);
    return cudaGetLastError();
}

__global__ void k_transpose(const float* __restrict__ src, float* __restrict__ dst, int R, int C) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < C) tile[i][threadIdx.x] = src[(int64_t)r * C + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < C) dst[(int64_t)c * R + r] = tile[threadIdx.x][i];
    }
}

cudaError_t launch_transpose(const float* src, float* dst, int R, int C, cudaStream_t s) {
    k_transpose<<<dim3((C + 31) / 32, (R + 31) / 32), dim3(32, 8), 0, s>>>(src, dst, R, C);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// router: TT tokens per CTA; fx in shared memory; warp per expert row with double accumulation
// ---------------------------------------------------------------------------------------------
constexpr int ROUTE_TT = 4;
constexpr int MAX_K = 16;

template <typename R>
__global__ void __launch_bounds__(256) k_route(const R* __restrict__ x, int T, int H, int E, int k, int renorm,
                                               float eps, const float* __restrict__ w_norm,
                                               const float* __restrict__ w_router, float* __restrict__ fx_out,
                                               int32_t* sel_out, float* w_out) {
    extern __shared__ __align__(16) float smem[];
    float* fxs = smem;                    // [TT][H]
    float* lg = smem + ROUTE_TT * H;      // [TT][E]
    __shared__ double redd[32];
    __shared__ float redf[32];
    __shared__ int s_sel[MAX_K];
    __shared__ float s_w[MAX_K];
    const int t0 = blockIdx.x * ROUTE_TT;
    const int nt = min(ROUTE_TT, T - t0);
    for (int tt = 0; tt < nt; ++tt) {
        const R* xr = x + (size_t)(t0 + tt) * H;
        double ss = 0.0;
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const float v = to_f32<R>(xr[i]);
            fxs[tt * H + i] = v;
            ss += (double)(v * v);
        }
        ss = block_sum_d(ss, redd);
        const float mean = (float)(ss / H);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            const float v = (fxs[tt * H + i] * scale) * w_norm[i];
            fxs[tt * H + i] = v;
            fx_out[(size_t)(t0 + tt) * H + i] = v;
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int e = warp; e < E; e += nw) {
        double acc[ROUTE_TT];
#pragma unroll
        for (int tt = 0; tt < ROUTE_TT; ++tt) acc[tt] = 0.0;
        const float* wr = w_router + (size_t)e * H;
        for (int i = lane * 4; i < H; i += 128) {
            const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + i));
#pragma unroll
            for (int tt = 0; tt < ROUTE_TT; ++tt) {
                if (tt < nt) {
                    const float4 f = *reinterpret_cast<const float4*>(fxs + tt * H + i);
                    acc[tt] += (double)wv.x * (double)f.x + (double)wv.y * (double)f.y +
                               (double)wv.z * (double)f.z + (double)wv.w * (double)f.w;
                }
            }
        }
#pragma unroll
        for (int tt = 0; tt < ROUTE_TT; ++tt) {
            const double v = warp_sum(acc[tt]);
            if (lane == 0 && tt < nt) lg[tt * E + e] = (float)v;
        }
    }
    __syncthreads();
    for (int tt = 0; tt < nt; ++tt)
        softmax_topk(lg + tt * E, E, k, renorm, sel_out + (size_t)(t0 + tt) * k, w_out + (size_t)(t0 + tt) * k,
                     redd, redf, s_sel, s_w);
}

cudaError_t launch_route(const Dims& d, const LayerWeights& lw, const void* x, int T, float* fx, int32_t* sel,
                         float* w, float* /*sh_gate*/, cudaStream_t s) {
    const size_t smem = (size_t)ROUTE_TT * (d.H + d.E) * sizeof(float);
    const int blocks = (T + ROUTE_TT - 1) / ROUTE_TT;
    if (d.resid_bf16) {
        cudaFuncSetAttribute(k_route<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_route<__nv_bfloat16><<<blocks, 256, smem, s>>>((const __nv_bfloat16*)x, T, d.H, d.E, d.k, d.renorm, d.eps,
                                                         lw.w_norm, lw.w_router, fx, sel, w);
    } else {
        cudaFuncSetAttribute(k_route<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_route<float><<<blocks, 256, smem, s>>>((const float*)x, T, d.H, d.E, d.k, d.renorm, d.eps, lw.w_norm,
                                                 lw.w_router, fx, sel, w);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Q8_K quantisation of rows [R][K]: one 256-segment per CTA
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_quant_q8(const float* __restrict__ x, int K, int8_t* __restrict__ q,
                                                  float* __restrict__ dout, int* __restrict__ bs) {
    __shared__ float redf[32];
    const int nseg = K / QK;
    const int64_t r = blockIdx.x / nseg;       // one CTA per (row, 256-segment), 1-D grid
    const int seg = (int)(blockIdx.x - r * nseg);
    const float v = x[r * K + seg * QK + threadIdx.x];
    const float amax = block_max_f(fabsf(v), redf);
    int qi = 0;
    float dd = 0.f;
    if (amax != 0.f) {
        const float iscale = 127.f / amax;
        qi = min(127, __float2int_rn(iscale * v));
        dd = 1.f / iscale;
    }
    q[r * K + seg * QK + threadIdx.x] = (int8_t)qi;
    int sum = qi;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 15) == 0) bs[r * (K / 16) + seg * 16 + (threadIdx.x >> 4)] = sum;
    if (threadIdx.x == 0) dout[r * nseg + seg] = dd;
}

// ---------------------------------------------------------------------------------------------
// dispatch: counting sort of entry ids e = t*KK + j by pool slot (one CTA)
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_dispatch(const int32_t* __restrict__ slot_of, int T, int k, int KK,
                                                   int n_slots, int* __restrict__ counts, int* __restrict__ offsets,
                                                   int* __restrict__ perm, unsigned* err) {
    extern __shared__ int sm[];
    const int NS = n_slots + (KK > k ? 1 : 0);
    int* cnt = sm;
    int* cur = sm + NS + 1;
    for (int i = threadIdx.x; i <= NS; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const int n = T * KK;
    for (int e = threadIdx.x; e < n; e += blockDim.x) {
        const int t = e / KK, j = e - t * KK;
        int s = (j < k) ? slot_of[(size_t)t * k + j] : n_slots;
        if (s < 0 || s >= NS || (j < k && s >= n_slots)) {
            atomicOr(err, 1u);
            continue;
        }
        atomicAdd(&cnt[s], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int i = 0; i < NS; ++i) {
            cur[i] = acc;
            offsets[i] = acc;
            counts[i] = cnt[i];
            acc += cnt[i];
        }
        offsets[NS] = acc;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += blockDim.x) {
        const int t = e / KK, j = e - t * KK;
        const int s = (j < k) ? slot_of[(size_t)t * k + j] : n_slots;
        if (s < 0 || s >= NS || (j < k && s >= n_slots)) continue;
        perm[atomicAdd(&cur[s], 1)] = e;
    }
}

// ---------------------------------------------------------------------------------------------
// grouped expert matmuls
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float row_dot_rt(int type, const uint8_t* base, int64_t nblk, int64_t row, int nb,
                                            const ActRow& a, int lane) {
    return type == T_Q4K ? row_dot_lane<T_Q4K>(base, nblk, row, nb, a, lane)
                         : row_dot_lane<T_Q6K>(base, nblk, row, nb, a, lane);
}

struct SlotMats {
    const uint8_t *g, *u, *d;
    int gt, ut, dt;
};

__device__ __forceinline__ SlotMats slot_mats(const LayerWeights& lw, int s) {
    SlotMats m;
    if (s < lw.n_slots) {
        const uint8_t* b = lw.pool + (int64_t)s * lw.slot_stride;
        m.g = b; m.u = b + lw.off_up; m.d = b + lw.off_down;
        m.gt = lw.gate_type; m.ut = lw.up_type; m.dt = lw.down_type;
    } else {
        m.g = lw.shared; m.u = lw.shared + lw.sh_off_up; m.d = lw.shared + lw.sh_off_down;
        m.gt = lw.sh_gate_type; m.ut = lw.sh_up_type; m.dt = lw.sh_down_type;
    }
    return m;
}

constexpr int GU_ROWS = 16;    // gate/up rows per CTA (8 warps x 2)
constexpr int DN_ROWS = 16;    // down rows per CTA

__global__ void __launch_bounds__(256) k_gateup(LayerWeights lw, int H, int I, int KK, const int* __restrict__ offsets,
                                                const int* __restrict__ perm, const int8_t* __restrict__ xq,
                                                const float* __restrict__ xd, const int* __restrict__ xbs,
                                                float* __restrict__ h) {
    const int s = blockIdx.x;
    const int start = offsets[s], end = offsets[s + 1];
    if (start == end) return;
    const SlotMats m = slot_mats(lw, s);
    const int nb = H / QK;
    const int64_t nblk = (int64_t)I * nb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r1 = min(I, (int)(blockIdx.y + 1) * GU_ROWS);
    for (int i = blockIdx.y * GU_ROWS + warp; i < r1; i += 8) {
        for (int p = start; p < end; ++p) {
            const int ent = perm[p];
            const int t = ent / KK;
            const ActRow a{xq + (size_t)t * H, xd + (size_t)t * nb, xbs + (size_t)t * (H / 16)};
            float g = row_dot_rt(m.gt, m.g, nblk, i, nb, a, lane);
            float u = row_dot_rt(m.ut, m.u, nblk, i, nb, a, lane);
            g = warp_sum(g);
            u = warp_sum(u);
            if (lane == 0) h[(size_t)ent * I + i] = silu_f(g) * u;
        }
    }
}

__global__ void __launch_bounds__(256) k_down(LayerWeights lw, int H, int I, const int* __restrict__ offsets,
                                              const int* __restrict__ perm, const int8_t* __restrict__ hq,
                                              const float* __restrict__ hd, const int* __restrict__ hbs,
                                              float* __restrict__ y) {
    const int s = blockIdx.x;
    const int start = offsets[s], end = offsets[s + 1];
    if (start == end) return;
    const SlotMats m = slot_mats(lw, s);
    const int nb = I / QK;
    const int64_t nblk = (int64_t)H * nb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r1 = min(H, (int)(blockIdx.y + 1) * DN_ROWS);
    for (int dr = blockIdx.y * DN_ROWS + warp; dr < r1; dr += 8) {
        for (int p = start; p < end; ++p) {
            const int ent = perm[p];
            const ActRow a{hq + (size_t)ent * I, hd + (size_t)ent * nb, hbs + (size_t)ent * (I / 16)};
            const float v = warp_sum(row_dot_rt(m.dt, m.d, nblk, dr, nb, a, lane));
            if (lane == 0) y[(size_t)ent * H + dr] = v;
        }
    }
}

// sigmoid(gate_inp . fx[t]) per token (double accumulation, as the router GEMV)
__global__ void __launch_bounds__(256) k_shared_gate(const float* __restrict__ fx, const float* __restrict__ g, int H,
                                                     float* __restrict__ out) {
    __shared__ double redd[32];
    const int t = blockIdx.x;
    double acc = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) acc += (double)g[i] * (double)fx[(size_t)t * H + i];
    acc = block_sum_d(acc, redd);
    if (threadIdx.x == 0) out[t] = sigmoid_f((float)acc);
}

template <typename R>
__global__ void __launch_bounds__(256) k_combine(const float* __restrict__ y, const float* __restrict__ w,
                                                 const float* __restrict__ sh_gate, int k, int KK, int H, int T,
                                                 R* x) {
    const int64_t n = (int64_t)T * H;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = idx / H;
        const int64_t dcol = idx - t * H;
        float acc = 0.f;
        for (int j = 0; j < k; ++j) acc += w[t * k + j] * y[(t * KK + j) * H + dcol];
        if (KK > k) acc = acc + y[(t * KK + k) * H + dcol] * sh_gate[t];
        x[idx] = from_f32<R>(acc + to_f32<R>(x[idx]));
    }
}

cudaError_t launch_shared_gate(const float* fx, const float* gate_inp, int H, int T, float* out, cudaStream_t s) {
    k_shared_gate<<<T, 256, 0, s>>>(fx, gate_inp, H, out);
    return cudaGetLastError();
}

cudaError_t launch_dispatch(const int32_t* slot_of_sel, int T, int k, int KK, int n_slots, const Scratch& sc,
                            cudaStream_t s) {
    const int NS = n_slots + (KK > k ? 1 : 0);
    const size_t dsm = (size_t)2 * (NS + 1) * sizeof(int);
    k_dispatch<<<1, 1024, dsm, s>>>(slot_of_sel, T, k, KK, n_slots, sc.counts, sc.offsets, sc.perm, sc.sync);
    return cudaGetLastError();
}

cudaError_t launch_combine(const Dims& d, const Scratch& sc, const float* w, void* x_inout, int T, int KK,
                           cudaStream_t s) {
    const int64_t n = (int64_t)T * d.H;
    const int cb = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    if (d.resid_bf16)
        k_combine<__nv_bfloat16><<<cb, 256, 0, s>>>(sc.y, w, sc.sh_gate, d.k, KK, d.H, T, (__nv_bfloat16*)x_inout);
    else
        k_combine<float><<<cb, 256, 0, s>>>(sc.y, w, sc.sh_gate, d.k, KK, d.H, T, (float*)x_inout);
    return cudaGetLastError();
}

cudaError_t launch_experts_grouped(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                                   const int32_t* slot_of_sel, const float* w, void* x_inout, int T,
                                   bool /*need_sh_gate*/, cudaStream_t s, int* launches) {
    const bool shared = lw.shared != nullptr;
    const int KK = d.k + (shared ? 1 : 0);
    const int NS = lw.n_slots + (shared ? 1 : 0);
    int nl = 0;
    cudaError_t e;
    // 1. quantise fx
    k_quant_q8<<<(unsigned)((d.H / QK) * T), 256, 0, s>>>(fx, d.H, sc.fx_q, sc.fx_d, sc.fx_bs);
    ++nl;
    if (shared) {
        if ((e = launch_shared_gate(fx, lw.sh_gate_inp, d.H, T, sc.sh_gate, s)) != cudaSuccess) return e;
        ++nl;
    }
    // 2. group entries by slot
    if ((e = launch_dispatch(slot_of_sel, T, d.k, KK, lw.n_slots, sc, s)) != cudaSuccess) return e;
    ++nl;
    // 3. gate/up + SwiGLU
    k_gateup<<<dim3(NS, (d.I + GU_ROWS - 1) / GU_ROWS), 256, 0, s>>>(lw, d.H, d.I, KK, sc.offsets, sc.perm, sc.fx_q,
                                                                      sc.fx_d, sc.fx_bs, sc.h);
    ++nl;
    // 4. quantise h
    k_quant_q8<<<(unsigned)((d.I / QK) * T * KK), 256, 0, s>>>(sc.h, d.I, sc.h_q, sc.h_d, sc.h_bs);
    ++nl;
    // 5. down
    k_down<<<dim3(NS, (d.H + DN_ROWS - 1) / DN_ROWS), 256, 0, s>>>(lw, d.H, d.I, sc.offsets, sc.perm, sc.h_q, sc.h_d,
                                                                    sc.h_bs, sc.y);
    ++nl;
    // 6. weighted combine into the residual
    if ((e = launch_combine(d, sc, w, x_inout, T, KK, s)) != cudaSuccess) return e;
    ++nl;
    if (launches) *launches += nl;
    return cudaGetLastError();
}

}  // namespace hoard
