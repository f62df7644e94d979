// kernels_grouped.cu -- the router and the token-grouped expert path, valid for any T.
//
// One MoE layer for T tokens runs as:
//   k_rmsnorm, k_router_logits (k_router_tc for T >= 1024), k_route_topk
//                   RMSNorm -> f32 router GEMV -> softmax over all E -> top-k (+renorm), per token
//   k_quant_q8      Q8_K quantisation of the normed activations fx
//   k_dispatch      group the (token, j) pairs by pool slot (counting sort, one CTA; k_disp_* above
//                   4096 entries)
//   k_gateup_sw     per slot and row tile: h = silu(gate . fx) * (up . fx) for the slot's tokens
//   k_quant_q8      Q8_K quantisation of h
//   k_down_sw       per slot and row tile: y = down . h for the slot's tokens
//   k_combine       x = (sum_j w_j * y_j + sigmoid(g_sh . fx) * y_sh) + x, j ascending
// (for T <= 64 with every expert resident, k_route_fused replaces the first five kernels; the
// per-entry kernels k_gateup / k_down serve the shapes the streaming kernels do not), which restates
// graph A's router tail and graph B of hoard (src/run_moe_stream.cpp:352-373, :425-447) and the
// batched mul_mat_id form (src/run_specloop.cpp:115-140). Every kernel here is a programmatic
// dependent launch.
#include "common.cuh"
#include "kernels.h"
#include "block_ops.cuh"
#include "async_copy.cuh"
#include <algorithm>
#include <type_traits>

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

// The same re-lay with wide source reads, for a batch of matrices in one launch: tiles of RP_TB
// blocks (RP_TB * bytes per block is a multiple of 16) are read with 16-byte loads, all of a thread's
// loads issued before any is used, into shared memory and scattered into the planes from there. Used
// whenever every source is 16-byte aligned; it matters most when the source is pinned host memory
// read over PCIe, where the bus is only kept busy by many wide reads in flight.
constexpr int RP_TB = 64;
constexpr int RP_THREADS = 256;

__device__ __forceinline__ void repack_tile(int type, const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                            int64_t nblk, int64_t b0, uint8_t* sb) {
    const int bb = block_bytes(type);
    const int nb = (int)(nblk - b0 < RP_TB ? nblk - b0 : RP_TB);
    const int bytes = nb * bb, n16 = bytes / 16;
    const uint8_t* st = src + b0 * bb;
    uint4 v[(RP_TB * 210 / 16 + RP_THREADS - 1) / RP_THREADS];
#pragma unroll
    for (int u = 0; u < (int)(sizeof(v) / sizeof(v[0])); ++u) {
        const int i = threadIdx.x + u * RP_THREADS;
        if (i < n16) v[u] = reinterpret_cast<const uint4*>(st)[i];
    }
#pragma unroll
    for (int u = 0; u < (int)(sizeof(v) / sizeof(v[0])); ++u) {
        const int i = threadIdx.x + u * RP_THREADS;
        if (i < n16) reinterpret_cast<uint4*>(sb)[i] = v[u];
    }
    for (int i = n16 * 16 + threadIdx.x; i < bytes; i += RP_THREADS) sb[i] = st[i];
    __syncthreads();
    for (int i = threadIdx.x; i < bytes; i += RP_THREADS) {
        const int bl = i / bb, o = i - bl * bb;
        const int64_t b = b0 + bl;
        int64_t off;
        if (type == T_Q4K) {
            off = (o < 16) ? nblk * 128 + b * 16 + o : b * 128 + (o - 16);
        } else {
            if (o < 128) off = b * 128 + o;
            else if (o < 192) off = nblk * 128 + b * 64 + (o - 128);
            else if (o < 208) off = nblk * 192 + b * 16 + (o - 192);
            else off = nblk * 208 + b * 2 + (o - 208);
        }
        dst[off] = sb[i];
    }
    __syncthreads();
}

struct RepackBatch {
    const uint8_t* src[REPACK_MAX_JOBS];
    uint8_t* dst[REPACK_MAX_JOBS];
    int64_t nblk[REPACK_MAX_JOBS];
    int type[REPACK_MAX_JOBS];
    int64_t tile0[REPACK_MAX_JOBS + 1];   // first tile of each job; tile0[n] = all tiles
    int n;
};

__global__ void __launch_bounds__(RP_THREADS) k_repack_tiled(const RepackBatch bt) {
    __shared__ __align__(16) uint8_t sb[RP_TB * 210];
    int j = 0;
    for (int64_t t = blockIdx.x; t < bt.tile0[bt.n]; t += gridDim.x) {
        while (t >= bt.tile0[j + 1]) ++j;            // tiles are visited in increasing order
        repack_tile(bt.type[j], bt.src[j], bt.dst[j], bt.nblk[j], (t - bt.tile0[j]) * RP_TB, sb);
    }
}

cudaError_t launch_repack_batch(const RepackJob* jobs, int n, cudaStream_t s) {
    if (n < 0 || n > REPACK_MAX_JOBS) return cudaErrorInvalidValue;
    RepackBatch bt{};
    bt.n = n;
    for (int i = 0; i < n; ++i) {
        if (jobs[i].type != T_Q4K && jobs[i].type != T_Q6K) return cudaErrorInvalidValue;
        if ((reinterpret_cast<uintptr_t>(jobs[i].src) & 15) != 0 || jobs[i].nblk < 0) return cudaErrorInvalidValue;
        bt.src[i] = jobs[i].src;
        bt.dst[i] = jobs[i].dst;
        bt.nblk[i] = jobs[i].nblk;
        bt.type[i] = jobs[i].type;
        bt.tile0[i + 1] = bt.tile0[i] + (jobs[i].nblk + RP_TB - 1) / RP_TB;
    }
    const int64_t tiles = bt.tile0[n];
    if (tiles == 0) return cudaSuccess;
    k_repack_tiled<<<(unsigned)(tiles < 148 * 6 ? tiles : 148 * 6), RP_THREADS, 0, s>>>(bt);
    return cudaGetLastError();
}

cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int64_t nblk, cudaStream_t s) {
    if (type != T_Q4K && type != T_Q6K) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const RepackJob j{type, src, dst, nblk};
        return launch_repack_batch(&j, 1, s);
    }
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
// router (graph A's tail, src/run_moe_stream.cpp:352-373): three kernels
//   k_rmsnorm        fx = (x * 1/sqrt(mean(x^2) + eps)) * ffn_norm, one CTA per token
//   k_router_logits  logits = W_r . fx as a tiled GEMM (32 tokens x 128 experts per CTA, K staged
//                    in shared memory, split over K when there are few tiles); f32 products summed
//                    over 32-wide K chunks, chunks summed in double; partial sums per K split
//   k_route_topk     one warp per token: sum the K splits in order, softmax over all E, top-k by
//                    (probability desc, id asc), optional renorm with the 6.103515625e-5 clamp
// ---------------------------------------------------------------------------------------------
constexpr int MAX_K = 16;
constexpr int RL_TT = 32;      // tokens per tile: 8 warps x 4
constexpr int RL_EB = 128;     // experts per tile: 32 lanes x 4
constexpr int RL_KC = 32;      // K chunk staged in shared memory
constexpr int RL_MIN_KLEN = 32;      // one K chunk per split at small T (the K splits are summed 8 loads at a time)
constexpr int RL_TARGET_CTAS = 296;

constexpr int RMS_MAXV = 32;   // H <= 8192: values per thread held in registers

// VPT values per thread (a multiple of 4, loaded 4 at a time; H a multiple of 4)
template <typename R> struct Vec4;
template <> struct Vec4<float> {
    static __device__ __forceinline__ void load(const float* p, float* v) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    }
};
template <> struct Vec4<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
        const uint2 a = *reinterpret_cast<const uint2*>(p);
        v[0] = __uint_as_float(a.x << 16); v[1] = __uint_as_float(a.x & 0xFFFF0000u);
        v[2] = __uint_as_float(a.y << 16); v[3] = __uint_as_float(a.y & 0xFFFF0000u);
    }
};

// RMS scale of one row by a 256-thread CTA: thread t holds values 4*(t + 256*j) + 0..3, j < VPT/4, in v
// (zeros past H); the squares are summed per thread in j order and over the CTA by block_sum_d.
template <typename R, int VPT>
__device__ __forceinline__ float rms_row_scale(const R* __restrict__ xr, int H, float eps, float* v, double* redd) {
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
        const int i = 4 * (threadIdx.x + 256 * j);
        if (i < H) Vec4<R>::load(xr + i, v + 4 * j);
        else v[4 * j] = v[4 * j + 1] = v[4 * j + 2] = v[4 * j + 3] = 0.f;
    }
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) ss += (double)(v[j] * v[j]);
    ss = block_sum_d(ss, redd);
    const float mean = (float)(ss / H);
    return 1.0f / sqrtf(mean + eps);
}

template <typename R, int VPT>
__global__ void __launch_bounds__(256) k_rmsnorm(const R* __restrict__ x, int H, float eps,
                                                 const float* __restrict__ w_norm, float* __restrict__ fx) {
    pdl_enter();
    __shared__ double redd[32];
    const int64_t t = blockIdx.x;
    float v[VPT];
    const float scale = rms_row_scale<R, VPT>(x + t * H, H, eps, v, redd);
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
        const int i = 4 * (threadIdx.x + 256 * j);
        if (i < H) {
            const float4 w = *reinterpret_cast<const float4*>(w_norm + i);
            *reinterpret_cast<float4*>(fx + t * H + i) =
                make_float4((v[4 * j] * scale) * w.x, (v[4 * j + 1] * scale) * w.y, (v[4 * j + 2] * scale) * w.z,
                            (v[4 * j + 3] * scale) * w.w);
        }
    }
}

template <typename R>
cudaError_t launch_rmsnorm_rows(const R* x, int rows, int H, float eps, const float* w, float* out, cudaStream_t s) {
    if (rows <= 0 || H <= 0 || H % 4 || H > 256 * RMS_MAXV) return cudaErrorInvalidValue;
    if (H <= 1024) launch_pdl(k_rmsnorm<R, 4>, rows, 256, 0, s, x, H, eps, w, out);
    else if (H <= 2048) launch_pdl(k_rmsnorm<R, 8>, rows, 256, 0, s, x, H, eps, w, out);
    else if (H <= 4096) launch_pdl(k_rmsnorm<R, 16>, rows, 256, 0, s, x, H, eps, w, out);
    else launch_pdl(k_rmsnorm<R, 32>, rows, 256, 0, s, x, H, eps, w, out);
    return cudaGetLastError();
}

// grid (ceil(T/32), ceil(E/128), ksplit); CTA z covers K range [z*klen, (z+1)*klen)
__global__ void __launch_bounds__(256) k_router_logits(const float* __restrict__ fx, const float* __restrict__ w_router,
                                                       int T, int H, int E, int klen, double* __restrict__ part) {
    pdl_enter();
    __shared__ __align__(16) float sf[RL_KC][RL_TT];          // fx chunk, k-major
    __shared__ __align__(16) float sw[RL_KC][RL_EB + 4];      // router chunk, k-major (padded rows)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * RL_TT, e0 = blockIdx.y * RL_EB;
    const int k0 = blockIdx.z * klen;
    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
    // global -> registers for chunk kb (fx: one float4 per thread, router: four)
    const int st = tid >> 3, skq = (tid & 7) * 4;
    float4 pf, pw[4];
    auto fetch = [&](int kb) {
        pf = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + st < T) pf = *reinterpret_cast<const float4*>(fx + (int64_t)(t0 + st) * H + kb + skq);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int e = (tid + 256 * r) >> 3;
            pw[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 + e < E) pw[r] = __ldg(reinterpret_cast<const float4*>(w_router + (int64_t)(e0 + e) * H + kb + skq));
        }
    };
    fetch(k0);
    for (int kb = k0; kb < k0 + klen; kb += RL_KC) {
        sf[skq][st] = pf.x; sf[skq + 1][st] = pf.y; sf[skq + 2][st] = pf.z; sf[skq + 3][st] = pf.w;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int e = (tid + 256 * r) >> 3;
            sw[skq][e] = pw[r].x; sw[skq + 1][e] = pw[r].y; sw[skq + 2][e] = pw[r].z; sw[skq + 3][e] = pw[r].w;
        }
        __syncthreads();
        if (kb + RL_KC < k0 + klen) fetch(kb + RL_KC);     // next chunk in flight during this one
        float a[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) a[i][j] = 0.f;
#pragma unroll 8
        for (int kk = 0; kk < RL_KC; ++kk) {
            const float4 f = *reinterpret_cast<const float4*>(&sf[kk][warp * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&sw[kk][lane * 4]);
            const float fv[4] = {f.x, f.y, f.z, f.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) a[i][j] = fmaf(fv[i], wv[j], a[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] += (double)a[i][j];
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + warp * 4 + i;
        if (t >= T) continue;
        double* dst = part + ((int64_t)blockIdx.z * T + t) * E;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = e0 + lane * 4 + j;
            if (e < E) dst[e] = acc[i][j];
        }
    }
}

// Softmax over the E logits of one token (max subtracted, double sum), then k rounds of arg-max over
// (probability desc, id asc) and the optional renormalisation (sequential f32 sum in rank order, clamped
// at 6.103515625e-5); one warp, E <= 32 * NV. Lanes < k write rank `lane` to sel_t / w_t.
template <int NV>
__device__ __forceinline__ void route_topk_row(const float* lgrow, int E, int k, int renorm, int lane,
                                               int32_t* __restrict__ sel_t, float* __restrict__ w_t) {
    float p[NV];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int e = lane + 32 * i;
        p[i] = e < E ? lgrow[e] : -INFINITY;
        m = fmaxf(m, p[i]);
    }
    m = warp_max(m);
    double ssum = 0.0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        if (lane + 32 * i < E) {
            p[i] = expf(p[i] - m);
            ssum += (double)p[i];
        }
    }
    ssum = warp_sum(ssum);
    const float inv = (float)(1.0 / ssum);
#pragma unroll
    for (int i = 0; i < NV; ++i) p[i] = lane + 32 * i < E ? p[i] * inv : -1.f;
    // k rounds of arg-max over (p desc, id asc): each lane's best value (lowest id among equal p), then
    // the warp's largest key (an order-preserving unsigned image of p) and, among lanes holding it, the
    // lowest id (two redux instructions); the winner's entry is retired with p = -1
    float my_w = 0.f, wsum = 0.f;
    int my_e = 0;
    for (int r = 0; r < k; ++r) {
        float bp = -1.f;
        int be = 0x7FFFFFFF;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int e = lane + 32 * i;
            if (p[i] > bp || (p[i] == bp && e < be)) { bp = p[i]; be = e; }
        }
        const unsigned u = __float_as_uint(bp);
        const unsigned key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        const unsigned M = __reduce_max_sync(0xFFFFFFFFu, key);
        const int W = (int)__reduce_min_sync(0xFFFFFFFFu, key == M ? (unsigned)be : 0xFFFFFFFFu);
        const float wp = __uint_as_float((M & 0x80000000u) ? (M & 0x7FFFFFFFu) : ~M);
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (lane + 32 * i == W) p[i] = -1.f;
        wsum += wp;                                   // sequential f32 sum in rank order
        if (lane == r) { my_w = wp; my_e = W; }
    }
    if (renorm) {
        if (wsum < 6.103515625e-5f) wsum = 6.103515625e-5f;
        my_w /= wsum;
    }
    if (lane < k) {
        sel_t[lane] = my_e;
        w_t[lane] = my_w;
    }
}

// TT tokens per CTA (1 at small T, so that the split sums of a batch of a few tokens are spread over
// many CTAs, with TOPK_SMALL_THREADS threads; 8 at large T, 256 threads): the CTA's threads sum the K
// splits into shared memory, then one warp per token does softmax + top-k (E <= 1024). Where the
// CTA's (token, expert) elements number at most half its threads, SUBS = threads / elements threads
// share an element: each sums a contiguous range of the splits (eight independent loads in flight,
// added in split order) and the range sums are added in range order, so the result depends only on
// (ksplit, T, E).
constexpr int TOPK_TT = 8;
constexpr int TOPK_SMALL_T = 1024;   // at most this many tokens: one token per CTA
constexpr int TOPK_SMALL_THREADS = 512;

template <int NV>
__global__ void __launch_bounds__(TOPK_SMALL_THREADS) k_route_topk(const double* __restrict__ part, int ksplit, int T,
                                                                   int E, int k, int renorm, int32_t* __restrict__ sel,
                                                                   float* __restrict__ w) {
    pdl_enter();
    __shared__ float lg[TOPK_TT][32 * NV];
    __shared__ double rs[TOPK_SMALL_THREADS];
    const int tpc = T <= TOPK_SMALL_T ? 1 : TOPK_TT;
    const int t0 = blockIdx.x * tpc;
    const int nt = min(tpc, T - t0);
    const int nel = nt * E;
    int subs = 1;
    while (subs < 16 && subs * 2 * nel <= (int)blockDim.x && subs * 2 <= ksplit) subs *= 2;
    const int64_t zs = (int64_t)T * E;
    for (int i = threadIdx.x; i < subs * nel; i += blockDim.x) {
        const int el = i % nel, sub = i / nel;
        const int tt = el / E, e = el - tt * E;
        const int z0 = (int)((int64_t)ksplit * sub / subs), z1 = (int)((int64_t)ksplit * (sub + 1) / subs);
        const double* src = part + (int64_t)(t0 + tt) * E + e;
        double s = 0.0;
        int z = z0;
        for (; z + 8 <= z1; z += 8) {
            double v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = src[(int64_t)(z + u) * zs];
#pragma unroll
            for (int u = 0; u < 8; ++u) s += v[u];
        }
        for (; z < z1; ++z) s += src[(int64_t)z * zs];
        if (subs == 1) lg[tt][e] = (float)s;
        else rs[i] = s;
    }
    if (subs > 1) {
        __syncthreads();
        for (int el = threadIdx.x; el < nel; el += blockDim.x) {
            double s = rs[el];
            for (int sub = 1; sub < subs; ++sub) s += rs[sub * nel + el];
            const int tt = el / E;
            lg[tt][el - tt * E] = (float)s;
        }
    }
    __syncthreads();
    const int tt = threadIdx.x >> 5;
    if (tt >= nt) return;
    const int t = t0 + tt;
    route_topk_row<NV>(lg[tt], E, k, renorm, threadIdx.x & 31, sel + (int64_t)t * k, w + (int64_t)t * k);
}

// Large batches (T >= RB_MIN_T): the logits come from the tensor-core router GEMM (launch_router_tc,
// kernels_prefill.cu) in RB_KC-aligned K splits, one 128-token x 128-expert tile per CTA.
constexpr int RB_TT = 128, RB_KC = 32;
constexpr int RB_MIN_T = 1024;         // T at or above which the tensor-core router runs
constexpr int RB_TARGET_CTAS = 148;    // K splits sized for about one CTA per SM

int router_ksplit_big(int T, int E, int H) {
    const int tiles = ((T + RB_TT - 1) / RB_TT) * ((E + 127) / 128);
    int ks = RB_TARGET_CTAS / tiles;
    const int max_ks = H / (4 * RB_KC);                  // at least 4 chunks per split
    if (ks > max_ks) ks = max_ks;
    while (ks > 1 && (H % (ks * RB_KC) != 0)) --ks;
    return ks < 1 ? 1 : ks;
}

int router_ksplit(int T, int E, int H) {
    const int tiles = ((T + RL_TT - 1) / RL_TT) * ((E + RL_EB - 1) / RL_EB);
    int ks = RL_TARGET_CTAS / tiles;
    const int max_ks = H / RL_MIN_KLEN;
    if (ks > max_ks) ks = max_ks;
    while (ks > 1 && (H % (ks * RL_KC) != 0)) --ks;    // equal K ranges, whole chunks
    return ks < 1 ? 1 : ks;
}

int64_t router_partial_elems(int max_tokens, int E) {
    // ksplit * T <= (RL_TARGET_CTAS / tiles) * tile_tokens * tiles for either kernel, and T when ks = 1
    const int64_t tile = RB_TT > RL_TT ? RB_TT : RL_TT;
    const int64_t rows = max_tokens > RL_TARGET_CTAS * tile ? max_tokens : RL_TARGET_CTAS * tile;
    return rows * E;
}

cudaError_t launch_route(const Dims& d, const LayerWeights& lw, const void* x, int T, float* fx, int32_t* sel,
                         float* w, double* part, cudaStream_t s, int* launches, unsigned* err) {
    cudaError_t e0 = d.resid_bf16
        ? launch_rmsnorm_rows((const __nv_bfloat16*)x, T, d.H, d.eps, lw.w_norm, fx, s)
        : launch_rmsnorm_rows((const float*)x, T, d.H, d.eps, lw.w_norm, fx, s);
    if (e0 != cudaSuccess) return e0;
    int ks;
    if (T >= RB_MIN_T && d.H % RB_KC == 0) {
        ks = router_ksplit_big(T, d.E, d.H);
        cudaError_t e = launch_router_tc(fx, lw.w_router, T, d.H, d.E, ks, part, err, s);
        if (e != cudaSuccess) return e;
    } else {
        ks = router_ksplit(T, d.E, d.H);
        const dim3 grid((T + RL_TT - 1) / RL_TT, (d.E + RL_EB - 1) / RL_EB, ks);
        launch_pdl(k_router_logits, grid, 256, 0, s, fx, lw.w_router, T, d.H, d.E, d.H / ks, part);
    }
    const int tpc = T <= TOPK_SMALL_T ? 1 : TOPK_TT;
    const unsigned tgrid = (unsigned)((T + tpc - 1) / tpc);
    const int tth = tpc == 1 ? TOPK_SMALL_THREADS : 256;
    if (d.E <= 64) launch_pdl(k_route_topk<2>, tgrid, tth, 0, s, part, ks, T, d.E, d.k, d.renorm, sel, w);
    else if (d.E <= 128) launch_pdl(k_route_topk<4>, tgrid, tth, 0, s, part, ks, T, d.E, d.k, d.renorm, sel, w);
    else if (d.E <= 256) launch_pdl(k_route_topk<8>, tgrid, tth, 0, s, part, ks, T, d.E, d.k, d.renorm, sel, w);
    else if (d.E <= 512) launch_pdl(k_route_topk<16>, tgrid, tth, 0, s, part, ks, T, d.E, d.k, d.renorm, sel, w);
    else launch_pdl(k_route_topk<32>, tgrid, tth, 0, s, part, ks, T, d.E, d.k, d.renorm, sel, w);
    if (launches) *launches += 3;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Q8_K quantisation of rows [R][K]: one 256-segment per CTA
// ---------------------------------------------------------------------------------------------
// Q8_K of one 256-value segment by a 256-thread CTA, thread i holding value i: scale = max|v| / 127,
// q = min(127, round(v * 127 / max|v|)), 16-value sums of q; q, d and bs point at the segment's outputs.
__device__ __forceinline__ void quant_seg256(float v, float* redf, int8_t* __restrict__ q, float* __restrict__ d,
                                             int* __restrict__ bs) {
    const float amax = block_max_f(fabsf(v), redf);
    int qi = 0;
    float dd = 0.f;
    if (amax != 0.f) {
        const float iscale = 127.f / amax;
        qi = min(127, __float2int_rn(iscale * v));
        dd = 1.f / iscale;
    }
    q[threadIdx.x] = (int8_t)qi;
    int sum = qi;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 15) == 0) bs[threadIdx.x >> 4] = sum;
    if (threadIdx.x == 0) *d = dd;
}

__global__ void __launch_bounds__(256) k_quant_q8(const float* __restrict__ x, int K, int8_t* __restrict__ q,
                                                  float* __restrict__ dout, int* __restrict__ bs) {
    pdl_enter();
    __shared__ float redf[32];
    const int nseg = K / QK;
    const int64_t r = blockIdx.x / nseg;       // one CTA per (row, 256-segment), 1-D grid
    const int seg = (int)(blockIdx.x - r * nseg);
    quant_seg256(x[r * K + seg * QK + threadIdx.x], redf, q + r * K + seg * QK, dout + r * nseg + seg,
                 bs + r * (K / 16) + seg * 16);
}

// ---------------------------------------------------------------------------------------------
// dispatch: counting sort of entry ids e = t*KK + j by pool slot (one CTA of 1024 threads), and
// optionally the tensor-core work list: one (slot, M tile) item per `tile_m` entries of a slot.
// Entries are read 8 per thread at a time so their loads overlap; the offsets come from a
// CTA-wide scan. The order of entries within a slot is arbitrary (every consumer is per entry).
// ---------------------------------------------------------------------------------------------
constexpr int DISP_THREADS = 1024;
constexpr int DISP_UNROLL = 8;

// exclusive scan of one int2 per thread over a CTA of NT threads (NT / 32 <= 32 warps)
template <int NT>
__device__ __forceinline__ int2 scan_excl_cta(int2 v, int2* wtot, int2& total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int2 inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xFFFFFFFFu, inc.x, o), b = __shfl_up_sync(0xFFFFFFFFu, inc.y, o);
        if (lane >= o) { inc.x += a; inc.y += b; }
    }
    if (lane == 31) wtot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int2 t = lane < NW ? wtot[lane] : make_int2(0, 0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xFFFFFFFFu, t.x, o), b = __shfl_up_sync(0xFFFFFFFFu, t.y, o);
            if (lane >= o) { t.x += a; t.y += b; }
        }
        if (lane < NW) wtot[lane] = t;
    }
    __syncthreads();
    const int2 pre = warp > 0 ? wtot[warp - 1] : make_int2(0, 0);
    total = wtot[NW - 1];
    return make_int2(pre.x + inc.x - v.x, pre.y + inc.y - v.y);
}

// The counting sort of one CTA of NT threads: entries e = t*KK + j (slot slot_of[t*k + j] for j < k,
// the shared slot n_slots for j = k) -> counts, offsets, perm and, with tile_m > 0, the work list
// items (one (slot, M tile) per tile_m entries of a slot). sm holds 2 * (NS + 1) ints. slot_of is
// read through L2 (it may have been written earlier in the same launch by another CTA).
template <int NT>
__device__ __forceinline__ void dispatch_cta(const int32_t* slot_of, int T, int k, int KK, int n_slots,
                                             int* __restrict__ counts, int* __restrict__ offsets,
                                             int* __restrict__ perm, unsigned* err, int tile_m,
                                             int2* __restrict__ items, int* __restrict__ n_items, bool skip_neg,
                                             int* sm, int2* wtot) {
    const int NS = n_slots + (KK > k ? 1 : 0);
    int* cnt = sm;
    int* cur = sm + NS + 1;
    for (int i = threadIdx.x; i <= NS; i += NT) cnt[i] = 0;
    __syncthreads();
    const int n = T * KK;
    auto slot_at = [&](int e) {
        const int t = e / KK, j = e - t * KK;
        return (j < k) ? (int)__ldcg(slot_of + (size_t)t * k + j) : n_slots;
    };
    auto valid = [&](int e, int sl) {
        const int j = e % KK;
        return !(sl < 0 || sl >= NS || (j < k && sl >= n_slots));
    };
    for (int e0 = threadIdx.x; e0 < n; e0 += NT * DISP_UNROLL) {
        int sv[DISP_UNROLL];
#pragma unroll
        for (int u = 0; u < DISP_UNROLL; ++u) {
            const int e = e0 + u * NT;
            sv[u] = e < n ? slot_at(e) : -1;
        }
#pragma unroll
        for (int u = 0; u < DISP_UNROLL; ++u) {
            const int e = e0 + u * NT;
            if (e >= n) continue;
            if (!valid(e, sv[u])) {
                if (!(skip_neg && sv[u] < 0)) atomicOr(err, 1u);
                continue;
            }
            atomicAdd(&cnt[sv[u]], 1);
        }
    }
    __syncthreads();
    // exclusive scan of (entries, M tiles) over the slots; thread i owns slots [i*c, (i+1)*c)
    const int c = (NS + NT - 1) / NT;
    const int s0 = threadIdx.x * c, s1 = min(NS, s0 + c);
    int2 mine = make_int2(0, 0);
    for (int sl = s0; sl < s1; ++sl) {
        mine.x += cnt[sl];
        if (tile_m > 0) mine.y += (cnt[sl] + tile_m - 1) / tile_m;
    }
    int2 total;
    int2 off = scan_excl_cta<NT>(mine, wtot, total);
    for (int sl = s0; sl < s1; ++sl) {
        const int cn = cnt[sl];
        offsets[sl] = off.x;
        counts[sl] = cn;
        cur[sl] = off.x;
        off.x += cn;
        if (tile_m > 0) {
            for (int mt = 0; mt * tile_m < cn; ++mt) items[off.y + mt] = make_int2(sl, mt);
            off.y += (cn + tile_m - 1) / tile_m;
        }
    }
    if (threadIdx.x == 0) {
        offsets[NS] = total.x;
        if (tile_m > 0) *n_items = total.y;
    }
    __syncthreads();
    for (int e0 = threadIdx.x; e0 < n; e0 += NT * DISP_UNROLL) {
        int sv[DISP_UNROLL];
#pragma unroll
        for (int u = 0; u < DISP_UNROLL; ++u) {
            const int e = e0 + u * NT;
            sv[u] = e < n ? slot_at(e) : -1;
        }
#pragma unroll
        for (int u = 0; u < DISP_UNROLL; ++u) {
            const int e = e0 + u * NT;
            if (e >= n || !valid(e, sv[u])) continue;
            perm[atomicAdd(&cur[sv[u]], 1)] = e;
        }
    }
}

// The counting sort of a small batch (n = T*KK entries) by one CTA of NT threads in one pass over
// slot_of: each entry's slot and its rank within the slot (a shared-memory atomic) are kept in shared
// memory, the scan gives the slots' offsets, and perm[offset + rank] = e. sm holds NS + 1 + 2n ints.
template <int NT>
__device__ __forceinline__ void dispatch_small(const int32_t* slot_of, int T, int k, int KK, int n_slots,
                                               int* __restrict__ counts, int* __restrict__ offsets,
                                               int* __restrict__ perm, unsigned* err, int tile_m,
                                               int2* __restrict__ items, int* __restrict__ n_items, int* sm,
                                               int2* wtot) {
    const int NS = n_slots + (KK > k ? 1 : 0);
    const int n = T * KK;
    int* cnt = sm;
    int* es = sm + NS + 1;
    int* er = es + n;
    for (int i = threadIdx.x; i <= NS; i += NT) cnt[i] = 0;
#pragma unroll 4
    for (int e = threadIdx.x; e < n; e += NT) {
        const int t = e / KK, j = e - t * KK;
        es[e] = (j < k) ? (int)__ldcg(slot_of + (size_t)t * k + j) : n_slots;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += NT) {
        const int sl = es[e], j = e % KK;
        if (sl < 0 || sl >= NS || (j < k && sl >= n_slots)) {
            atomicOr(err, 1u);
            es[e] = -1;
        } else {
            er[e] = atomicAdd(&cnt[sl], 1);
        }
    }
    __syncthreads();
    const int c = (NS + NT - 1) / NT;
    const int s0 = threadIdx.x * c, s1 = min(NS, s0 + c);
    int2 mine = make_int2(0, 0);
    for (int sl = s0; sl < s1; ++sl) {
        mine.x += cnt[sl];
        if (tile_m > 0) mine.y += (cnt[sl] + tile_m - 1) / tile_m;
    }
    int2 total;
    int2 off = scan_excl_cta<NT>(mine, wtot, total);
    for (int sl = s0; sl < s1; ++sl) {
        const int cn = cnt[sl];
        offsets[sl] = off.x;
        counts[sl] = cn;
        cnt[sl] = off.x;
        off.x += cn;
        if (tile_m > 0) {
            for (int mt = 0; mt * tile_m < cn; ++mt) items[off.y + mt] = make_int2(sl, mt);
            off.y += (cn + tile_m - 1) / tile_m;
        }
    }
    if (threadIdx.x == 0) {
        offsets[NS] = total.x;
        if (tile_m > 0) *n_items = total.y;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += NT)
        if (es[e] >= 0) perm[cnt[es[e]] + er[e]] = e;
}

__global__ void __launch_bounds__(DISP_THREADS) k_dispatch(const int32_t* __restrict__ slot_of, int T, int k, int KK,
                                                           int n_slots, int* __restrict__ counts,
                                                           int* __restrict__ offsets, int* __restrict__ perm,
                                                           unsigned* err, int tile_m, int2* __restrict__ items,
                                                           int* __restrict__ n_items, bool skip_neg) {
    pdl_enter();
    extern __shared__ int sm[];
    __shared__ int2 wtot[32];
    dispatch_cta<DISP_THREADS>(slot_of, T, k, KK, n_slots, counts, offsets, perm, err, tile_m, items, n_items,
                               skip_neg, sm, wtot);
}

// ---------------------------------------------------------------------------------------------
// Small batches through a whole layer: one kernel for graph A's RMSNorm, router GEMV, softmax + top-k,
// the Q8_K of the FFN input and the dispatch, for T <= RF_MAX_T tokens with every expert resident.
// CTA (ec, tg) takes tpg (<= RF_TPG) tokens from tpg*tg and experts [RF_EC*ec, +RF_EC) (one per warp):
//   1. the experts' router rows are copied into shared memory one K half at a time (the first before
//      the wait on the previous kernel: constant weights), the tokens' fx = rms_norm(x) * ffn_norm
//      into shared memory (the arithmetic of k_rmsnorm, so fx is bit-identical; the ec = 0 CTA also
//      stores it);
//   2. logits: each lane forms the f32 sums of its 32-wide K chunks, then the chunk sums are added
//      in double exactly as k_router_logits (per K split) and k_route_topk (splits in `subs`
//      ranges) add them for the same (T, E, H), so the logits -- and the routing -- are identical
//      to the three-kernel path;
//   3. 256-value segments ec, ec + n_ec, ... of each token's fx are quantised to Q8_K (k_quant_q8's
//      arithmetic);
//   4. the CTA counts itself in its token group's counter (release: CTA barrier + fence + atomic);
//      the group's last CTA runs the top-k of the group's tokens and counts the group in; the last
//      group's CTA runs the dispatch (counting sort by slot + the work list). Last arrivers reset the
//      counters, which are zero between launches. No CTA waits for another.
// ---------------------------------------------------------------------------------------------
constexpr int RF_THREADS = 256;
constexpr int RF_TPG = 4;              // most tokens per CTA
constexpr int RF_EC = RF_THREADS / 32; // experts per CTA
constexpr int RF_MAX_T = 64;
constexpr int RF_MAX_E = 512;
constexpr int RF_MAX_CH = 64;          // 32-wide K chunks per row (H <= 2048)
constexpr int RF_CPAD = 36;            // floats per staged K chunk (padding spreads the lanes' reads over the banks)
constexpr int RF_SMEM_MAX = 96 * 1024;  // dynamic shared memory limit of the kernel (two CTAs per SM)
constexpr int RF_CNT_OFF = 2560;       // the counters' place in the scratch sync words
constexpr int RF_CNT_STRIDE = 32;      // one 128-byte line per counter

struct RouteFusedArgs {
    const void* x;
    int T, H, E, k, KK, renorm, n_slots, tile_m;
    float eps;
    int ks, subs;                      // K splits and their summation ranges (k_route_topk's for this T)
    int tpg;                           // tokens per CTA (<= RF_TPG)
    const float* w_norm;
    const float* w_router;             // [E][H]
    float* fx;
    int8_t* fx_q;
    float* fx_d;
    int* fx_bs;
    float* logits;                     // [T][E] scratch
    int32_t* sel;
    float* w;
    int* counts;
    int* offsets;
    int* perm;
    int2* items;
    int* n_items;
    unsigned* err;
    unsigned* cnt;                     // [n_tg + 1] counters at stride RF_CNT_STRIDE (zero at rest)
    unsigned long long* stamp;         // optional {first start, last end} (%globaltimer) of this launch
};

template <typename R, int VPT, int NV>
__global__ void __launch_bounds__(RF_THREADS) k_route_fused(const RouteFusedArgs a) {
    // dynamic: fx [RF_TPG][chunks * RF_CPAD] | router rows, one K half [RF_EC][32 chunks][RF_CPAD];
    // later the logits and the dispatch
    extern __shared__ __align__(16) float rf_sm[];
    __shared__ float cs[RF_EC][RF_TPG][RF_MAX_CH];
    __shared__ double ps[RF_EC][RF_MAX_CH];
    __shared__ double redd[32];
    __shared__ float redf[32];
    __shared__ int2 wtot[32];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ec = blockIdx.x, tg = blockIdx.y, n_ec = gridDim.x, n_tg = gridDim.y;
    const int tpg = a.tpg;
    const int H = a.H, E = a.E;
    const int nch = H / 32, cpl = nch / 32;            // chunks per row, per lane (1 or 2)
    const int t0 = tg * tpg, nt = min(tpg, a.T - t0);
    const int e = ec * RF_EC + warp;
    const int rowf = nch * RF_CPAD;
    pdl_launch_dependents();
    // 1. the CTA's router rows, one K half (32 chunks of 32 values) at a time, copied into shared memory
    //    as 16-byte pieces with consecutive threads on consecutive pieces of a row (coalesced; a lane
    //    loading its own chunks touched 32 lines per load instruction); the first half before the wait
    //    (constant weights), the second half into L2 meanwhile
    float* ws = rf_sm + RF_TPG * rowf;
    auto load_w_half = [&](int half) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int idx = tid + RF_THREADS * j;                // expert idx / 256, chunk (idx / 8) % 32, piece idx % 8
            const int we = idx >> 8, c = (idx >> 3) & 31, pc = idx & 7;
            const int eg = ec * RF_EC + we;
            if (eg < E)
                cp_async16(ws + (we * 32 + c) * RF_CPAD + 4 * pc, a.w_router + (int64_t)eg * H + 32 * (32 * half + c) + 4 * pc);
        }
        cp_async_commit();
    };
    load_w_half(0);
    if (cpl > 1 && ec * RF_EC + (tid >> 5) < E)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.w_router + (int64_t)(ec * RF_EC + (tid >> 5)) * H + 32 * (32 + lane)));
    pdl_wait();
    if (a.stamp && tid == 0) atomicMin(a.stamp, gtimer());
    const R* x = reinterpret_cast<const R*>(a.x);
    // f32 rows: all the CTA's rows are copied into the fx layout at once (cp.async), then normalised
    // in place; bf16 rows are read per token
    if (std::is_same<R, float>::value) {
        for (int pc = tid; pc < nt * (H / 4); pc += RF_THREADS) {
            const int tt = pc / (H / 4), i = 4 * (pc - tt * (H / 4));
            cp_async16(rf_sm + tt * rowf + (i >> 5) * RF_CPAD + (i & 31), x + (int64_t)(t0 + tt) * H + i);
        }
        cp_async_commit();
    }
    cp_async_wait_all();
    __syncthreads();
#pragma unroll 1
    for (int tt = 0; tt < nt; ++tt) {
        // the arithmetic of rms_row_scale (thread order of the squares, warp butterfly, warps in order)
        const int64_t t = t0 + tt;
        float* fr = rf_sm + tt * rowf;
        float v[VPT];
#pragma unroll
        for (int j = 0; j < VPT / 4; ++j) {
            const int i = 4 * (tid + 256 * j);
            if (i < H) {
                if (std::is_same<R, float>::value) {
                    const float4 f = *reinterpret_cast<const float4*>(fr + (i >> 5) * RF_CPAD + (i & 31));
                    v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
                } else {
                    Vec4<R>::load(x + t * H + i, v + 4 * j);
                }
            } else {
                v[4 * j] = v[4 * j + 1] = v[4 * j + 2] = v[4 * j + 3] = 0.f;
            }
        }
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < VPT; ++j) ss += (double)(v[j] * v[j]);
        ss = block_sum_d(ss, redd);
        const float scale = 1.0f / sqrtf((float)(ss / H) + a.eps);
#pragma unroll
        for (int j = 0; j < VPT / 4; ++j) {
            const int i = 4 * (tid + 256 * j);
            if (i < H) {
                const float4 wn = *reinterpret_cast<const float4*>(a.w_norm + i);
                const float4 f = make_float4((v[4 * j] * scale) * wn.x, (v[4 * j + 1] * scale) * wn.y,
                                             (v[4 * j + 2] * scale) * wn.z, (v[4 * j + 3] * scale) * wn.w);
                *reinterpret_cast<float4*>(fr + (i >> 5) * RF_CPAD + (i & 31)) = f;
                if (ec == 0) *reinterpret_cast<float4*>(a.fx + t * H + i) = f;
            }
        }
    }
    __syncthreads();
    // 2. logits of expert e for the CTA's tokens: lane = chunk within the K half; the f32 sum of a chunk
    //    runs over its 32 values in order (the chunk sums of k_router_logits)
    for (int half = 0; half < cpl; ++half) {
        if (half > 0) {
            __syncthreads();                                 // every warp is done with the first half
            load_w_half(half);
            cp_async_wait_all();
            __syncthreads();
        }
        if (e < E) {
            const float* wrow = ws + (warp * 32 + lane) * RF_CPAD;
            float4 wv[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) wv[q] = *reinterpret_cast<const float4*>(wrow + 4 * q);
            const int c = 32 * half + lane;
#pragma unroll 1
            for (int tt = 0; tt < nt; ++tt) {
                const float* fr = rf_sm + tt * rowf + c * RF_CPAD;
                float acc = 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 f = *reinterpret_cast<const float4*>(fr + 4 * q);
                    acc = fmaf(f.x, wv[q].x, acc);
                    acc = fmaf(f.y, wv[q].y, acc);
                    acc = fmaf(f.z, wv[q].z, acc);
                    acc = fmaf(f.w, wv[q].w, acc);
                }
                cs[warp][tt][c] = acc;
            }
        }
    }
    __syncwarp();
    if (e < E) {
        const int cps = nch / a.ks;
#pragma unroll 1
        for (int tt = 0; tt < nt; ++tt) {
            // split sums: split z covers chunks [z*cps, (z+1)*cps), added in double from 0
            for (int z = lane; z < a.ks; z += 32) {
                double sz = 0.0;
                for (int c = z * cps; c < (z + 1) * cps; ++c) sz += (double)cs[warp][tt][c];
                ps[warp][z] = sz;
            }
            __syncwarp();
            double rs = 0.0;
            if (lane < a.subs) {
                const int z0 = (int)((int64_t)a.ks * lane / a.subs), z1 = (int)((int64_t)a.ks * (lane + 1) / a.subs);
                for (int z = z0; z < z1; ++z) rs += ps[warp][z];
            }
            double tot = __shfl_sync(0xFFFFFFFFu, rs, 0);
            for (int sb = 1; sb < a.subs; ++sb) tot += __shfl_sync(0xFFFFFFFFu, rs, sb);
            if (lane == 0) a.logits[(t0 + tt) * (int64_t)E + e] = (float)tot;
            __syncwarp();
        }
    }
    // 3. Q8_K of fx segments ec, ec + n_ec, ...
    const int nseg = H / QK;
    for (int sg = ec; sg < nseg; sg += n_ec) {
#pragma unroll 1
        for (int tt = 0; tt < nt; ++tt) {
            const int i = sg * QK + tid;
            const int64_t t = t0 + tt;
            quant_seg256(rf_sm[tt * rowf + (i >> 5) * RF_CPAD + (i & 31)], redf, a.fx_q + t * H + sg * QK,
                         a.fx_d + t * nseg + sg, a.fx_bs + t * (H / 16) + sg * 16);
        }
    }
    // 4. arrival of the CTA in its token group (release: CTA barrier, fence, atomic; the last arriver
    //    fences again before it reads what the others wrote, through L2)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const bool last = atomicAdd(&a.cnt[RF_CNT_STRIDE * tg], 1u) == (unsigned)(n_ec - 1);
        if (last) __threadfence();
        s_last = last;
    }
    __syncthreads();
    if (!s_last) {
        if (a.stamp && tid == 0) atomicMax(a.stamp + 1, gtimer());
        return;
    }
    float* lgs = rf_sm;                                  // [tpg][32 * NV]
    for (int i = tid; i < nt * E; i += RF_THREADS) {
        const int tt = i / E;
        lgs[tt * 32 * NV + (i - tt * E)] = __ldcg(a.logits + (int64_t)t0 * E + i);
    }
    __syncthreads();
    if (warp < nt)
        route_topk_row<NV>(lgs + warp * 32 * NV, E, a.k, a.renorm, lane, a.sel + (int64_t)(t0 + warp) * a.k,
                           a.w + (int64_t)(t0 + warp) * a.k);
    __syncthreads();
    if (tid == 0) {
        a.cnt[RF_CNT_STRIDE * tg] = 0u;                  // every CTA of the group has arrived
        __threadfence();
        const bool last = atomicAdd(&a.cnt[RF_CNT_STRIDE * n_tg], 1u) == (unsigned)(n_tg - 1);
        if (last) {
            __threadfence();
            a.cnt[RF_CNT_STRIDE * n_tg] = 0u;
        }
        s_last = last;
    }
    __syncthreads();
    if (!s_last) {
        if (a.stamp && tid == 0) atomicMax(a.stamp + 1, gtimer());
        return;
    }
    dispatch_small<RF_THREADS>(a.sel, a.T, a.k, a.KK, a.n_slots, a.counts, a.offsets, a.perm, a.err, a.tile_m,
                               a.items, a.n_items, reinterpret_cast<int*>(rf_sm), wtot);
    if (a.stamp) {
        __syncthreads();
        if (tid == 0) atomicMax(a.stamp + 1, gtimer());
    }
}

bool route_fused_supported(const Dims& d, int T) {
    if (T < 1 || T > RF_MAX_T || T >= RB_MIN_T) return false;
    if (d.H != 1024 && d.H != 2048) return false;            // one or two K chunks per lane
    if (d.E < 1 || d.E > RF_MAX_E || d.k < 1 || d.k > MAX_K || d.k > d.E) return false;
    const int ks = router_ksplit(T, d.E, d.H);
    return ks >= 1 && (d.H / RL_KC) % ks == 0;
}

template <typename R, int VPT, int NV>
static cudaError_t launch_route_fused_nv(const RouteFusedArgs& a, dim3 grid, size_t dyn, cudaStream_t s) {
    static unsigned long long attr_set = 0;             // devices on which the shared-memory limit was raised
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(attr_set >> dev & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_route_fused<R, VPT, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             RF_SMEM_MAX);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set |= 1ull << dev;
    }
    return launch_pdl(k_route_fused<R, VPT, NV>, grid, RF_THREADS, dyn, s, a);
}
template <typename R, int VPT>
static cudaError_t launch_route_fused_t(const RouteFusedArgs& a, dim3 grid, size_t dyn, cudaStream_t s) {
    if (a.E <= 128) return launch_route_fused_nv<R, VPT, 4>(a, grid, dyn, s);
    return launch_route_fused_nv<R, VPT, 16>(a, grid, dyn, s);
}

cudaError_t launch_route_fused(const Dims& d, const LayerWeights& lw, const Scratch& sc, const void* x, int T, int KK,
                               int32_t* sel, float* w, int tile_m, cudaStream_t s, unsigned long long* stamp) {
    if (!route_fused_supported(d, T)) return cudaErrorInvalidValue;
    RouteFusedArgs a{};
    a.x = x;
    a.T = T; a.H = d.H; a.E = d.E; a.k = d.k; a.KK = KK; a.renorm = d.renorm; a.n_slots = lw.n_slots;
    a.tile_m = tile_m;
    a.eps = d.eps;
    a.ks = router_ksplit(T, d.E, d.H);
    // k_route_topk's summation ranges of the K splits with one token per CTA (T <= TOPK_SMALL_T)
    int subs = 1;
    while (subs < 16 && subs * 2 * d.E <= TOPK_SMALL_THREADS && subs * 2 <= a.ks) subs *= 2;
    a.subs = subs;
    a.w_norm = lw.w_norm; a.w_router = lw.w_router;
    a.fx = sc.fx; a.fx_q = sc.fx_q; a.fx_d = sc.fx_d; a.fx_bs = sc.fx_bs;
    a.logits = reinterpret_cast<float*>(sc.rpart);
    a.sel = sel; a.w = w;
    a.counts = sc.counts; a.offsets = sc.offsets; a.perm = sc.perm; a.items = sc.items; a.n_items = sc.n_items;
    a.err = sc.sync;
    a.cnt = sc.sync + RF_CNT_OFF;
    a.stamp = stamp;
    // tokens per CTA: the fewest (most parallel) that keep the grid within two CTAs per SM
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int n_ec = (d.E + RF_EC - 1) / RF_EC;
    a.tpg = RF_TPG;
    for (int tp = 1; tp < RF_TPG; tp *= 2)
        if ((int64_t)n_ec * ((T + tp - 1) / tp) <= 2 * (int64_t)sms[dev]) { a.tpg = tp; break; }
    const dim3 grid(n_ec, (T + a.tpg - 1) / a.tpg);
    const int NS = lw.n_slots + (KK > d.k ? 1 : 0);
    size_t dyn = (size_t)RF_TPG * (d.H / RL_KC) * RF_CPAD * 4 + (size_t)RF_EC * 32 * RF_CPAD * 4;   // fx + a W half
    dyn = std::max(dyn, (size_t)RF_TPG * 32 * (d.E <= 128 ? 4 : 16) * 4);
    dyn = std::max(dyn, (size_t)(NS + 1 + 2 * T * KK) * 4);
    if (dyn > (size_t)RF_SMEM_MAX) return cudaErrorInvalidValue;
    if (d.H <= 1024)
        return d.resid_bf16 ? launch_route_fused_t<__nv_bfloat16, 4>(a, grid, dyn, s)
                            : launch_route_fused_t<float, 4>(a, grid, dyn, s);
    return d.resid_bf16 ? launch_route_fused_t<__nv_bfloat16, 8>(a, grid, dyn, s)
                        : launch_route_fused_t<float, 8>(a, grid, dyn, s);
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

// A row's units held in registers: lane takes units lane, lane + 32, ... (UPL of them), loaded once
// and dotted against every entry of the slot. The float sum runs over the units in the same order as
// row_dot_lane's, so the result is bit-identical to re-reading the row for each entry.
template <int TYPE, int UPL>
struct RowRegs {
    RowUnit<TYPE> u[UPL];
    bool has[UPL];
    __device__ __forceinline__ void load(const uint8_t* base, int64_t nblk, int64_t row, int nb, int unit0, int nunits) {
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
            const int un = unit0 + 32 * i;
            has[i] = un < nunits;
            if (has[i]) u[i].load(base, nblk, row, nb, un);
        }
    }
    __device__ __forceinline__ float dot(const ActRow& a) const {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < UPL; ++i)
            if (has[i]) acc += u[i].dot(a);
        return acc;
    }
};

// Gate/up of Q4_K slots for small batches: a warp loads its two rows (gate and up) once and runs every
// entry of the slot against them; other weight types take the per-entry row dots.
template <int UPL>
__global__ void __launch_bounds__(256) k_gateup_regs(LayerWeights lw, int H, int I, int KK,
                                                     const int* __restrict__ offsets, const int* __restrict__ perm,
                                                     const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                                     const int* __restrict__ xbs, float* __restrict__ h) {
    pdl_enter();
    const int s = blockIdx.x;
    const int start = offsets[s], end = offsets[s + 1];
    if (start == end) return;
    const SlotMats m = slot_mats(lw, s);
    const int nb = H / QK;
    const int64_t nblk = (int64_t)I * nb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i0 = blockIdx.y * GU_ROWS + warp, i1 = i0 + 8;
    const int r1 = min(I, (int)(blockIdx.y + 1) * GU_ROWS);
    if (m.gt != T_Q4K || m.ut != T_Q4K) {
        for (int i = i0; i < r1; i += 8) {
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
        return;
    }
    const int nunits = nb * 8;
    const bool v0 = i0 < r1, v1 = i1 < r1;
    RowRegs<T_Q4K, UPL> g0, u0, g1, u1;
    if (v0) { g0.load(m.g, nblk, i0, nb, lane, nunits); u0.load(m.u, nblk, i0, nb, lane, nunits); }
    if (v1) { g1.load(m.g, nblk, i1, nb, lane, nunits); u1.load(m.u, nblk, i1, nb, lane, nunits); }
    for (int p = start; p < end; ++p) {
        const int ent = perm[p];
        const int t = ent / KK;
        const ActRow a{xq + (size_t)t * H, xd + (size_t)t * nb, xbs + (size_t)t * (H / 16)};
        if (v0) {
            const float g = warp_sum(g0.dot(a)), u = warp_sum(u0.dot(a));
            if (lane == 0) h[(size_t)ent * I + i0] = silu_f(g) * u;
        }
        if (v1) {
            const float g = warp_sum(g1.dot(a)), u = warp_sum(u1.dot(a));
            if (lane == 0) h[(size_t)ent * I + i1] = silu_f(g) * u;
        }
    }
}

// Down rows for small batches: G lanes per row (G = the power of two covering the row's units, so a
// warp holds 32/G rows), each lane's unit loaded once and run against every entry of the slot; two
// row sets per warp in flight. The G-lane reduction equals a warp-wide one over a single row (the
// lanes it leaves out hold zeros), so results match the per-entry kernel bit for bit.
template <int G>
__global__ void __launch_bounds__(256) k_down_regs(LayerWeights lw, int H, int I, const int* __restrict__ offsets,
                                                   const int* __restrict__ perm, const int8_t* __restrict__ hq,
                                                   const float* __restrict__ hd, const int* __restrict__ hbs,
                                                   float* __restrict__ y) {
    pdl_enter();
    const int s = blockIdx.x;
    const int start = offsets[s], end = offsets[s + 1];
    if (start == end) return;
    const SlotMats m = slot_mats(lw, s);
    const int nb = I / QK;
    const int64_t nblk = (int64_t)H * nb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int RPW = 32 / G;                    // rows per warp and row set
    const int sub = lane / G, gl = lane - sub * G;
    const int rows_cta = 16 * RPW;                 // two row sets of 8 warps
    const int base = blockIdx.y * rows_cta;
    const int r1 = min(H, base + rows_cta);
    const int ra = base + warp * RPW + sub, rb = ra + 8 * RPW;
    auto run = [&](auto tag) {
        constexpr int DT = decltype(tag)::value;
        const int nunits = nb * (DT == T_Q4K ? 8 : 4);
        const bool va = ra < r1 && gl < nunits, vb = rb < r1 && gl < nunits;
        RowUnit<DT> xa, xb;
        if (va) xa.load(m.d, nblk, ra, nb, gl);
        if (vb) xb.load(m.d, nblk, rb, nb, gl);
        for (int p = start; p < end; ++p) {
            const int ent = perm[p];
            const ActRow a{hq + (size_t)ent * I, hd + (size_t)ent * nb, hbs + (size_t)ent * (I / 16)};
            float fa = va ? xa.dot(a) : 0.f, fb = vb ? xb.dot(a) : 0.f;
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) {
                fa += __shfl_xor_sync(0xffffffffu, fa, o);
                fb += __shfl_xor_sync(0xffffffffu, fb, o);
            }
            if (gl == 0 && ra < r1) y[(size_t)ent * H + ra] = fa;
            if (gl == 0 && rb < r1) y[(size_t)ent * H + rb] = fb;
        }
    };
    if (m.dt == T_Q4K) run(std::integral_constant<int, T_Q4K>());
    else run(std::integral_constant<int, T_Q6K>());
}

__global__ void __launch_bounds__(256) k_gateup(LayerWeights lw, int H, int I, int KK, const int* __restrict__ offsets,
                                                const int* __restrict__ perm, const int8_t* __restrict__ xq,
                                                const float* __restrict__ xd, const int* __restrict__ xbs,
                                                float* __restrict__ h) {
    pdl_enter();
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
    pdl_enter();
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
    pdl_enter();
    __shared__ double redd[32];
    const int t = blockIdx.x;
    double acc = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) acc += (double)g[i] * (double)fx[(size_t)t * H + i];
    acc = block_sum_d(acc, redd);
    if (threadIdx.x == 0) out[t] = sigmoid_f((float)acc);
}

// x[t] += sum_j w[t][j] * y[row(t, j)] (+ sh_gate[t] * y[t*KK + k]), j ascending; row(t, j) =
// t*KK + j, or pos[t*k + j] for rows that came back from an expert-parallel exchange. Four columns
// per thread, the k rows' loads issued together.
__device__ __forceinline__ float4 ld_y4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld_y4(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// YT: float (grouped path) or __half (tensor-core path) expert outputs
template <typename R, typename YT>
__global__ void __launch_bounds__(256) k_combine(const YT* __restrict__ y, const float* __restrict__ w,
                                                 const float* __restrict__ sh_gate, int k, int KK, int H, int T,
                                                 R* x, const int* __restrict__ pos) {
    pdl_enter();
    const int64_t nq = (int64_t)T * H / 4;
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < nq; q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = (q * 4) / H;
        const int64_t dcol = q * 4 - t * H;
        const YT* yb = y + t * KK * H + dcol;
        float4 yv[MAX_K];
#pragma unroll
        for (int j = 0; j < MAX_K; ++j)
            if (j < k) {
                const int row = pos ? pos[t * k + j] : -1;
                yv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (!pos)
                    yv[j] = ld_y4(yb + (int64_t)j * H);
                else if (row >= 0)                         // < 0: the entry was rejected at pack time
                    yv[j] = ld_y4(y + (int64_t)row * H + dcol);
            }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < MAX_K; ++j) {
            if (j < k) {
                const float wj = w[t * k + j];
                acc.x = fmaf(wj, yv[j].x, acc.x);
                acc.y = fmaf(wj, yv[j].y, acc.y);
                acc.z = fmaf(wj, yv[j].z, acc.z);
                acc.w = fmaf(wj, yv[j].w, acc.w);
            }
        }
        if (KK > k && !pos) {
            const float4 ys = ld_y4(yb + (int64_t)k * H);
            const float g = sh_gate[t];
            acc.x = fmaf(ys.x, g, acc.x);
            acc.y = fmaf(ys.y, g, acc.y);
            acc.z = fmaf(ys.z, g, acc.z);
            acc.w = fmaf(ys.w, g, acc.w);
        }
        R* xp = x + q * 4;
        xp[0] = from_f32<R>(acc.x + to_f32<R>(xp[0]));
        xp[1] = from_f32<R>(acc.y + to_f32<R>(xp[1]));
        xp[2] = from_f32<R>(acc.z + to_f32<R>(xp[2]));
        xp[3] = from_f32<R>(acc.w + to_f32<R>(xp[3]));
    }
}

// The same combine over f16 expert outputs (tensor-core path and expert-parallel returns): eight
// columns per thread (one 16-byte load per row), the k rows in batches of eight loads in flight.
template <typename R>
__global__ void __launch_bounds__(256) k_combine_h(const __half* __restrict__ y, const float* __restrict__ w,
                                                   const float* __restrict__ sh_gate, int k, int KK, int H, int T,
                                                   R* x, const int* __restrict__ pos) {
    pdl_enter();
    const int64_t n8 = (int64_t)T * H / 8;
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n8; q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = (q * 8) / H;
        const int64_t dcol = q * 8 - t * H;
        float acc[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = 0.f;
        for (int j0 = 0; j0 < k; j0 += 8) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = make_uint4(0, 0, 0, 0);
                const int j = j0 + u;
                if (j < k) {
                    const int64_t row = pos ? (int64_t)pos[t * k + j] : t * KK + j;
                    if (row >= 0) v[u] = *reinterpret_cast<const uint4*>(y + row * H + dcol);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int j = j0 + u;
                if (j < k) {
                    const float wj = w[t * k + j];
                    const uint32_t pw[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[c]));
                        acc[2 * c] += wj * f.x;
                        acc[2 * c + 1] += wj * f.y;
                    }
                }
            }
        }
        if (KK > k && !pos) {
            const uint4 vs = *reinterpret_cast<const uint4*>(y + (t * KK + k) * H + dcol);
            const float g = sh_gate[t];
            const uint32_t pw[4] = {vs.x, vs.y, vs.z, vs.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[c]));
                acc[2 * c] = acc[2 * c] + f.x * g;
                acc[2 * c + 1] = acc[2 * c + 1] + f.y * g;
            }
        }
        R* xp = x + q * 8;
#pragma unroll
        for (int c = 0; c < 8; ++c) xp[c] = from_f32<R>(acc[c] + to_f32<R>(xp[c]));
    }
}

cudaError_t launch_shared_gate(const float* fx, const float* gate_inp, int H, int T, float* out, cudaStream_t s) {
    launch_pdl(k_shared_gate, T, 256, 0, s, fx, gate_inp, H, out);
    return cudaGetLastError();
}

// Large batches: per-CTA shared-memory histograms added into global counts, a one-CTA scan, and a
// scatter through global cursors (warp-aggregated atomics).
constexpr int DISP_SMALL = 4096;     // entries handled by the single-CTA kernel
constexpr int DISP_CHUNK = 512;      // entries per CTA in the multi-CTA kernels (one per thread)

__global__ void __launch_bounds__(512) k_disp_count(const int32_t* __restrict__ slot_of, int T, int k, int KK,
                                                    int n_slots, int* __restrict__ gcount, unsigned* err,
                                                    bool skip_neg) {
    pdl_enter();
    extern __shared__ int hist[];
    const int NS = n_slots + (KK > k ? 1 : 0);
    for (int i = threadIdx.x; i < NS; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int n = T * KK;
    const int e0 = blockIdx.x * DISP_CHUNK, e1 = min(n, e0 + DISP_CHUNK);
    for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
        const int t = e / KK, j = e - t * KK;
        const int sl = (j < k) ? (int)slot_of[(size_t)t * k + j] : n_slots;
        if (sl < 0 || sl >= NS || (j < k && sl >= n_slots)) {
            if (!(skip_neg && sl < 0)) atomicOr(err, 1u);
            continue;
        }
        atomicAdd(&hist[sl], 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NS; i += blockDim.x)
        if (hist[i]) atomicAdd(&gcount[i], hist[i]);
}

__global__ void __launch_bounds__(DISP_THREADS) k_disp_scan(int NS, int* __restrict__ gcount, int* __restrict__ counts,
                                                            int* __restrict__ offsets, int* __restrict__ cursor,
                                                            int tile_m, int2* __restrict__ items,
                                                            int* __restrict__ n_items) {
    pdl_enter();
    __shared__ int2 wtot[32];
    const int c = (NS + DISP_THREADS - 1) / DISP_THREADS;
    const int s0 = threadIdx.x * c, s1 = min(NS, s0 + c);
    int2 mine = make_int2(0, 0);
    for (int sl = s0; sl < s1; ++sl) {
        mine.x += gcount[sl];
        if (tile_m > 0) mine.y += (gcount[sl] + tile_m - 1) / tile_m;
    }
    int2 total;
    int2 off = scan_excl_cta<DISP_THREADS>(mine, wtot, total);
    for (int sl = s0; sl < s1; ++sl) {
        const int cn = gcount[sl];
        offsets[sl] = off.x;
        counts[sl] = cn;
        cursor[sl] = off.x;
        off.x += cn;
        if (tile_m > 0) {
            for (int mt = 0; mt * tile_m < cn; ++mt) items[off.y + mt] = make_int2(sl, mt);
            off.y += (cn + tile_m - 1) / tile_m;
        }
        gcount[sl] = 0;                       // ready for the next call
    }
    if (threadIdx.x == 0) {
        offsets[NS] = total.x;
        if (tile_m > 0) *n_items = total.y;
    }
}

__global__ void __launch_bounds__(512) k_disp_scatter(const int32_t* __restrict__ slot_of, int T, int k, int KK,
                                                      int n_slots, int* __restrict__ cursor, int* __restrict__ perm) {
    pdl_enter();
    const int NS = n_slots + (KK > k ? 1 : 0);
    const int n = T * KK;
    const int lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * DISP_CHUNK, e1 = min(n, e0 + DISP_CHUNK);
    for (int base = e0; base < e1; base += blockDim.x) {
        const int e = base + threadIdx.x;
        int sl = -1;
        if (e < e1) {
            const int t = e / KK, j = e - t * KK;
            sl = (j < k) ? (int)slot_of[(size_t)t * k + j] : n_slots;
            if (sl < 0 || sl >= NS || (j < k && sl >= n_slots)) sl = -1;
        }
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, sl);
        const int leader = __ffs(peers) - 1;
        int pos = 0;
        if (lane == leader && sl >= 0) pos = atomicAdd(&cursor[sl], __popc(peers));
        pos = __shfl_sync(0xFFFFFFFFu, pos, leader);
        if (sl >= 0) perm[pos + __popc(peers & ((1u << lane) - 1u))] = e;
    }
}

cudaError_t launch_rmsnorm_f32(const float* x, int rows, int cols, float eps, const float* w, float* out,
                               cudaStream_t s) {
    return launch_rmsnorm_rows(x, rows, cols, eps, w, out, s);
}

cudaError_t launch_quant_q8(const float* x, int rows, int K, int8_t* q, float* d, int* bs, cudaStream_t s) {
    if (rows <= 0 || K <= 0 || K % QK) return cudaErrorInvalidValue;
    return launch_pdl(k_quant_q8, (unsigned)((int64_t)(K / QK) * rows), 256, 0, s, x, K, q, d, bs);
}

cudaError_t launch_dispatch(const int32_t* slot_of_sel, int T, int k, int KK, int n_slots, const Scratch& sc,
                            int tile_m, cudaStream_t s, int* launches, bool skip_neg) {
    const int NS = n_slots + (KK > k ? 1 : 0);
    const int n = T * KK;
    if (n <= DISP_SMALL) {
        const size_t dsm = (size_t)2 * (NS + 1) * sizeof(int);
        launch_pdl(k_dispatch, 1, DISP_THREADS, dsm, s, slot_of_sel, T, k, KK, n_slots, sc.counts, sc.offsets, sc.perm,
                                                sc.sync, tile_m, sc.items, sc.n_items, skip_neg);
        if (launches) *launches += 1;
        return cudaGetLastError();
    }
    const int grid = (n + DISP_CHUNK - 1) / DISP_CHUNK;
    launch_pdl(k_disp_count, grid, 512, (size_t)NS * sizeof(int), s, slot_of_sel, T, k, KK, n_slots, sc.dcount, sc.sync,
                                                                    skip_neg);
    launch_pdl(k_disp_scan, 1, DISP_THREADS, 0, s, NS, sc.dcount, sc.counts, sc.offsets, sc.dcursor, tile_m, sc.items,
                                           sc.n_items);
    launch_pdl(k_disp_scatter, grid, 512, 0, s, slot_of_sel, T, k, KK, n_slots, sc.dcursor, sc.perm);
    if (launches) *launches += 3;
    return cudaGetLastError();
}

cudaError_t launch_combine(const Dims& d, const Scratch& sc, const float* w, void* x_inout, int T, int KK,
                           cudaStream_t s, bool y_half) {
    const int64_t n = (int64_t)T * d.H / 4;
    const int cb = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    const __half* yh = reinterpret_cast<const __half*>(sc.y);
    const int64_t n8 = (int64_t)T * d.H / 8;
    const int cbh = (int)((n8 + 255) / 256 < 148 * 16 ? (n8 + 255) / 256 : 148 * 16);
    if (d.resid_bf16) {
        auto* x = (__nv_bfloat16*)x_inout;
        if (y_half) launch_pdl(k_combine_h<__nv_bfloat16>, cbh, 256, 0, s, yh, w, sc.sh_gate, d.k, KK, d.H, T, x, nullptr);
        else launch_pdl(k_combine<__nv_bfloat16, float>, cb, 256, 0, s, sc.y, w, sc.sh_gate, d.k, KK, d.H, T, x, nullptr);
    } else {
        auto* x = (float*)x_inout;
        if (y_half) launch_pdl(k_combine_h<float>, cbh, 256, 0, s, yh, w, sc.sh_gate, d.k, KK, d.H, T, x, nullptr);
        else launch_pdl(k_combine<float, float>, cb, 256, 0, s, sc.y, w, sc.sh_gate, d.k, KK, d.H, T, x, nullptr);
    }
    return cudaGetLastError();
}

cudaError_t launch_combine_rows(const Dims& d, const uint16_t* y, const int* pos, const float* w, void* x_inout, int T,
                                cudaStream_t s) {
    const int64_t n8 = (int64_t)T * d.H / 8;
    const int cb = (int)((n8 + 255) / 256 < 148 * 16 ? (n8 + 255) / 256 : 148 * 16);
    const __half* yh = reinterpret_cast<const __half*>(y);
    if (d.resid_bf16)
        launch_pdl(k_combine_h<__nv_bfloat16>, cb, 256, 0, s, yh, w, nullptr, d.k, d.k, d.H, T, (__nv_bfloat16*)x_inout, pos);
    else
        launch_pdl(k_combine_h<float>, cb, 256, 0, s, yh, w, nullptr, d.k, d.k, d.H, T, (float*)x_inout, pos);
    return cudaGetLastError();
}

cudaError_t launch_experts_grouped(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                                   const int32_t* slot_of_sel, const float* w, void* x_inout, int T,
                                   bool /*need_sh_gate*/, cudaStream_t s, int* launches, bool prepared,
                                   unsigned long long* stamp) {
    const bool shared = lw.shared != nullptr;
    const int KK = d.k + (shared ? 1 : 0);
    const int NS = lw.n_slots + (shared ? 1 : 0);
    int nl = 0;
    cudaError_t e;
    // 1. quantise fx (done by the fused route kernel when `prepared`, with the dispatch)
    if (!prepared) {
        launch_pdl(k_quant_q8, (unsigned)((d.H / QK) * T), 256, 0, s, fx, d.H, sc.fx_q, sc.fx_d, sc.fx_bs);
        ++nl;
    }
    if (shared) {
        if ((e = launch_shared_gate(fx, lw.sh_gate_inp, d.H, T, sc.sh_gate, s)) != cudaSuccess) return e;
        ++nl;
    }
    // 2. group entries by slot (with a work list of the non-empty slots for the streaming kernels)
    const bool gu_sw = gateup_sw_supported(d, lw), dn_sw = down_sw_supported(d, lw);
    if (prepared && !(gu_sw || dn_sw)) return cudaErrorInvalidValue;      // the work list must exist
    if (!prepared &&
        (e = launch_dispatch(slot_of_sel, T, d.k, KK, lw.n_slots, sc, (gu_sw || dn_sw) ? (1 << 20) : 0, s, &nl)) !=
            cudaSuccess)
        return e;
    // 3. gate/up + SwiGLU: each selected slot's rows streamed once; otherwise weight rows held in
    //    registers across a slot's entries where the row fits in two units per lane
    const dim3 gu_grid(NS, (d.I + GU_ROWS - 1) / GU_ROWS);
    const int gu_units = (d.H / QK) * 8;
    if (gu_sw) {
        if ((e = launch_gateup_sw(d, lw, sc, KK, s, stamp)) != cudaSuccess) return e;
    } else if (gu_units <= 32)
        launch_pdl(k_gateup_regs<1>, gu_grid, 256, 0, s, lw, d.H, d.I, KK, sc.offsets, sc.perm, sc.fx_q, sc.fx_d, sc.fx_bs, sc.h);
    else if (gu_units <= 64)
        launch_pdl(k_gateup_regs<2>, gu_grid, 256, 0, s, lw, d.H, d.I, KK, sc.offsets, sc.perm, sc.fx_q, sc.fx_d, sc.fx_bs, sc.h);
    else
        launch_pdl(k_gateup, gu_grid, 256, 0, s, lw, d.H, d.I, KK, sc.offsets, sc.perm, sc.fx_q, sc.fx_d, sc.fx_bs, sc.h);
    ++nl;
    // 4. quantise h
    launch_pdl(k_quant_q8, (unsigned)((d.I / QK) * T * KK), 256, 0, s, sc.h, d.I, sc.h_q, sc.h_d, sc.h_bs);
    ++nl;
    // 5. down (the widest row type present sets the lanes per row)
    const int nbI = d.I / QK;
    int dn_units = nbI * (lw.down_type == T_Q4K ? 8 : 4);
    if (shared) dn_units = std::max(dn_units, nbI * (lw.sh_down_type == T_Q4K ? 8 : 4));
    if (dn_sw) {
        if ((e = launch_down_sw(d, lw, sc, s, stamp ? stamp + 2 : nullptr)) != cudaSuccess) return e;
    } else if (dn_units <= 8)
        launch_pdl(k_down_regs<8>, dim3(NS, (d.H + 63) / 64), 256, 0, s, lw, d.H, d.I, sc.offsets, sc.perm, sc.h_q, sc.h_d,
                                                                 sc.h_bs, sc.y);
    else if (dn_units <= 16)
        launch_pdl(k_down_regs<16>, dim3(NS, (d.H + 31) / 32), 256, 0, s, lw, d.H, d.I, sc.offsets, sc.perm, sc.h_q, sc.h_d,
                                                                  sc.h_bs, sc.y);
    else if (dn_units <= 32)
        launch_pdl(k_down_regs<32>, dim3(NS, (d.H + 15) / 16), 256, 0, s, lw, d.H, d.I, sc.offsets, sc.perm, sc.h_q, sc.h_d,
                                                                  sc.h_bs, sc.y);
    else
        launch_pdl(k_down, dim3(NS, (d.H + DN_ROWS - 1) / DN_ROWS), 256, 0, s, lw, d.H, d.I, sc.offsets, sc.perm, sc.h_q,
                                                                        sc.h_d, sc.h_bs, sc.y);
    ++nl;
    // 6. weighted combine into the residual
    if ((e = launch_combine(d, sc, w, x_inout, T, KK, s, false)) != cudaSuccess) return e;
    ++nl;
    if (launches) *launches += nl;
    return cudaGetLastError();
}

}  // namespace hoard
