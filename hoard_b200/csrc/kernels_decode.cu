// kernels_decode.cu -- persistent fused decode kernel: T = 1, every expert resident, any number of
// consecutive layers in one cooperative launch (one CTA per SM).
//
// Per layer l (hoard's graph A router tail + graph B + host combine, src/run_moe_stream.cpp:352-447):
//   A  every CTA reduces the router sums of layer l (accumulated by all CTAs at the end of layer
//      l-1), runs softmax + top-k itself (identical arithmetic in every CTA), and builds the Q8_K
//      activation of fx = rms_norm(x) * ffn_norm in shared memory;
//   B  one thread issues cp.async.bulk copies of this CTA's share of the selected experts' bytes
//      (gate/up row pairs AND down rows) plus the next layer's router slice, all at once, so the
//      whole layer's weight bytes are in flight while the CTA computes;
//   C  gate/up row pairs from shared memory: h = silu(gate . fx) * (up . fx) -> global, plus a
//      per-256-block max|h| (the Q8_K scale of h) by atomicMax;
//      ---- grid barrier ----
//   D  Q8_K of h in shared memory; this CTA's output rows for every selected expert; the combine
//      x[d] = sum_j w_j*y_j[d] + x[d] (j ascending); then the next layer's router partial sums over
//      these rows (sum x^2 and W_r^T[d,:] . (ffn_norm[d]*x[d])) added into double accumulators;
//      ---- grid barrier ----
// Every wait (grid barrier, mbarrier) is bounded by %globaltimer; on expiry the kernel sets
// bit 2 of the error word, stops computing, drains its own copies (bounded) and exits.
#include "common.cuh"
#include "kernels.h"
#include "block_ops.cuh"

namespace hoard {

namespace {

constexpr int DEC_THREADS = 512;
constexpr unsigned long long WAIT_NS = 2000000000ull;   // 2 s bound on any wait

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier; false if the bound expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > WAIT_NS) return false;
    }
    return true;
}
// 1-D bulk copy global -> shared, completion counted on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_add_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ld_f32(const float* p) {   // coherent load of data written in this launch
    float v;
    asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ double ld_f64(const double* p) {
    double v;
    asm volatile("ld.relaxed.gpu.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float ld_resid(const float* p) { return ld_f32(p); }
__device__ __forceinline__ float ld_resid(const __nv_bfloat16* p) {
    unsigned short v;
    asm volatile("ld.relaxed.gpu.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
    return __bfloat162float(__ushort_as_bfloat16(v));
}
__device__ __forceinline__ float4 ld_f32x4(const float* p) {
    float4 v;
    asm volatile("ld.relaxed.gpu.global.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p) : "memory");
    return v;
}

// Grid barrier number `n` (0, 1, 2, ... within this launch). Returns false on timeout / error.
__device__ bool grid_barrier(unsigned* sync, unsigned n, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        red_add_release(&sync[1], 1u);
        const unsigned target = (n + 1) * gridDim.x;
        if (ld_acquire(&sync[1]) < target) {
            const unsigned long long t0 = gtimer();
            while (ld_acquire(&sync[1]) < target) {
                if (ld_relaxed(&sync[0]) & 2u) { ok = 0; break; }
                if (gtimer() - t0 > WAIT_NS) { atomicOr(&sync[0], 2u); ok = 0; break; }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

inline __host__ __device__ int64_t a16(int64_t v) { return (v + 15) & ~(int64_t)15; }

}  // namespace

// Shared-memory plan; identical on host (sizing) and device (offsets). Sized for the largest
// share of any CTA: ceil(k*I/G) gate/up row pairs and ceil(H/G) output rows.
struct DecodePlan {
    int H, E, k, I, nbH, nbI, dt;
    int np_max, nr_max;
    int64_t gu_row_qs, gu_row_hdr;          // bytes per gate/up row in the two Q4_K planes
    int64_t off_gate_qs, off_gate_hdr, off_up_qs, off_up_hdr;
    int64_t dn_stride;                      // bytes of one expert's down rows (all planes)
    int64_t dn_p0, dn_p1, dn_p2, dn_p3;     // plane offsets inside an expert's down region
    int64_t off_dn, off_wt, off_wn, off_fxq, off_fxd, off_fxbs, off_hq, off_hd, off_hbs, off_y, off_xs,
        off_lg, off_misc, total;

    __host__ __device__ void init(int H_, int E_, int k_, int I_, int dt_, int G) {
        H = H_; E = E_; k = k_; I = I_; dt = dt_;
        nbH = H / QK; nbI = I / QK;
        np_max = (k * I + G - 1) / G;
        nr_max = (H + G - 1) / G;
        gu_row_qs = (int64_t)nbH * 128;
        gu_row_hdr = (int64_t)nbH * 16;
        int64_t o = 0;
        off_gate_qs = o; o += np_max * gu_row_qs;
        off_gate_hdr = o; o += np_max * gu_row_hdr;
        off_up_qs = o; o += np_max * gu_row_qs;
        off_up_hdr = o; o += np_max * gu_row_hdr;
        // down planes of one expert for nr_max rows (+16 slack for supersets of unaligned planes);
        // the region stride is the larger of the two formats so that nothing after it moves when
        // the down type changes from layer to layer
        const int64_t rq = (int64_t)nbI * 128;
        const int64_t q4_p1 = a16(nr_max * rq) + 16;
        const int64_t q4_end = q4_p1 + a16(nr_max * (int64_t)nbI * 16) + 16;
        const int64_t q6_p1 = a16(nr_max * rq) + 16;
        const int64_t q6_p2 = q6_p1 + a16(nr_max * (int64_t)nbI * 64) + 16;
        const int64_t q6_p3 = q6_p2 + a16(nr_max * (int64_t)nbI * 16) + 16;
        const int64_t q6_end = q6_p3 + a16(nr_max * (int64_t)nbI * 2) + 32;
        dn_stride = q4_end > q6_end ? q4_end : q6_end;
        dn_p0 = 0;
        if (dt == T_Q4K) { dn_p1 = q4_p1; dn_p2 = q4_end; dn_p3 = q4_end; }
        else { dn_p1 = q6_p1; dn_p2 = q6_p2; dn_p3 = q6_p3; }
        off_dn = o; o += (int64_t)k * dn_stride;
        off_wt = o; o += a16((int64_t)nr_max * E * 4) + 16;
        off_wn = o; o += a16((int64_t)nr_max * 4) + 32;
        off_fxq = o; o += a16(H);
        off_fxd = o; o += a16((int64_t)nbH * 4);
        off_fxbs = o; o += a16((int64_t)(H / 16) * 4);
        off_hq = o; o += a16((int64_t)k * I);
        off_hd = o; o += a16((int64_t)k * nbI * 4);
        off_hbs = o; o += a16((int64_t)k * (I / 16) * 4);
        off_y = o; o += a16((int64_t)nr_max * k * 4);
        off_xs = o; o += a16((int64_t)nr_max * 4);
        off_lg = o; o += a16((int64_t)E * 4);
        off_misc = o; o += 256;                  // mbarriers, sel/w, flags
        total = o;
    }
};

struct DecodeArgs {
    const LayerWeights* lw;     // [n_layers] (device)
    int n_layers;
    int H, E, k, I, renorm;
    float eps;
    int resid_bf16;
    void* x;                    // [H] residual, f32 or bf16, updated in place
    int32_t* sel_out;           // [n_layers][k] or null
    float* w_out;
    float* h;                   // [k][I]
    unsigned* amax;             // [2][k][I/256]
    double* racc;               // [2][E+1]
    unsigned* sync;             // [0] error bits, [1] barrier counter, [2] exit counter
};

template <int DT>
__device__ __forceinline__ float down_unit(const uint8_t* reg, const DecodePlan& P, int r, int u, const int8_t* aq,
                                           const float* ad, const int* abs_, int d0_sub) {
    // reg: this expert's down region; r: row within the CTA's rows; u: unit within the row
    if (DT == T_Q4K) {
        const int b = u >> 3, c8 = u & 7;
        const int64_t blk = (int64_t)r * P.nbI + b;
        const uint4 w = *reinterpret_cast<const uint4*>(reg + P.dn_p0 + blk * 128 + 16 * c8);
        const uint4 hh = *reinterpret_cast<const uint4*>(reg + P.dn_p1 + blk * 16);
        return q4k_unit_dot(w, hh, c8, aq + QK * b, abs_ + 16 * b, ad[b]);
    } else {
        const int b = u >> 2, v = u & 3, h2 = v >> 1, rr = v & 1;
        const int64_t blk = (int64_t)r * P.nbI + b;
        const uint4 A = *reinterpret_cast<const uint4*>(reg + P.dn_p0 + blk * 128 + 64 * h2 + 16 * rr);
        const uint4 B = *reinterpret_cast<const uint4*>(reg + P.dn_p0 + blk * 128 + 64 * h2 + 32 + 16 * rr);
        const uint4 C = *reinterpret_cast<const uint4*>(reg + P.dn_p1 + blk * 64 + 32 * h2 + 16 * rr);
        const uint4 S = *reinterpret_cast<const uint4*>(reg + P.dn_p2 + blk * 16);
        const unsigned short dbits = *reinterpret_cast<const unsigned short*>(reg + P.dn_p3 + d0_sub + blk * 2);
        const float d6 = __half2float(__ushort_as_half(dbits));
        return ad[b] * d6 * (float)q6k_unit_isum(A, B, C, S, v, aq + QK * b, abs_ + 16 * b);
    }
}

template <int DT>
__device__ void down_phase(const DecodePlan& P, uint8_t* smem, int nr, int KKk, int dsub) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int sub = lane & 15, hw = warp * 2 + (lane >> 4);
    const int nunits = P.nbI * (DT == T_Q4K ? 8 : 4);
    const int8_t* hq = reinterpret_cast<const int8_t*>(smem + P.off_hq);
    const float* hd = reinterpret_cast<const float*>(smem + P.off_hd);
    const int* hbs = reinterpret_cast<const int*>(smem + P.off_hbs);
    float* y = reinterpret_cast<float*>(smem + P.off_y);
    const int items = nr * KKk;
    for (int it0 = 0; it0 < items; it0 += 2 * nw) {
        const int it = it0 + hw;
        float acc = 0.f;
        int r = 0, j = 0;
        if (it < items) {
            r = it / KKk;
            j = it - r * KKk;
            const uint8_t* reg = smem + P.off_dn + (int64_t)j * P.dn_stride;
            for (int u = sub; u < nunits; u += 16)
                acc += down_unit<DT>(reg, P, r, u, hq + (int64_t)j * P.I, hd + j * P.nbI, hbs + j * (P.I / 16),
                                     dsub);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (it < items && sub == 0) y[r * KKk + j] = acc;
    }
}

template <typename R>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double redd[32];
    __shared__ float redf[32];
    __shared__ int s_sel[16];
    __shared__ float s_w[16];
    __shared__ int s_ok;
    __shared__ float s_scale;

    const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
    const int H = a.H, E = a.E, k = a.k, I = a.I;
    const int nbH = H / QK, nbI = I / QK;
    const int P_pairs = k * I;
    const int q0 = (int)((int64_t)c * P_pairs / G), q1 = (int)((int64_t)(c + 1) * P_pairs / G);
    const int np = q1 - q0;
    const int d0 = (int)((int64_t)c * H / G), d1 = (int)((int64_t)(c + 1) * H / G);
    const int nr = d1 - d0;
    R* x = reinterpret_cast<R*>(a.x);

    float* xs = nullptr;
    bool alive = true;
    unsigned nbar = 0;

    // plan for layer 0's down type (re-initialised per layer: only the down planes depend on it)
    DecodePlan P;
    P.init(H, E, k, I, a.lw[0].down_type, G);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_misc);
    uint64_t* bar_gu = bars + 0;
    uint64_t* bar_dn = bars + 1;
    uint64_t* bar_wt = bars + 2;
    if (tid == 0) {
        mbar_init(bar_gu, 1);
        mbar_init(bar_dn, 1);
        mbar_init(bar_wt, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    xs = reinterpret_cast<float*>(smem + P.off_xs);
    float* wt = reinterpret_cast<float*>(smem + P.off_wt);
    unsigned ph_gu = 0, ph_dn = 0, ph_wt = 0;

    // ---- prologue: residual rows, router slice of layer 0, partial router sums ------------------
    for (int r = tid; r < nr; r += blockDim.x) xs[r] = to_f32<R>(x[d0 + r]);
    int wn_sub = 0;
    {
        const LayerWeights& L0 = a.lw[0];
        if (tid == 0) {
            const unsigned wt_bytes = (unsigned)((int64_t)nr * E * 4);
            const int64_t wn_lo = ((int64_t)d0 * 4) & ~(int64_t)15;
            const int64_t wn_hi = a16((int64_t)d1 * 4);
            mbar_expect_tx(bar_wt, wt_bytes + (unsigned)(wn_hi - wn_lo));
            bulk_g2s(wt, L0.w_router_t + (int64_t)d0 * E, wt_bytes, bar_wt);
            bulk_g2s(smem + P.off_wn, reinterpret_cast<const uint8_t*>(L0.w_norm) + wn_lo, (unsigned)(wn_hi - wn_lo),
                     bar_wt);
        }
        wn_sub = (int)(((int64_t)d0 * 4) & 15) / 4;
        if (!mbar_wait(bar_wt, ph_wt)) { atomicOr(&a.sync[0], 2u); alive = false; }
        ph_wt ^= 1;
        __syncthreads();
        const float* wn = reinterpret_cast<const float*>(smem + P.off_wn) + wn_sub;
        double* acc = a.racc;                       // buffer 0
        for (int e = tid; e <= E; e += blockDim.x) {
            double s = 0.0;
            if (e < E) {
                for (int r = 0; r < nr; ++r) s += (double)wt[r * E + e] * (double)(wn[r] * xs[r]);
            } else {
                for (int r = 0; r < nr; ++r) s += (double)(xs[r] * xs[r]);
            }
            if (alive) atomicAdd(&acc[e], s);
        }
    }
    if (!grid_barrier(a.sync, nbar++, &s_ok)) alive = false;

    for (int l = 0; l < a.n_layers; ++l) {
        const LayerWeights& L = a.lw[l];
        const int buf = l & 1;
        P.init(H, E, k, I, L.down_type, G);
        // ---- A. routing ------------------------------------------------------------------------
        float* lg = reinterpret_cast<float*>(smem + P.off_lg);
        const double* racc = a.racc + (int64_t)buf * (E + 1);
        if (tid == 0) {
            const double ss = ld_f64(&racc[E]);
            const float mean = (float)(ss / H);
            s_scale = 1.0f / sqrtf(mean + a.eps);
        }
        __syncthreads();
        const float scale = s_scale;
        for (int e = tid; e < E; e += blockDim.x) lg[e] = (float)((double)scale * ld_f64(&racc[e]));
        __syncthreads();
        int32_t* sel_o = a.sel_out ? a.sel_out + (int64_t)l * k : nullptr;
        float* w_o = a.w_out ? a.w_out + (int64_t)l * k : nullptr;
        {
            // softmax + top-k into shared s_sel/s_w (thread 0 also writes the caller's outputs)
            __shared__ int32_t t_sel[16];
            __shared__ float t_w[16];
            softmax_topk(lg, E, k, a.renorm, t_sel, t_w, redd, redf, s_sel, s_w);
            if (tid < k) {
                s_sel[tid] = t_sel[tid];
                s_w[tid] = t_w[tid];
                if (c == 0 && sel_o) { sel_o[tid] = t_sel[tid]; w_o[tid] = t_w[tid]; }
            }
            __syncthreads();
        }
        // ---- B. issue this CTA's weight copies for the whole layer ---------------------------------
        // (every CTA issues or skips as a whole: `alive` is uniform inside a CTA)
        const bool issued = alive;
        const bool issued_wt = alive && (l + 1 < a.n_layers);
        if (tid == 0 && alive) {
            fence_proxy_async();
            // gate/up row pairs [q0, q1), split at expert boundaries
            unsigned gu_bytes = (unsigned)(2 * (int64_t)np * (P.gu_row_qs + P.gu_row_hdr));
            mbar_expect_tx(bar_gu, gu_bytes);
            const int64_t nblk_gu = (int64_t)I * nbH;
            for (int q = q0; q < q1;) {
                const int j = q / I, i = q - j * I;
                const int qe = min(q1, (j + 1) * I);
                const int n = qe - q;
                const uint8_t* base = L.pool + (int64_t)s_sel[j] * L.slot_stride;
                const int64_t p = q - q0;
                bulk_g2s(smem + P.off_gate_qs + p * P.gu_row_qs, base + (int64_t)i * P.gu_row_qs,
                         (unsigned)(n * P.gu_row_qs), bar_gu);
                bulk_g2s(smem + P.off_gate_hdr + p * P.gu_row_hdr, base + nblk_gu * 128 + (int64_t)i * P.gu_row_hdr,
                         (unsigned)(n * P.gu_row_hdr), bar_gu);
                const uint8_t* ub = base + L.off_up;
                bulk_g2s(smem + P.off_up_qs + p * P.gu_row_qs, ub + (int64_t)i * P.gu_row_qs,
                         (unsigned)(n * P.gu_row_qs), bar_gu);
                bulk_g2s(smem + P.off_up_hdr + p * P.gu_row_hdr, ub + nblk_gu * 128 + (int64_t)i * P.gu_row_hdr,
                         (unsigned)(n * P.gu_row_hdr), bar_gu);
                q = qe;
            }
            // down rows [d0, d1) of every selected expert
            const int64_t nblk_dn = (int64_t)H * nbI;
            unsigned dn_bytes = 0;
            int64_t plane_off[4], plane_row[4];
            int nplanes;
            if (P.dt == T_Q4K) {
                nplanes = 2;
                plane_off[0] = 0; plane_row[0] = (int64_t)nbI * 128;
                plane_off[1] = nblk_dn * 128; plane_row[1] = (int64_t)nbI * 16;
            } else {
                nplanes = 4;
                plane_off[0] = 0; plane_row[0] = (int64_t)nbI * 128;
                plane_off[1] = nblk_dn * 128; plane_row[1] = (int64_t)nbI * 64;
                plane_off[2] = nblk_dn * 192; plane_row[2] = (int64_t)nbI * 16;
                plane_off[3] = nblk_dn * 208; plane_row[3] = (int64_t)nbI * 2;
            }
            const int64_t dst_off[4] = {P.dn_p0, P.dn_p1, P.dn_p2, P.dn_p3};
            for (int pl = 0; pl < nplanes; ++pl) {
                const int64_t lo = plane_off[pl] + (int64_t)d0 * plane_row[pl];
                const int64_t hi = plane_off[pl] + (int64_t)d1 * plane_row[pl];
                const int64_t alo = lo & ~(int64_t)15, ahi = a16(hi);
                dn_bytes += (unsigned)(k * (ahi - alo));
            }
            mbar_expect_tx(bar_dn, dn_bytes);
            for (int j = 0; j < k; ++j) {
                const uint8_t* base = L.pool + (int64_t)s_sel[j] * L.slot_stride + L.off_down;
                uint8_t* reg = smem + P.off_dn + (int64_t)j * P.dn_stride;
                for (int pl = 0; pl < nplanes; ++pl) {
                    const int64_t lo = plane_off[pl] + (int64_t)d0 * plane_row[pl];
                    const int64_t hi = plane_off[pl] + (int64_t)d1 * plane_row[pl];
                    const int64_t alo = lo & ~(int64_t)15, ahi = a16(hi);
                    bulk_g2s(reg + dst_off[pl], base + alo, (unsigned)(ahi - alo), bar_dn);
                }
            }
            // router slice of the next layer
            if (l + 1 < a.n_layers) {
                const LayerWeights& Ln = a.lw[l + 1];
                const unsigned wt_bytes = (unsigned)((int64_t)nr * E * 4);
                const int64_t wn_lo = ((int64_t)d0 * 4) & ~(int64_t)15;
                const int64_t wn_hi = a16((int64_t)d1 * 4);
                mbar_expect_tx(bar_wt, wt_bytes + (unsigned)(wn_hi - wn_lo));
                bulk_g2s(wt, Ln.w_router_t + (int64_t)d0 * E, wt_bytes, bar_wt);
                bulk_g2s(smem + P.off_wn, reinterpret_cast<const uint8_t*>(Ln.w_norm) + wn_lo,
                         (unsigned)(wn_hi - wn_lo), bar_wt);
            }
        }
        // ---- A'. fx = rms_norm(x) * ffn_norm -> Q8_K in shared memory ------------------------------
        {
            int8_t* fxq = reinterpret_cast<int8_t*>(smem + P.off_fxq);
            float* fxd = reinterpret_cast<float*>(smem + P.off_fxd);
            int* fxbs = reinterpret_cast<int*>(smem + P.off_fxbs);
            const int ng = H / 16;
            for (int g0 = 0; g0 < ng; g0 += blockDim.x) {   // groups of 16; a 256-block = 16 groups
                const int g = g0 + tid;
                float v[16];
                float am = 0.f;
                if (g < ng) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int dd = 16 * g + i;
                        const float xr = ld_resid(x + dd);
                        v[i] = (xr * scale) * __ldg(L.w_norm + dd);
                        am = fmaxf(am, fabsf(v[i]));
                    }
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                if (g < ng) {
                    int bs = 0;
                    float iscale = am != 0.f ? 127.f / am : 0.f;
                    uint32_t packed[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int q = am != 0.f ? min(127, __float2int_rn(iscale * v[i])) : 0;
                        bs += q;
                        packed[i >> 2] |= ((uint32_t)(q & 0xFF)) << (8 * (i & 3));
                    }
                    *reinterpret_cast<uint4*>(fxq + 16 * g) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    fxbs[g] = bs;
                    if ((g & 15) == 0) fxd[g >> 4] = am != 0.f ? 1.f / iscale : 0.f;
                }
            }
        }
        __syncthreads();
        // ---- C. gate/up + SwiGLU -------------------------------------------------------------------
        if (issued && !mbar_wait(bar_gu, ph_gu)) { atomicOr(&a.sync[0], 2u); alive = false; }
        ph_gu ^= 1;
        const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
        unsigned* amax = a.amax + (int64_t)buf * k * nbI;
        if (alive) {
            const int8_t* fxq = reinterpret_cast<const int8_t*>(smem + P.off_fxq);
            const float* fxd = reinterpret_cast<const float*>(smem + P.off_fxd);
            const int* fxbs = reinterpret_cast<const int*>(smem + P.off_fxbs);
            const int nunits = nbH * 8;
            for (int p = warp; p < np; p += nw) {
                const int q = q0 + p, j = q / I, i = q - j * I;
                float g = 0.f, u = 0.f;
                for (int un = lane; un < nunits; un += 32) {
                    const int b = un >> 3, c8 = un & 7;
                    const uint4 wg = *reinterpret_cast<const uint4*>(smem + P.off_gate_qs + p * P.gu_row_qs + 16 * un);
                    const uint4 hg = *reinterpret_cast<const uint4*>(smem + P.off_gate_hdr + p * P.gu_row_hdr + 16 * b);
                    const uint4 wu = *reinterpret_cast<const uint4*>(smem + P.off_up_qs + p * P.gu_row_qs + 16 * un);
                    const uint4 hu = *reinterpret_cast<const uint4*>(smem + P.off_up_hdr + p * P.gu_row_hdr + 16 * b);
                    g += q4k_unit_dot(wg, hg, c8, fxq + QK * b, fxbs + 16 * b, fxd[b]);
                    u += q4k_unit_dot(wu, hu, c8, fxq + QK * b, fxbs + 16 * b, fxd[b]);
                }
                g = warp_sum(g);
                u = warp_sum(u);
                if (lane == 0) {
                    const float hv = silu_f(g) * u;
                    a.h[(int64_t)j * I + i] = hv;
                    atomicMax(&amax[j * nbI + (i >> 8)], __float_as_uint(fabsf(hv)));
                }
            }
        }
        if (!grid_barrier(a.sync, nbar++, &s_ok)) alive = false;
        // ---- D. down + combine -------------------------------------------------------------------
        if (c == 0 && alive) {
            double* rz = a.racc + (int64_t)buf * (E + 1);
            for (int e = tid; e <= E; e += blockDim.x) rz[e] = 0.0;
            unsigned* az = a.amax + (int64_t)(buf ^ 1) * k * nbI;
            for (int e = tid; e < k * nbI; e += blockDim.x) az[e] = 0u;
        }
        {
            int8_t* hq = reinterpret_cast<int8_t*>(smem + P.off_hq);
            float* hd = reinterpret_cast<float*>(smem + P.off_hd);
            int* hbs = reinterpret_cast<int*>(smem + P.off_hbs);
            const int ng = k * I / 16;
            for (int g = tid; g < ng; g += blockDim.x) {
                const int e0 = 16 * g;
                const int j = e0 / I, blk = (e0 - j * I) >> 8;
                const float am = __uint_as_float(ld_relaxed(&amax[j * nbI + blk]));
                const float iscale = am != 0.f ? 127.f / am : 0.f;
                int bs = 0;
                uint32_t packed[4] = {0, 0, 0, 0};
                float hv16[16];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 t4 = ld_f32x4(a.h + e0 + 4 * i);
                    hv16[4 * i] = t4.x; hv16[4 * i + 1] = t4.y; hv16[4 * i + 2] = t4.z; hv16[4 * i + 3] = t4.w;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float hv = hv16[i];
                    const int q = am != 0.f ? min(127, __float2int_rn(iscale * hv)) : 0;
                    bs += q;
                    packed[i >> 2] |= ((uint32_t)(q & 0xFF)) << (8 * (i & 3));
                }
                *reinterpret_cast<uint4*>(hq + e0) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                hbs[g] = bs;
                if (((e0 - j * I) & 255) == 0) hd[j * nbI + blk] = am != 0.f ? 1.f / iscale : 0.f;
            }
        }
        __syncthreads();
        // offset of row d0 inside the 16-byte-aligned copy of the fp16 d plane (Q6_K only)
        const int dsub = P.dt == T_Q6K ? (int)(((int64_t)d0 * nbI * 2) & 15) : 0;
        if (issued && !mbar_wait(bar_dn, ph_dn)) { atomicOr(&a.sync[0], 2u); alive = false; }
        ph_dn ^= 1;
        if (alive) {
            if (P.dt == T_Q4K) down_phase<T_Q4K>(P, smem, nr, k, dsub);
            else down_phase<T_Q6K>(P, smem, nr, k, dsub);
        }
        __syncthreads();
        const float* y = reinterpret_cast<const float*>(smem + P.off_y);
        for (int r = tid; r < nr; r += blockDim.x) {
            float acc = 0.f;
            for (int j = 0; j < k; ++j) acc += s_w[j] * y[r * k + j];
            const R xn = from_f32<R>(acc + xs[r]);
            if (alive) x[d0 + r] = xn;
            xs[r] = to_f32<R>(xn);
        }
        if (l + 1 < a.n_layers) {
            if (issued_wt && !mbar_wait(bar_wt, ph_wt)) { atomicOr(&a.sync[0], 2u); alive = false; }
            ph_wt ^= 1;
            __syncthreads();
            const float* wn = reinterpret_cast<const float*>(smem + P.off_wn) + wn_sub;
            double* acc = a.racc + (int64_t)(buf ^ 1) * (E + 1);
            for (int e = tid; e <= E; e += blockDim.x) {
                double s = 0.0;
                if (e < E) {
                    for (int r = 0; r < nr; ++r) s += (double)wt[r * E + e] * (double)(wn[r] * xs[r]);
                } else {
                    for (int r = 0; r < nr; ++r) s += (double)(xs[r] * xs[r]);
                }
                if (alive) atomicAdd(&acc[e], s);
            }
            if (!grid_barrier(a.sync, nbar++, &s_ok)) alive = false;
        }
    }
    // ---- exit: the last CTA out restores the zero state of the counters and max buffers --------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.sync[2], 1u);
        if (old == (unsigned)G - 1) {
            __threadfence();
            unsigned* az = a.amax + (int64_t)((a.n_layers - 1) & 1) * k * nbI;
            for (int e = 0; e < k * nbI; ++e) az[e] = 0u;
            double* rz = a.racc + (int64_t)(a.n_layers & 1) * (E + 1);
            for (int e = 0; e <= E; ++e) rz[e] = 0.0;
            a.sync[1] = 0u;
            a.sync[2] = 0u;
            __threadfence();
        }
    }
}

int decode_max_tokens() { return 1; }

static int g_num_sms = 0;

bool decode_supported(const Dims& d, const LayerWeights* lws, int n_layers) {
    if (d.k > 16 || d.E % 4 != 0 || d.E > 1024) return false;
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_num_sms == 0) cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int G = g_num_sms;
    if ((int64_t)d.k * d.I < G || d.H < G) return false;   // every CTA must own rows
    for (int l = 0; l < n_layers; ++l) {
        const LayerWeights& L = lws[l];
        if (L.gate_type != T_Q4K || L.up_type != T_Q4K) return false;
        if (L.down_type != T_Q4K && L.down_type != T_Q6K) return false;
        if (L.shared) return false;
        DecodePlan P;
        P.init(d.H, d.E, d.k, d.I, L.down_type, G);
        if (P.total + 2048 > max_smem) return false;
    }
    return true;
}

cudaError_t launch_decode_persistent(const Dims& d, const LayerWeights* lws_dev, int n_layers, const Scratch& sc,
                                     void* x_inout, int T, int32_t* sel_out, float* w_out, cudaStream_t s,
                                     int* /*unused*/) {
    if (T != 1) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_num_sms == 0) cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    const int G = g_num_sms;
    int64_t smem = 0;
    for (int dt : {(int)T_Q4K, (int)T_Q6K}) {
        DecodePlan P;
        P.init(d.H, d.E, d.k, d.I, dt, G);
        smem = smem > P.total ? smem : P.total;
    }
    DecodeArgs a;
    a.lw = lws_dev;
    a.n_layers = n_layers;
    a.H = d.H; a.E = d.E; a.k = d.k; a.I = d.I; a.renorm = d.renorm; a.eps = d.eps; a.resid_bf16 = d.resid_bf16;
    a.x = x_inout;
    a.sel_out = sel_out;
    a.w_out = w_out;
    a.h = sc.h;
    a.amax = sc.amax;
    a.racc = reinterpret_cast<double*>(sc.partials);
    a.sync = sc.sync;
    void* args[] = {&a};
    cudaError_t e;
    if (d.resid_bf16) {
        e = cudaFuncSetAttribute(k_decode<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        e = cudaLaunchCooperativeKernel((const void*)k_decode<__nv_bfloat16>, dim3(G), dim3(DEC_THREADS), args,
                                        (size_t)smem, s);
    } else {
        e = cudaFuncSetAttribute(k_decode<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        e = cudaLaunchCooperativeKernel((const void*)k_decode<float>, dim3(G), dim3(DEC_THREADS), args, (size_t)smem,
                                        s);
    }
    return e;
}

}  // namespace hoard
