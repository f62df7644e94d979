// kernels_decode.cu -- persistent fused decode kernel: T = 1, every expert resident, any number of
// consecutive layers in one cooperative launch (one CTA per SM).
//
// Per layer l (hoard's graph A router tail + graph B + host combine, src/run_moe_stream.cpp:352-447):
//   A  every CTA reads the router sums of layer l (accumulated by all CTAs at the end of layer l-1),
//      runs softmax + top-k itself (identical arithmetic in every CTA) while its other warps build
//      the Q8_K activation of fx = rms_norm(x) * ffn_norm in shared memory;
//   B  warp 0 issues cp.async.bulk copies of this CTA's share of the selected experts' bytes
//      (gate/up row pairs in four chunks, and the down rows) plus the next layer's router slice, all
//      at once, so the whole layer's weight bytes are in flight while the CTA computes;
//   C  gate/up row pairs from shared memory as each chunk lands: h = silu(gate . fx) * (up . fx) to
//      global, plus a per-256-block max|h| (the Q8_K scale of h) by atomicMax;
//      ---- grid barrier ----
//   D  Q8_K of h in shared memory; this CTA's output rows for every selected expert; the combine
//      x[d] = sum_j w_j*y_j[d] + x[d] (j ascending); then the next layer's router partial sums over
//      these rows (sum x^2 and W_r^T[d,:] . (ffn_norm[d]*x[d])), each formed in double in row order,
//      divided by the layer's norm and added as 2^-40 fixed point into int64 accumulators: integer
//      adds commute, so the sums -- and the routing -- are bit-reproducible whatever order the
//      CTAs arrive in;
//      ---- grid barrier ----
// Matmul mapping: one lane owns one 256-weight block of a row (its scales are decoded once), lanes
// read the block's 16-byte chunks in a lane-rotated order so that a warp's shared-memory reads hit
// distinct banks, and the integer dot of each chunk is exact (dp4a).
// Every wait (grid barrier, mbarrier) is bounded by %globaltimer; on expiry the kernel sets
// bit 2 of the error word, stops computing, drains its own copies (bounded) and exits.
#include "common.cuh"
#include "kernels.h"
#include "block_ops.cuh"
#include "async_copy.cuh"


namespace hoard {

static int g_num_sms = 0;

namespace {

constexpr int DEC_THREADS = 512;
constexpr int DEC_TRACE_PHASES = 20;
constexpr int NCH = 4;                                   // gate/up arrival chunks
constexpr double RFIX = 1099511627776.0;      // 2^40: unit of a normalised router partial sum
constexpr double RFIX_MAX = 4.0e18;           // |partial| * 2^40 beyond this sets error bit 4
constexpr int RACC_COPIES = 4;   // router accumulators spread over copies (4 measured best of 1, 2, 4, 8, 16)
constexpr int HREADY_OFF = 64;         // h block readiness counters: sync word HREADY_OFF + HREADY_STRIDE * b
constexpr int HREADY_STRIDE = 32;      // one 128-byte line per counter (pollers of different blocks do not share)

__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Loads of data produced earlier in this launch by other CTAs go through L2 only (ld.global.cg):
// L2 is the point of coherence, and the grid barrier's acquire fence orders them after the
// producers' writes. They are ordinary loads, so the compiler can issue them back to back.
__device__ __forceinline__ float4 ld_resid4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld_resid4(const __nv_bfloat16* p) {
    const unsigned short* q = reinterpret_cast<const unsigned short*>(p);
    return make_float4(__bfloat162float(__ushort_as_bfloat16(__ldcg(q))),
                       __bfloat162float(__ushort_as_bfloat16(__ldcg(q + 1))),
                       __bfloat162float(__ushort_as_bfloat16(__ldcg(q + 2))),
                       __bfloat162float(__ushort_as_bfloat16(__ldcg(q + 3))));
}

// Grid barrier number `n` (0, 1, 2, ... within this launch): arrive by a release add, poll with
// acquire loads (no separate gpu-scope fences: measured 0.9 us per layer less than fence + relaxed
// add / relaxed polls + fence). Returns false on timeout / error.
// It is driven by the last warp, which issues no bulk copies, so that its release does not wait on
// weight copies still in flight.
__device__ bool grid_barrier(unsigned* sync, unsigned n, int* s_ok, unsigned long long* st = nullptr) {
    __syncthreads();
    if (threadIdx.x == blockDim.x - 32) {
        int ok = 1;
        const unsigned target = (n + 1) * gridDim.x;
        if (st) st[0] = gtimer();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&sync[1]) : "memory");
        if (ld_acq(&sync[1]) < target) {
            const unsigned long long t0 = gtimer();
            for (unsigned it = 1;; ++it) {
                if (ld_acq(&sync[1]) >= target) break;
                if ((it & 15) == 0) {
                    if (ld_relaxed(&sync[0]) & 2u) { ok = 0; break; }
                    if (gtimer() - t0 > WAIT_NS) { atomicOr(&sync[0], 2u); ok = 0; break; }
                }
            }
        }
        if (st) st[1] = gtimer();
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Bounded wait until the counter reaches `target` (acquire polls); false if the bound expired or
// another CTA has given up.
__device__ bool wait_count(const unsigned* cnt, unsigned target, unsigned* sync) {
    if ((int)(ld_acq(cnt) - target) < 0) {
        const unsigned long long t0 = gtimer();
        for (unsigned it = 1;; ++it) {
            __nanosleep(64);
            if ((int)(ld_acq(cnt) - target) >= 0) break;
            if ((it & 15) == 0) {
                if (ld_relaxed(&sync[0]) & 2u) return false;
                if (gtimer() - t0 > WAIT_NS) { atomicOr(&sync[0], 2u); return false; }
            }
        }
    }
    return true;
}

inline __host__ __device__ int64_t a16(int64_t v) { return (v + 15) & ~(int64_t)15; }

// Q8_K activations in shared memory are padded so that lanes reading the same offset of different
// 256-value blocks (stride 272 B) or of different experts (stride = odd multiple of 16 B mod 128)
// land in different banks.
constexpr int ACT_BLK = 272;
inline __host__ __device__ int hq_stride(int nbI) {
    const int s = nbI * ACT_BLK;
    return ((s / 16) & 1) ? s : s + 16;
}

__device__ __forceinline__ void named_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// unsigned bytes of a . signed bytes of b, accumulated into c
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int sext8(unsigned x) { return (int)(signed char)(x & 0xFFu); }
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ int4 lds128i(const void* p) { return *reinterpret_cast<const int4*>(p); }

// The 6-bit scales and mins of a Q4_K block header, unpacked four per register (one byte each):
// sc[0..3], sc[4..7], m[0..3], m[4..7] (GGUF packing: bytes 0..3 low 6 bits = sc[0..3], bytes 4..7
// = m[0..3]; bytes 8..11 low/high nibbles = low 4 bits of sc[4..7]/m[4..7], whose top 2 bits are
// the top 2 bits of bytes 0..3 / 4..7).
struct Q4Scales {
    uint32_t sc_lo, sc_hi, m_lo, m_hi;
};
__device__ __forceinline__ Q4Scales q4_scales(const uint4& h) {
    Q4Scales s;
    s.sc_lo = h.y & 0x3F3F3F3Fu;
    s.m_lo = h.z & 0x3F3F3F3Fu;
    s.sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    s.m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    return s;
}
__device__ __forceinline__ int byte_of(uint32_t lo, uint32_t hi, int j) {   // byte j (0..7) of (lo, hi)
    return (int)(((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xFFu);
}

// Exact integer parts of one 16-byte Q4_K chunk c (0..7) of a block against the activation block:
// low nibbles belong to sub-block 2g, high nibbles to 2g+1 (g = c/2); returns sc0*dot_lo + sc1*dot_hi.
__device__ __forceinline__ int q4_chunk(const uint4& w, const int4& alo, const int4& ahi, int sc0, int sc1) {
    int lo = __dp4a((int)(w.x & 0x0F0F0F0Fu), alo.x, 0);
    lo = __dp4a((int)(w.y & 0x0F0F0F0Fu), alo.y, lo);
    lo = __dp4a((int)(w.z & 0x0F0F0F0Fu), alo.z, lo);
    lo = __dp4a((int)(w.w & 0x0F0F0F0Fu), alo.w, lo);
    int hi = dp4a_us(w.x & 0xF0F0F0F0u, ahi.x, 0);
    hi = dp4a_us(w.y & 0xF0F0F0F0u, ahi.y, hi);
    hi = dp4a_us(w.z & 0xF0F0F0F0u, ahi.z, hi);
    hi = dp4a_us(w.w & 0xF0F0F0F0u, ahi.w, hi);
    return sc0 * lo + sc1 * (hi >> 4);
}

// sum_j m_j * bs32_j over the 8 sub-blocks (the dmin part of a Q4_K block dot)
__device__ __forceinline__ int q4_min_dot(const Q4Scales& s, const int* bs32) {
    const int4 b0 = lds128i(bs32), b1 = lds128i(bs32 + 4);
    return (int)(s.m_lo & 0xFF) * b0.x + (int)((s.m_lo >> 8) & 0xFF) * b0.y + (int)((s.m_lo >> 16) & 0xFF) * b0.z +
           (int)(s.m_lo >> 24) * b0.w + (int)(s.m_hi & 0xFF) * b1.x + (int)((s.m_hi >> 8) & 0xFF) * b1.y +
           (int)((s.m_hi >> 16) & 0xFF) * b1.z + (int)(s.m_hi >> 24) * b1.w;
}

// Adds one CTA's router partial sum s (formed in double) into a fixed-point accumulator: s * fix
// rounded to an integer (fix = 2^40 / the layer's norm, or / its square for sum x^2). Out-of-range
// values set error bit 4 instead.
__device__ __forceinline__ void add_fixed(long long* acc, double s, double fix, unsigned* sync) {
    const double v = s * fix;
    if (fabs(v) < RFIX_MAX)
        atomicAdd(reinterpret_cast<unsigned long long*>(acc), (unsigned long long)__double2ll_rn(v));
    else
        atomicOr(&sync[0], 4u);
}

// Warp 0's router tail for E <= 32*NV, in two parts so that the expert copies can be issued between
// them. route_select: logits -> top-k. The logits are selected in descending order (ties to the
// lower expert id): softmax is monotonic, so this is the order of the probabilities except where
// two different logits round to the same probability (a tie far below any parity tolerance). Each
// lane sorts its NV logits once; every round takes the warp-wide maximum of the lanes' heads (keys
// are order-preserving unsigned images of the floats) and, among equal keys, the lowest expert id.
// Lanes < k leave expert id and logit of rank `lane` in s_sel and *my_logit.
template <int NV>
__device__ __forceinline__ void route_select(const double* s_lgd, int E, int k, float scale, int lane, int* s_sel,
                                             float* my_logit) {
    unsigned key[NV], idx[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int e = lane + 32 * i;
        const float p = e < E ? (float)((double)scale * s_lgd[e]) : 0.f;
        const unsigned u = __float_as_uint(p);
        key[i] = e < E ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;
        idx[i] = (unsigned)e;
    }
#pragma unroll
    for (int i = 1; i < NV; ++i) {
#pragma unroll
        for (int j = i; j > 0; --j) {
            const bool sw = key[j] > key[j - 1] || (key[j] == key[j - 1] && idx[j] < idx[j - 1]);
            const unsigned k0 = key[j - 1], i0 = idx[j - 1];
            key[j - 1] = sw ? key[j] : k0;
            idx[j - 1] = sw ? idx[j] : i0;
            key[j] = sw ? k0 : key[j];
            idx[j] = sw ? i0 : idx[j];
        }
    }
    int my_sel = 0;
    unsigned my_key = 0;
    for (int r = 0; r < k; ++r) {
        const unsigned M = __reduce_max_sync(0xFFFFFFFFu, key[0]);
        const unsigned W = __reduce_min_sync(0xFFFFFFFFu, key[0] == M ? idx[0] : 0xFFFFFFFFu);
        if (key[0] == M && idx[0] == W) {
#pragma unroll
            for (int i = 0; i + 1 < NV; ++i) { key[i] = key[i + 1]; idx[i] = idx[i + 1]; }
            key[NV - 1] = 0u;
        }
        if (lane == r) { my_sel = (int)W; my_key = M; }
    }
    if (lane < k) s_sel[lane] = my_sel;
    const unsigned u = (my_key & 0x80000000u) ? (my_key & 0x7FFFFFFFu) : ~my_key;
    *my_logit = __uint_as_float(u);
}

// route_weights: softmax over all E (max subtracted, double sum, as ggml's soft_max) evaluated at
// the selected logits, then the optional renormalisation with clamp (sum in rank order, as hoard's
// host loop). Lanes < k leave the weight of rank `lane` in s_w (and sel_out / w_out).
template <int NV>
__device__ __forceinline__ void route_weights(const double* s_lgd, int E, int k, int renorm, float scale, int lane,
                                              float my_logit, const int* s_sel, float* s_w, int32_t* sel_out,
                                              float* w_out) {
    float p[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) p[i] = lane + 32 * i < E ? (float)((double)scale * s_lgd[lane + 32 * i]) : -INFINITY;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) mx = fmaxf(mx, p[i]);
    mx = warp_max(mx);
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (lane + 32 * i < E) sum += (double)expf(p[i] - mx);
    sum = warp_sum(sum);
    const float inv = (float)(1.0 / sum);
    float my_w = lane < k ? expf(my_logit - mx) * inv : 0.f;
    float wsum = 0.f;
    for (int r = 0; r < k; ++r) wsum += __shfl_sync(0xFFFFFFFFu, my_w, r);
    if (renorm) {
        if (wsum < 6.103515625e-5f) wsum = 6.103515625e-5f;
        my_w /= wsum;
    }
    if (lane < k) {
        s_w[lane] = my_w;
        if (sel_out) { sel_out[lane] = s_sel[lane]; w_out[lane] = my_w; }
    }
}

}  // namespace

// Shared-memory plan; identical on host (sizing) and device (offsets). Sized for the largest
// share of any CTA: ceil(k*I/G) gate/up row pairs and ceil(H/G) output rows. k counts the expert
// positions of a token: the routed experts, plus the shared expert where the model has one.
struct DecodePlan {
    int H, E, k, I, nbH, nbI, dt;
    int np_max, nr_max;
    int64_t gu_row_qs, gu_row_hdr;          // bytes per gate/up row in the two Q4_K planes
    int64_t off_gate_qs, off_gate_hdr, off_up_qs, off_up_hdr;
    int64_t dn_stride;                      // bytes of one expert's down rows (all planes)
    int64_t dn_p0, dn_p1, dn_p2, dn_p3;     // plane offsets inside an expert's down region
    int64_t off_dn, off_wt, off_wn, off_gs, off_fxq, off_fxd, off_fxbs32, off_hq, off_hd, off_hbs, off_y, off_xs,
        off_misc, total;

    // alias: the down rows go to the start of the gate/up region (issued once the CTA's gate/up rows
    // are consumed) when both shares do not fit in shared memory together
    __host__ __device__ void init(int H_, int E_, int k_, int I_, int dt_, int G, int alias = 0) {
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
        if (alias) {
            off_dn = off_gate_qs;
            o = o > off_dn + (int64_t)k * dn_stride ? o : off_dn + (int64_t)k * dn_stride;
        } else {
            off_dn = o; o += (int64_t)k * dn_stride;
        }
        off_wt = o; o += a16((int64_t)nr_max * E * 4) + 16;
        off_wn = o; o += a16((int64_t)nr_max * 4) + 32;
        off_gs = o; o += a16((int64_t)nr_max * 4) + 32;     // the shared expert's gate-input slice
        off_fxq = o; o += (int64_t)nbH * ACT_BLK + 16;

        off_fxd = o; o += a16((int64_t)nbH * 4);
        off_fxbs32 = o; o += a16((int64_t)(H / 32) * 4);
        off_hq = o; o += (int64_t)k * hq_stride(nbI) + 16;
        off_hd = o; o += a16((int64_t)k * nbI * 4);
        off_hbs = o; o += a16((int64_t)k * (I / 16) * 4);   // Q6_K: 16-sums in unit order; Q4_K: 32-sums
        off_y = o; o += a16((int64_t)nr_max * k * 4);
        off_xs = o; o += a16((int64_t)nr_max * 4);
        off_misc = o; o += 128;                  // mbarriers
        total = o;
    }
};

// plane offsets (qs/ql, hdr/qh, sc, d) inside a position's staged down region for type dt
__host__ __device__ inline void dn_planes(int dt, int nr_max, int nbI, int64_t* p1, int64_t* p2, int64_t* p3) {
    const int64_t rq = (int64_t)nbI * 128;
    if (dt == T_Q4K) {
        *p1 = a16(nr_max * rq) + 16;
        *p2 = *p3 = 0;
    } else {
        *p1 = a16(nr_max * rq) + 16;
        *p2 = *p1 + a16(nr_max * (int64_t)nbI * 64) + 16;
        *p3 = *p2 + a16(nr_max * (int64_t)nbI * 16) + 16;
    }
}

struct DecodeArgs {
    const LayerWeights* lw;     // [n_layers] (device)
    int n_layers;
    int H, E, k, I, renorm;
    int KK;                     // expert positions: k routed, plus the shared expert when KK = k + 1
    int sh_dt;                  // down type of the shared expert
    float eps;
    int resid_bf16;
    void* x;                    // [H] residual, f32 or bf16, updated in place
    int32_t* sel_out;           // [n_layers][k] or null
    float* w_out;
    float* h;                   // [k][I]
    unsigned* amax;             // [2][k][I/256]
    long long* racc;            // [2][RACC_COPIES][E+1] fixed-point router sums (zero at rest)
    unsigned* sync;             // [0] error bits, [1] barrier counter, [2] exit counter
    unsigned long long* trace;  // optional [G][n_layers][DEC_TRACE_PHASES] %globaltimer stamps
    int alias_dn;               // DecodePlan alias mode (down rows over the consumed gate/up rows)
};

// NV = router logits per lane (E <= 32 * NV): one instantiation per width keeps only the routing code
// the launch uses inside the layer loop (measured: 0.35 us per layer less than dispatching at run time)
// TRACE: the instantiation with phase stamps (launched only when a trace buffer is set)
template <typename R, int NV, bool TRACE>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_sel[16];
    __shared__ float s_w[16];              // routing weights; position k (the shared expert) its sigmoid gate
    __shared__ int s_ok;
    __shared__ int s_pos_ok[16];           // per expert position: its h blocks were seen ready
    __shared__ int4 s_cd_gu[32];           // gate/up copy descriptors: [NCH chunks][2 segments][4 planes]
    __shared__ int4 s_cd_dn[2][64];        // down copy descriptors per type (Q4_K, Q6_K): [position][planes]
    __shared__ unsigned s_gu_bytes[NCH];
    __shared__ unsigned s_amax[16 * 4];    // per (expert position, 256 block) max|h| of this CTA
    __shared__ double s_lgd[514];          // router sums: [E] logits/scale, [E] sum x^2, [E+1] shared gate

    const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int H = a.H, E = a.E, k = a.k, I = a.I, KK = a.KK;
    const int nbH = H / QK, nbI = I / QK;
    const int P_pairs = KK * I;
    const int q0 = (int)((int64_t)c * P_pairs / G), q1 = (int)((int64_t)(c + 1) * P_pairs / G);
    const int np = q1 - q0;
    const int d0 = (int)((int64_t)c * H / G), d1 = (int)((int64_t)(c + 1) * H / G);
    const int nr = d1 - d0;
    const int NA = E + 2;                   // accumulators per copy: logits, sum x^2, shared gate
    const int racc_stride = RACC_COPIES * NA;
    R* x = reinterpret_cast<R*>(a.x);
    unsigned* hready = a.sync + HREADY_OFF;   // readiness counter of block b of h at hready[HREADY_STRIDE * b]
    bool alive = true;
    unsigned nbar = 0;
#define DEC_TR(layer, ph)                                                                                  \
    do {                                                                                                   \
        if (TRACE && tid == 0)                                                                             \
            a.trace[((int64_t)c * a.n_layers + (layer)) * DEC_TRACE_PHASES + (ph)] = gtimer();            \
    } while (0)

#define DEC_TRP(layer, ph) \
    (TRACE ? a.trace + ((int64_t)c * a.n_layers + (layer)) * DEC_TRACE_PHASES + (ph) : nullptr)
    // gate/up row pairs are processed in groups of RPW pairs per warp (LPR lanes per row)
    const int LPR = nbH;                    // lanes per gate/up row: one per 256-weight block
    const int RPW = 32 / LPR;
    const int ngroups = (np + RPW - 1) / RPW;

    DecodePlan P;
    P.init(H, E, KK, I, a.lw[0].down_type, G, a.alias_dn);
    int64_t sh_p1 = 0, sh_p2 = 0, sh_p3 = 0;     // the shared position's plane offsets (its own down type)
    dn_planes(a.sh_dt, P.nr_max, nbI, &sh_p1, &sh_p2, &sh_p3);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_misc);
    uint64_t* bar_gu = bars;                // [NCH]
    uint64_t* bar_dn = bars + NCH;
    uint64_t* bar_wt = bars + NCH + 1;
    if (tid == 0) {
        for (int i = 0; i < NCH + 2; ++i) mbar_init(bars + i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    float* xs = reinterpret_cast<float*>(smem + P.off_xs);
    float* wt = reinterpret_cast<float*>(smem + P.off_wt);
    unsigned ph_gu = 0, ph_dn = 0, ph_wt = 0;
    const int wn_sub = (int)(((int64_t)d0 * 4) & 15) / 4;
    const int64_t wn_lo = ((int64_t)d0 * 4) & ~(int64_t)15, wn_hi = a16((int64_t)d1 * 4);
    const unsigned wt_bytes = (unsigned)((int64_t)nr * E * 4);
    // bytes of one position's down rows [d0, d1), per down type (16-byte supersets)
    unsigned dn_bytes_q4 = 0, dn_bytes_q6 = 0;
    {
        const int64_t nblk_dn = (int64_t)H * nbI;
        const int64_t q4_off[2] = {0, nblk_dn * 128}, q4_row[2] = {(int64_t)nbI * 128, (int64_t)nbI * 16};
        const int64_t q6_off[4] = {0, nblk_dn * 128, nblk_dn * 192, nblk_dn * 208};
        const int64_t q6_row[4] = {(int64_t)nbI * 128, (int64_t)nbI * 64, (int64_t)nbI * 16, (int64_t)nbI * 2};
        for (int pl = 0; pl < 2; ++pl)
            dn_bytes_q4 += (unsigned)(a16(q4_off[pl] + (int64_t)d1 * q4_row[pl]) -
                                      ((q4_off[pl] + (int64_t)d0 * q4_row[pl]) & ~(int64_t)15));
        for (int pl = 0; pl < 4; ++pl)
            dn_bytes_q6 += (unsigned)(a16(q6_off[pl] + (int64_t)d1 * q6_row[pl]) -
                                      ((q6_off[pl] + (int64_t)d0 * q6_row[pl]) & ~(int64_t)15));
    }
    const unsigned dn_bytes_sh = KK > k ? (a.sh_dt == T_Q4K ? dn_bytes_q4 : dn_bytes_q6) : 0u;

    // Copy descriptors of this CTA's share, fixed for the whole launch: {src offset lo, hi, smem
    // offset, meta = bytes | j << 20 | chunk << 25 | up << 28 | valid << 29}; gate/up sources are
    // relative to the slot base, down sources to the down matrix.
    if (warp == 0) {
        {
            const int ci = lane, ch = ci >> 3, sg = (ci >> 2) & 1, m = ci & 3;
            const int pa = min(np, (ch * ngroups / NCH) * RPW);
            const int pb = min(np, ((ch + 1) * ngroups / NCH) * RPW);
            int4 d = make_int4(0, 0, 0, 0);
            if (pa < pb) {
                const int j = (q0 + pa) / I + sg;
                const int qa = max(q0 + pa, j * I), qe = min(q0 + pb, (j + 1) * I);
                if (qa < qe && j < KK) {
                    const int i = qa - j * I, n = qe - qa;
                    const int64_t pp = qa - q0;
                    const int64_t nblk_gu = (int64_t)I * nbH;
                    const bool hdr = m & 1, up = m >> 1;
                    const int64_t src = hdr ? nblk_gu * 128 + (int64_t)i * P.gu_row_hdr : (int64_t)i * P.gu_row_qs;
                    const int64_t dst = (hdr ? (up ? P.off_up_hdr : P.off_gate_hdr) : (up ? P.off_up_qs : P.off_gate_qs)) +
                                        pp * (hdr ? P.gu_row_hdr : P.gu_row_qs);
                    const unsigned bytes = (unsigned)(n * (hdr ? P.gu_row_hdr : P.gu_row_qs));
                    d = make_int4((int)(unsigned)(src & 0xFFFFFFFF), (int)(unsigned)(src >> 32), (int)dst,
                                  (int)(bytes | ((unsigned)j << 20) | ((unsigned)ch << 25) | ((unsigned)up << 28) | (1u << 29)));
                }
            }
            s_cd_gu[ci] = d;
            if (lane < NCH) {
                const int qa = min(np, (lane * ngroups / NCH) * RPW), qb = min(np, ((lane + 1) * ngroups / NCH) * RPW);
                s_gu_bytes[lane] = (unsigned)(2 * (int64_t)(qb - qa) * (P.gu_row_qs + P.gu_row_hdr));
            }
        }
        const int64_t nblk_dn = (int64_t)H * nbI;
        for (int tsel = 0; tsel < 2; ++tsel) {
            DecodePlan Pt;
            Pt.init(H, E, KK, I, tsel == 0 ? T_Q4K : T_Q6K, G, a.alias_dn);
            const int nplanes = tsel == 0 ? 2 : 4;
            for (int ci = lane; ci < KK * nplanes; ci += 32) {
                const int j = ci / nplanes, pl = ci - j * nplanes;
                int64_t off, row, dst;
                if (pl == 0) { off = 0; row = (int64_t)nbI * 128; dst = Pt.dn_p0; }
                else if (tsel == 0) { off = nblk_dn * 128; row = (int64_t)nbI * 16; dst = Pt.dn_p1; }
                else if (pl == 1) { off = nblk_dn * 128; row = (int64_t)nbI * 64; dst = Pt.dn_p1; }
                else if (pl == 2) { off = nblk_dn * 192; row = (int64_t)nbI * 16; dst = Pt.dn_p2; }
                else { off = nblk_dn * 208; row = (int64_t)nbI * 2; dst = Pt.dn_p3; }
                const int64_t alo = (off + (int64_t)d0 * row) & ~(int64_t)15, ahi = a16(off + (int64_t)d1 * row);
                const int64_t so = Pt.off_dn + (int64_t)j * Pt.dn_stride + dst;
                s_cd_dn[tsel][ci] = make_int4((int)(unsigned)(alo & 0xFFFFFFFF), (int)(unsigned)(alo >> 32), (int)so,
                                              (int)((unsigned)(ahi - alo) | ((unsigned)j << 20) | (1u << 29)));
            }
        }
    }

    for (int i = tid; i < 16 * 4; i += blockDim.x) s_amax[i] = 0u;

    // ---- prologue: residual rows, router slice of layer 0, partial router sums ------------------
    for (int r = tid; r < nr; r += blockDim.x) xs[r] = to_f32<R>(x[d0 + r]);
    // the norm that scales layer 0's fixed-point sums: every CTA sums the squares of the whole input in
    // the same order, so all CTAs hold the same value
    double Sprev;
    {
        __shared__ double s_red[DEC_THREADS / 32];
        double sq = 0.0;
        for (int i = tid; i < H; i += blockDim.x) {
            const float v = to_f32<R>(x[i]);
            sq += (double)(v * v);
        }
        sq = warp_sum(sq);
        if (lane == 0) s_red[warp] = sq;
        __syncthreads();
        double t = 0.0;
        for (int w = 0; w < nw; ++w) t += s_red[w];
        Sprev = t > 0.0 ? sqrt(t) : 1.0;
    }
    if (tid == 0) {
        mbar_expect_tx(bar_wt, wt_bytes + (unsigned)(wn_hi - wn_lo) * (KK > k ? 2u : 1u));
        bulk_g2s(wt, a.lw[0].w_router_t + (int64_t)d0 * E, wt_bytes, bar_wt);
        bulk_g2s(smem + P.off_wn, reinterpret_cast<const uint8_t*>(a.lw[0].w_norm) + wn_lo, (unsigned)(wn_hi - wn_lo),
                 bar_wt);
        if (KK > k)
            bulk_g2s(smem + P.off_gs, reinterpret_cast<const uint8_t*>(a.lw[0].sh_gate_inp) + wn_lo,
                     (unsigned)(wn_hi - wn_lo), bar_wt);
    }
    if (!mbar_wait(bar_wt, ph_wt)) { atomicOr(&a.sync[0], 2u); alive = false; }
    ph_wt ^= 1;
    __syncthreads();
    {
        const float* wn = reinterpret_cast<const float*>(smem + P.off_wn) + wn_sub;
        const float* gs = reinterpret_cast<const float*>(smem + P.off_gs) + wn_sub;
        long long* acc = a.racc + (int64_t)(c % RACC_COPIES) * NA;
        for (int e = tid; e < NA; e += blockDim.x) {
            double s = 0.0;
            if (e < E) {
                for (int r = 0; r < nr; ++r) s += (double)wt[r * E + e] * (double)(wn[r] * xs[r]);
            } else if (e == E) {
                for (int r = 0; r < nr; ++r) s += (double)(xs[r] * xs[r]);
            } else if (KK > k) {
                for (int r = 0; r < nr; ++r) s += (double)gs[r] * (double)(wn[r] * xs[r]);
            }
            if (alive && (e <= E || KK > k)) add_fixed(&acc[e], s, e == E ? RFIX / (Sprev * Sprev) : RFIX / Sprev, a.sync);
        }
    }
    if (!grid_barrier(a.sync, nbar++, &s_ok)) alive = false;

    for (int l = 0; l < a.n_layers; ++l) {
        const int buf = l & 1;
        // this layer's and the next layer's descriptors (global loads overlap the router read)
        const uint8_t* L_pool = a.lw[l].pool;
        const int64_t L_stride = a.lw[l].slot_stride, L_off_up = a.lw[l].off_up, L_off_down = a.lw[l].off_down;
        const int L_dt = a.lw[l].down_type;
        const float* L_wnorm = a.lw[l].w_norm;
        const uint8_t* L_sh = a.lw[l].shared;
        const int64_t L_sh_up = a.lw[l].sh_off_up, L_sh_down = a.lw[l].sh_off_down;
        const bool has_next = l + 1 < a.n_layers;
        const float* Ln_wrt = has_next ? a.lw[l + 1].w_router_t : nullptr;
        const float* Ln_wnorm = has_next ? a.lw[l + 1].w_norm : nullptr;
        const float* Ln_gs = has_next && KK > k ? a.lw[l + 1].sh_gate_inp : nullptr;
        P.init(H, E, KK, I, L_dt, G, a.alias_dn);
        DEC_TR(l, 0);
        // ---- A/B. warp 0: router sums -> softmax -> top-k -> copies -> renorm, all in registers;
        //      warps 1..: fx = rms_norm(x) * ffn_norm -> Q8_K (named barriers, no CTA-wide sync) ------
        const bool issued = alive;
        const bool issued_wt = alive && has_next;
        auto issue_down = [&]() {                       // warp 0: this CTA's down rows of every expert position
            const int tsel = L_dt == T_Q4K ? 0 : 1;
            const int np_l = L_dt == T_Q4K ? 2 : 4;
            for (int ci = lane; ci < k * np_l; ci += 32) {
                const int4 d = s_cd_dn[tsel][ci];
                const unsigned meta = (unsigned)d.w;
                const int j = (meta >> 20) & 31;
                const int64_t src = ((int64_t)(unsigned)d.y << 32) | (unsigned)d.x;
                bulk_g2s(smem + d.z, L_pool + (int64_t)s_sel[j] * L_stride + L_off_down + src, meta & 0xFFFFFu,
                         bar_dn);
            }
            if (KK > k) {                                // the shared expert: position k, its own down type
                const int ts = a.sh_dt == T_Q4K ? 0 : 1, np_s = a.sh_dt == T_Q4K ? 2 : 4;
                if (lane < np_s) {
                    const int4 d = s_cd_dn[ts][k * np_s + lane];
                    const int64_t src = ((int64_t)(unsigned)d.y << 32) | (unsigned)d.x;
                    bulk_g2s(smem + d.z, L_sh + L_sh_down + src, (unsigned)d.w & 0xFFFFFu, bar_dn);
                }
            }
        };
        int8_t* fxq = reinterpret_cast<int8_t*>(smem + P.off_fxq);
        float* fxd = reinterpret_cast<float*>(smem + P.off_fxd);
        int* fxbs32 = reinterpret_cast<int*>(smem + P.off_fxbs32);
        // the byte counts of this layer's copies do not depend on the routing: post them first
        if (warp == 0 && alive) {
            if (lane < NCH) {
                mbar_expect_tx(bar_gu + lane, s_gu_bytes[lane]);
            } else if (lane == NCH) {
                mbar_expect_tx(bar_dn, (unsigned)k * (L_dt == T_Q4K ? dn_bytes_q4 : dn_bytes_q6) + dn_bytes_sh);
            } else if (lane == NCH + 1 && has_next) {
                mbar_expect_tx(bar_wt, wt_bytes + (unsigned)(wn_hi - wn_lo) * (KK > k ? 2u : 1u));
            }
        }
        // router sums: every thread t <= E adds the RACC_COPIES partial copies of entry t (one L2 round trip)
        {
            const long long* racc = a.racc + (int64_t)buf * racc_stride;
            const double un1 = Sprev / RFIX, un2 = Sprev * Sprev / RFIX;
            for (int e = tid; e < NA; e += blockDim.x) {
                long long v = 0;
#pragma unroll
                for (int cp = 0; cp < RACC_COPIES; ++cp) v += __ldcg(racc + cp * NA + e);
                s_lgd[e] = (double)v * (e == E ? un2 : un1);
            }
        }
        __syncthreads();
        DEC_TR(l, 19);
        const float scale = 1.0f / sqrtf((float)(s_lgd[E] / H) + a.eps);
        const double Scur = s_lgd[E] > 0.0 ? sqrt(s_lgd[E]) : 1.0;   // scales the sums of layer l+1
        if (warp == 0) {
            // top-k on the logits, then the copies, then the weights (softmax) while the bytes fly
            float my_logit;
            route_select<NV>(s_lgd, E, k, scale, lane, s_sel, &my_logit);
            __syncwarp();
            DEC_TR(l, 1);
            // ---- B. this CTA's copies for the whole layer (descriptors precomputed at launch) ----
            if (alive) {
                const int4 d = s_cd_gu[lane];
                const unsigned meta = (unsigned)d.w;
                if (meta >> 29) {
                    const int j = (meta >> 20) & 31, ch = (meta >> 25) & 7;
                    const int64_t src = ((int64_t)(unsigned)d.y << 32) | (unsigned)d.x;
                    const bool upm = (meta >> 28) & 1;
                    const uint8_t* base = j < k ? L_pool + (int64_t)s_sel[j] * L_stride + (upm ? L_off_up : 0)
                                                : L_sh + (upm ? L_sh_up : 0);
                    bulk_g2s(smem + d.z, base + src, meta & 0xFFFFFu, bar_gu + ch);
                }
            }
            DEC_TR(l, 2);
            {
                int32_t* so = (c == 0 && a.sel_out) ? a.sel_out + (int64_t)l * k : nullptr;
                float* wo = (c == 0 && a.sel_out) ? a.w_out + (int64_t)l * k : nullptr;
                route_weights<NV>(s_lgd, E, k, a.renorm, scale, lane, my_logit, s_sel, s_w, so, wo);
                // the shared expert's weight: sigmoid of its gate logit (src/run_qwen35.cpp:659-666)
                if (KK > k && lane == 0) s_w[k] = sigmoid_f((float)((double)scale * s_lgd[E + 1]));
            }
            DEC_TR(l, 3);
            if (alive) {
                // the down rows are needed only after the gate/up phase: issue them once the first
                // gate/up chunk has landed, so that gate/up bytes are not queued behind them (in the
                // alias mode, after this CTA's gate/up rows are consumed)
                if (!a.alias_dn) {
                    if (!mbar_wait(bar_gu + 1, ph_gu)) { atomicOr(&a.sync[0], 2u); alive = false; }
                    issue_down();
                }
                if (has_next && lane == 0) bulk_g2s(wt, Ln_wrt + (int64_t)d0 * E, wt_bytes, bar_wt);
                if (has_next && lane == 1)
                    bulk_g2s(smem + P.off_wn, reinterpret_cast<const uint8_t*>(Ln_wnorm) + wn_lo,
                             (unsigned)(wn_hi - wn_lo), bar_wt);
                if (Ln_gs && lane == 2)
                    bulk_g2s(smem + P.off_gs, reinterpret_cast<const uint8_t*>(Ln_gs) + wn_lo, (unsigned)(wn_hi - wn_lo),
                             bar_wt);
            }
            DEC_TR(l, 4);
            DEC_TR(l, 5);
            named_sync(2, blockDim.x);              // fx (written by warps 1..) is complete
        } else {
            const int ng = H / 16;
            for (int g0 = 0; g0 < ng; g0 += blockDim.x - 32) {
                const int g = g0 + tid - 32;
                float v[16];
                float am = 0.f;
                if (g < ng) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 xr = ld_resid4(x + 16 * g + 4 * i);
                        const float4 wv = __ldg(reinterpret_cast<const float4*>(L_wnorm + 16 * g + 4 * i));
                        v[4 * i] = (xr.x * scale) * wv.x;
                        v[4 * i + 1] = (xr.y * scale) * wv.y;
                        v[4 * i + 2] = (xr.z * scale) * wv.z;
                        v[4 * i + 3] = (xr.w * scale) * wv.w;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[i]));
                }
                // the 16 groups of a 256 block are 16 consecutive lanes (warps 1.. start at group 0)
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                int bsum = 0;
                if (g < ng) {
                    const float iscale = am != 0.f ? 127.f / am : 0.f;
                    uint32_t packed[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int q = am != 0.f ? min(127, __float2int_rn(iscale * v[i])) : 0;
                        bsum += q;
                        packed[i >> 2] |= ((uint32_t)(q & 0xFF)) << (8 * (i & 3));
                    }
                    *reinterpret_cast<uint4*>(fxq + (g >> 4) * ACT_BLK + 16 * (g & 15)) =
                        make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    if ((g & 15) == 0) fxd[g >> 4] = am != 0.f ? 1.f / iscale : 0.f;
                }
                const int nb_sum = bsum + __shfl_xor_sync(0xffffffffu, bsum, 1);   // 32-value sub-block sum
                if (g < ng && (g & 1) == 0) fxbs32[g >> 1] = nb_sum;
            }
            named_arrive(2, blockDim.x);            // for warp 0
            named_sync(1, blockDim.x - 32);         // among warps 1..
        }
        // ---- C. gate/up + SwiGLU: lane = (row slot, 256-weight block) -----------------------------
        unsigned* amax = a.amax + (int64_t)buf * KK * nbI;
        {
            const int rs = lane / LPR, b = lane % LPR;
            const int8_t* act = fxq + ACT_BLK * b;
            const int* bs32 = fxbs32 + 8 * b;
            const float d8 = fxd[b];
            int waited = -1;
            for (int gi = warp - 1; warp > 0 && gi < ngroups; gi += nw - 1) {   // warp 0 routes and issues
                int ch = 0;
                while (ch + 1 < NCH && gi >= ((ch + 1) * ngroups) / NCH) ++ch;
                for (int cw = waited + 1; cw <= ch; ++cw) {
                    if (issued && alive && !mbar_wait(bar_gu + cw, ph_gu)) { atomicOr(&a.sync[0], 2u); alive = false; }
                }
                waited = max(waited, ch);
                if (TRACE && gi == 0 && tid == 32)
                    a.trace[((int64_t)c * a.n_layers + l) * DEC_TRACE_PHASES + 6] = gtimer();
                const int p = gi * RPW + rs;
                const bool valid = alive && p < np;
                float gsum = 0.f, usum = 0.f;
                if (valid) {
                    const uint8_t* gq = smem + P.off_gate_qs + p * P.gu_row_qs + 128 * b;
                    const uint8_t* uq = smem + P.off_up_qs + p * P.gu_row_qs + 128 * b;
                    const uint4 hg = lds128(smem + P.off_gate_hdr + p * P.gu_row_hdr + 16 * b);
                    const uint4 hu = lds128(smem + P.off_up_hdr + p * P.gu_row_hdr + 16 * b);
                    const Q4Scales sg = q4_scales(hg), su = q4_scales(hu);
                    int ig = 0, iu = 0;
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        const int cr = (cc + b) & 7, g = cr >> 1, hh = cr & 1;
                        const uint4 wg = lds128(gq + 16 * cr);
                        const uint4 wu = lds128(uq + 16 * cr);
                        const int4 alo = lds128i(act + 64 * g + 16 * hh);
                        const int4 ahi = lds128i(act + 64 * g + 32 + 16 * hh);
                        ig += q4_chunk(wg, alo, ahi, byte_of(sg.sc_lo, sg.sc_hi, 2 * g), byte_of(sg.sc_lo, sg.sc_hi, 2 * g + 1));
                        iu += q4_chunk(wu, alo, ahi, byte_of(su.sc_lo, su.sc_hi, 2 * g), byte_of(su.sc_lo, su.sc_hi, 2 * g + 1));
                    }
                    const int mg = q4_min_dot(sg, bs32), mu = q4_min_dot(su, bs32);
                    const float2 dg = __half22float2(*reinterpret_cast<const __half2*>(&hg.x));
                    const float2 du = __half22float2(*reinterpret_cast<const __half2*>(&hu.x));
                    gsum = d8 * (dg.x * (float)ig - dg.y * (float)mg);
                    usum = d8 * (du.x * (float)iu - du.y * (float)mu);
                }
                for (int o = 1; o < LPR; o <<= 1) {
                    gsum += __shfl_xor_sync(0xffffffffu, gsum, o);
                    usum += __shfl_xor_sync(0xffffffffu, usum, o);
                }
                if (valid && b == 0) {
                    const int q = q0 + p, j = q / I, i = q - j * I;
                    const float hv = silu_f(gsum) * usum;
                    a.h[(int64_t)j * I + i] = hv;
                    atomicMax(&s_amax[j * nbI + (i >> 8)], __float_as_uint(fabsf(hv)));
                }
            }
            // drain the chunks this warp did not need (every chunk's phase must complete)
            for (int cw = waited + 1; cw < NCH; ++cw)
                if (issued && !mbar_wait(bar_gu + cw, ph_gu)) { atomicOr(&a.sync[0], 2u); alive = false; }
        }
        ph_gu ^= 1;
        // publish this CTA's block maxima of h (a few atomics per CTA instead of one per row), then
        // count this CTA in the readiness counter of every 256-value block of h it produced to
        __syncthreads();
        if (tid < KK * nbI) {
            const unsigned v = s_amax[tid];
            if (v) atomicMax(&amax[tid], v);
            s_amax[tid] = 0u;
        }
        __syncthreads();
        if (a.alias_dn && warp == 0 && issued) {       // every warp is done with the gate/up rows
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_down();
        }
        if (tid == blockDim.x - 32 && alive) {        // the last warp issues no bulk copies
            for (int b = q0 / QK; b <= (q1 - 1) / QK; ++b)
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(hready + HREADY_STRIDE * b) : "memory");
        }
        DEC_TR(l, 7);
        // ---- D. expert positions are spread over the warps (wpe warps each). A position's warps
        //      wait until every CTA that produced part of its h has counted itself in, Q8_K that h
        //      into shared memory and run this CTA's down rows of the expert: no grid barrier, the
        //      quantisation and down rows of early experts overlap the production of later ones ----
        int8_t* hq = reinterpret_cast<int8_t*>(smem + P.off_hq);
        float* hd = reinterpret_cast<float*>(smem + P.off_hd);
        int* hbs = reinterpret_cast<int*>(smem + P.off_hbs);
        {
            float* y = reinterpret_cast<float*>(smem + P.off_y);
            const int wpe = nw / KK;
            const int j = warp / wpe, wi = warp - j * wpe;
            // the position's down type and plane offsets (the shared expert, position k, has its own)
            const int dtj = j < k ? L_dt : a.sh_dt;
            const int64_t pj1 = j < k ? P.dn_p1 : sh_p1, pj2 = j < k ? P.dn_p2 : sh_p2, pj3 = j < k ? P.dn_p3 : sh_p3;
            if (j < KK) {
                bool ok = alive;
                if (wi == 0 && lane < nbI && ok) {
                    // the CTAs owning pairs p0 and p0 + 255 of block (j, lane), and all between
                    const int64_t p0 = (int64_t)j * I + lane * QK;
                    const int need = (int)(((p0 + QK) * G - 1) / P_pairs - ((p0 + 1) * G - 1) / P_pairs + 1);
                    ok = wait_count(hready + HREADY_STRIDE * (j * nbI + lane), (unsigned)(l + 1) * (unsigned)need, a.sync);
                }
                if (wpe > 1) {                         // one warp of the position polls; the others follow
                    if (wi == 0) {
                        const bool all = __all_sync(0xffffffffu, ok);
                        if (lane == 0) s_pos_ok[j] = all ? 1 : 0;
                    }
                    named_sync(3 + j, 32 * wpe);
                    ok = ok && s_pos_ok[j] != 0;
                }
                ok = __all_sync(0xffffffffu, ok);
                __syncwarp();                          // orders the lanes' reads of h after the acquire polls
                if (tid == 0) DEC_TR(l, 8);
                for (int g0 = wi * 32; g0 < I / 16; g0 += wpe * 32) {
                    const int gg = g0 + lane;
                    const bool okg = ok && gg < I / 16;
                    const int eb = 16 * (okg ? gg : 0), blk = eb >> 8, gl = (eb & 255) >> 4;
                    int bsum = 0;
                    if (okg) {
                        const float am = __uint_as_float(__ldcg(amax + j * nbI + blk));
                        const float iscale = am != 0.f ? 127.f / am : 0.f;
                        float hv16[16];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 t4 = __ldcg(reinterpret_cast<const float4*>(a.h + (int64_t)j * I + eb + 4 * i));
                            hv16[4 * i] = t4.x; hv16[4 * i + 1] = t4.y; hv16[4 * i + 2] = t4.z; hv16[4 * i + 3] = t4.w;
                        }
                        uint32_t packed[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int q = am != 0.f ? min(127, __float2int_rn(iscale * hv16[i])) : 0;
                            bsum += q;
                            packed[i >> 2] |= ((uint32_t)(q & 0xFF)) << (8 * (i & 3));
                        }
                        *reinterpret_cast<uint4*>(hq + j * hq_stride(nbI) + blk * ACT_BLK + (eb & 255)) =
                            make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        if (gl == 0) hd[j * nbI + blk] = am != 0.f ? 1.f / iscale : 0.f;
                    }
                    const int pair = bsum + __shfl_xor_sync(0xffffffffu, bsum, 1);
                    if (okg) {
                        if (dtj == T_Q6K) {
                            // 16-sums in unit order [unit v = 2*h2 + r][a]: group gl = 8*h2 + 2*a + r
                            const int h2 = gl >> 3, aa = (gl >> 1) & 3, rr = gl & 1;
                            hbs[(j * nbI + blk) * 16 + 4 * (2 * h2 + rr) + aa] = bsum;
                        } else if ((gl & 1) == 0) {
                            hbs[(j * nbI + blk) * 8 + (gl >> 1)] = pair;     // 32-sums per sub-block
                        }
                    }
                }
                if (wpe > 1) named_sync(3 + j, 32 * wpe);
                else __syncwarp();
                if (tid == 0) DEC_TR(l, 9);
                if (issued && ok && !mbar_wait(bar_dn, ph_dn)) { atomicOr(&a.sync[0], 2u); ok = false; }
                if (tid == 0) DEC_TR(l, 10);
                // nbI consecutive lanes per row, one per 256-weight block; the lanes of a warp read the
                // same activation blocks (shared-memory broadcasts) and rotate their chunk order by
                // lane so that one load instruction spreads over the banks. Block sums of a row are
                // added as (b0 + b1) + (b2 + b3).
                const int dsub = dtj == T_Q6K ? (int)(((int64_t)d0 * nbI * 2) & 15) : 0;
                const int ipw = 32 / nbI, ui = lane / nbI, bl = lane - ui * nbI;
                const int rot = lane & 7;
                for (int gi = wi; gi * ipw < nr; gi += wpe) {
                    const int r = gi * ipw + ui;
                    const bool valid = ok && ui < ipw && r < nr;
                    float acc = 0.f;
                    if (valid) {
                        const uint8_t* reg = smem + P.off_dn + (int64_t)j * P.dn_stride;
                        const int64_t blk = (int64_t)r * nbI + bl;
                        const int8_t* act = hq + j * hq_stride(nbI) + ACT_BLK * bl;
                        const float d8 = hd[j * nbI + bl];
                        if (dtj == T_Q6K) {
                            const uint4 S = lds128(reg + pj2 + blk * 16);
                            const float d6 = __half2float(__ushort_as_half(
                                *reinterpret_cast<const unsigned short*>(reg + pj3 + dsub + blk * 2)));
                            const int* bsu = hbs + (j * nbI + bl) * 16;
                            const int sw = rot >> 2;       // half the lanes load the two ql chunks swapped
                            int isum = 0;
#pragma unroll
                            for (int vv = 0; vv < 4; ++vv) {
                                const int v = (vv + rot) & 3, h2 = v >> 1, rr = v & 1;
                                const uint8_t* ql = reg + blk * 128 + 64 * h2 + 16 * rr;
                                const uint4 P0 = lds128(ql + 32 * sw);
                                const uint4 P1 = lds128(ql + 32 * (sw ^ 1));
                                const uint4 A = sw ? P1 : P0, B = sw ? P0 : P1;
                                const uint4 C = lds128(reg + pj1 + blk * 64 + 32 * h2 + 16 * rr);
                                const int8_t* a0 = act + 128 * h2 + 16 * rr;
                                const int4 x0 = lds128i(a0), x1 = lds128i(a0 + 32), x2 = lds128i(a0 + 64),
                                           x3 = lds128i(a0 + 96);
                                const int4 bs4 = lds128i(bsu + 4 * v);
                                const uint32_t Aw[4] = {A.x, A.y, A.z, A.w}, Bw[4] = {B.x, B.y, B.z, B.w};
                                const uint32_t Cw[4] = {C.x, C.y, C.z, C.w};
                                const int xa0[4] = {x0.x, x0.y, x0.z, x0.w}, xa1[4] = {x1.x, x1.y, x1.z, x1.w};
                                const int xa2[4] = {x2.x, x2.y, x2.z, x2.w}, xa3[4] = {x3.x, x3.y, x3.z, x3.w};
                                int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
                                for (int i = 0; i < 4; ++i) {
                                    const uint32_t cw = Cw[i];
                                    s0 = __dp4a((int)((Aw[i] & 0x0F0F0F0Fu) | ((cw << 4) & 0x30303030u)), xa0[i], s0);
                                    s1 = __dp4a((int)((Bw[i] & 0x0F0F0F0Fu) | ((cw << 2) & 0x30303030u)), xa1[i], s1);
                                    s2 = __dp4a((int)(((Aw[i] >> 4) & 0x0F0F0F0Fu) | (cw & 0x30303030u)), xa2[i], s2);
                                    s3 = __dp4a((int)(((Bw[i] >> 4) & 0x0F0F0F0Fu) | ((cw >> 2) & 0x30303030u)), xa3[i], s3);
                                }
                                // int8 scales sc[8h2 + rr + 2a]: bytes of word 2h2 (a = 0, 1) and 2h2+1 (a = 2, 3)
                                const uint32_t wa = h2 ? S.z : S.x, wb = h2 ? S.w : S.y;
                                const int sh = 8 * rr;
                                isum += sext8(wa >> sh) * (s0 - 32 * bs4.x) + sext8(wa >> (sh + 16)) * (s1 - 32 * bs4.y) +
                                        sext8(wb >> sh) * (s2 - 32 * bs4.z) + sext8(wb >> (sh + 16)) * (s3 - 32 * bs4.w);
                            }
                            acc = d8 * d6 * (float)isum;
                        } else {
                            const uint8_t* wq = reg + blk * 128;
                            const uint4 hh4 = lds128(reg + pj1 + blk * 16);
                            const Q4Scales s4 = q4_scales(hh4);
                            int isc = 0;
#pragma unroll
                            for (int cc = 0; cc < 8; ++cc) {
                                const int cr = (cc + rot) & 7, g = cr >> 1, hh = cr & 1;
                                const uint4 w = lds128(wq + 16 * cr);
                                const int4 alo = lds128i(act + 64 * g + 16 * hh);
                                const int4 ahi = lds128i(act + 64 * g + 32 + 16 * hh);
                                isc += q4_chunk(w, alo, ahi, byte_of(s4.sc_lo, s4.sc_hi, 2 * g),
                                                byte_of(s4.sc_lo, s4.sc_hi, 2 * g + 1));
                            }
                            const int mn = q4_min_dot(s4, hbs + (j * nbI + bl) * 8);
                            const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hh4.x));
                            acc = d8 * (dm.x * (float)isc - dm.y * (float)mn);
                        }
                    }
                    const float t1 = __shfl_down_sync(0xffffffffu, acc, 1);
                    const float t2 = __shfl_down_sync(0xffffffffu, acc, 2);
                    const float t3 = __shfl_down_sync(0xffffffffu, acc, 3);
                    float sum = acc;
                    if (nbI == 2) sum = acc + t1;
                    else if (nbI == 3) sum = (acc + t1) + t2;
                    else if (nbI == 4) sum = (acc + t1) + (t2 + t3);
                    if (valid && bl == 0) y[r * KK + j] = sum;
                }
                if (!ok) alive = false;
            }
        }
        ph_dn ^= 1;
        __syncthreads();
        DEC_TR(l, 11);
        // every CTA has published its h, so every CTA has read this layer's router sums: clear them
        // for layer l + 2, and the block maxima that layer l + 1 will use
        if (c == 0 && alive) {
            long long* rz = a.racc + (int64_t)buf * racc_stride;
            for (int e = tid; e < racc_stride; e += blockDim.x) rz[e] = 0;
            unsigned* az = a.amax + (int64_t)(buf ^ 1) * KK * nbI;
            for (int e = tid; e < KK * nbI; e += blockDim.x) az[e] = 0u;
        }
        {
            const float* y = reinterpret_cast<const float*>(smem + P.off_y);
            for (int r = tid; r < nr; r += blockDim.x) {
                float acc = 0.f;
                for (int j = 0; j < k; ++j) acc += s_w[j] * y[r * KK + j];
                if (KK > k) acc = acc + y[r * KK + k] * s_w[k];      // shared expert, added after its gate
                const R xn = from_f32<R>(acc + xs[r]);
                if (alive) x[d0 + r] = xn;
                xs[r] = to_f32<R>(xn);
            }
        }
        DEC_TR(l, 14);
        if (has_next) {
            if (issued_wt && !mbar_wait(bar_wt, ph_wt)) { atomicOr(&a.sync[0], 2u); alive = false; }
            ph_wt ^= 1;
            __syncthreads();
            DEC_TR(l, 15);
            const float* wn = reinterpret_cast<const float*>(smem + P.off_wn) + wn_sub;
            const float* gs = reinterpret_cast<const float*>(smem + P.off_gs) + wn_sub;
            long long* acc = a.racc + (int64_t)(buf ^ 1) * racc_stride + (int64_t)(c % RACC_COPIES) * NA;
            for (int e = tid; e < NA; e += blockDim.x) {
                double s = 0.0;
                if (e < E) {
                    for (int r = 0; r < nr; ++r) s += (double)wt[r * E + e] * (double)(wn[r] * xs[r]);
                } else if (e == E) {
                    for (int r = 0; r < nr; ++r) s += (double)(xs[r] * xs[r]);
                } else if (KK > k) {
                    for (int r = 0; r < nr; ++r) s += (double)gs[r] * (double)(wn[r] * xs[r]);
                }
                if (alive && (e <= E || KK > k))
                    add_fixed(&acc[e], s, e == E ? RFIX / (Scur * Scur) : RFIX / Scur, a.sync);
            }
            DEC_TR(l, 12);
            if (!grid_barrier(a.sync, nbar++, &s_ok, DEC_TRP(l, 16))) alive = false;
        }
        Sprev = Scur;
        DEC_TR(l, 13);
    }
#undef DEC_TR
#undef DEC_TRP
    // ---- exit: the last CTA out restores the zero state of the counters and max buffers --------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.sync[2], 1u);
        if (old == (unsigned)G - 1) {
            __threadfence();
            unsigned* az = a.amax + (int64_t)((a.n_layers - 1) & 1) * KK * nbI;
            for (int e = 0; e < KK * nbI; ++e) az[e] = 0u;
            for (int e = 0; e < KK * nbI; ++e) hready[HREADY_STRIDE * e] = 0u;
            if (ld_relaxed(&a.sync[0]) & 6u)      // an aborted launch may leave partial sums behind
                for (int e = 0; e < 2 * racc_stride; ++e) a.racc[e] = 0;
            a.sync[1] = 0u;
            a.sync[2] = 0u;
            __threadfence();
        }
    }
}

int decode_max_tokens() { return 1; }
int decode_grid() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_num_sms == 0) cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    return g_num_sms;
}
int decode_trace_phases() { return DEC_TRACE_PHASES; }

// 0: both shares fit in shared memory, 1: only with the down rows over the gate/up rows, -1: neither
static const void* decode_fn(bool bf16, int nv, bool trace);
static int decode_alias_mode(const Dims& d, int KK, int G) {
    int dev = 0, max_smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};                          // static shared memory (the same in every instantiation)
    if (cudaFuncGetAttributes(&fa, decode_fn(false, 16, true)) != cudaSuccess) return -1;
    for (int alias = 0; alias < 2; ++alias) {
        int64_t need = 0;
        for (int dt : {(int)T_Q4K, (int)T_Q6K}) {
            DecodePlan P;
            P.init(d.H, d.E, KK, d.I, dt, G, alias);
            need = need > P.total ? need : P.total;
        }
        if (need + (int64_t)fa.sharedSizeBytes <= max_smem) return alias;
    }
    return -1;
}

bool decode_supported(const Dims& d, const LayerWeights* lws, int n_layers) {
    if (n_layers <= 0) return false;
    const int KK = d.k + (lws[0].shared ? 1 : 0);            // expert positions: routed + shared
    if (KK > 16 || d.E % 4 != 0 || d.E > 512) return false;
    const int nbH = d.H / QK, nbI = d.I / QK;
    if (nbH > 32 || (nbH & (nbH - 1)) != 0) return false;    // lanes per gate/up row: a power of two <= 32
    if (nbI > 4) return false;                                // down rows: one lane per block, 4 lanes per item
    const int G = decode_grid();
    if ((int64_t)KK * d.I < G || d.H < G) return false;      // every CTA must own rows
    if ((KK * d.I + G - 1) / G > d.I) return false;           // a CTA's pairs span at most 2 experts
    for (int l = 0; l < n_layers; ++l) {
        const LayerWeights& L = lws[l];
        if (L.gate_type != T_Q4K || L.up_type != T_Q4K) return false;
        if (L.down_type != T_Q4K && L.down_type != T_Q6K) return false;
        if ((L.shared != nullptr) != (KK > d.k)) return false;
        if (L.shared && (L.sh_gate_type != T_Q4K || L.sh_up_type != T_Q4K || L.sh_down_type != lws[0].sh_down_type ||
                         (L.sh_down_type != T_Q4K && L.sh_down_type != T_Q6K) || !L.sh_gate_inp))
            return false;
    }
    return decode_alias_mode(d, KK, G) >= 0;
}

template <typename R, bool TRACE>
const void* decode_fn_nv(int nv) {
    return nv == 2 ? (const void*)k_decode<R, 2, TRACE> : nv == 4 ? (const void*)k_decode<R, 4, TRACE>
         : nv == 8 ? (const void*)k_decode<R, 8, TRACE> : (const void*)k_decode<R, 16, TRACE>;
}

static const void* decode_fn(bool bf16, int nv, bool trace) {
    if (bf16) return trace ? decode_fn_nv<__nv_bfloat16, true>(nv) : decode_fn_nv<__nv_bfloat16, false>(nv);
    return trace ? decode_fn_nv<float, true>(nv) : decode_fn_nv<float, false>(nv);
}

cudaError_t launch_decode_persistent(const Dims& d, int KK, int sh_dt, const LayerWeights* lws_dev, int n_layers,
                                     const Scratch& sc, void* x_inout, int T, int32_t* sel_out, float* w_out,
                                     cudaStream_t s, unsigned long long* trace) {
    if (T != 1) return cudaErrorInvalidValue;
    const int G = decode_grid();
    const int alias = decode_alias_mode(d, KK, G);
    if (alias < 0) return cudaErrorInvalidValue;
    int64_t smem = 0;
    for (int dt : {(int)T_Q4K, (int)T_Q6K}) {
        DecodePlan P;
        P.init(d.H, d.E, KK, d.I, dt, G, alias);
        smem = smem > P.total ? smem : P.total;
    }
    DecodeArgs a;
    a.KK = KK;
    a.sh_dt = sh_dt;
    a.lw = lws_dev;
    a.n_layers = n_layers;
    a.H = d.H; a.E = d.E; a.k = d.k; a.I = d.I; a.renorm = d.renorm; a.eps = d.eps; a.resid_bf16 = d.resid_bf16;
    a.x = x_inout;
    a.sel_out = sel_out;
    a.w_out = w_out;
    a.h = sc.h;
    a.amax = sc.amax;
    a.racc = reinterpret_cast<long long*>(sc.partials);
    a.sync = sc.sync;
    a.trace = trace;
    a.alias_dn = alias;
    void* args[] = {&a};
    const int nv = d.E <= 64 ? 2 : d.E <= 128 ? 4 : d.E <= 256 ? 8 : 16;
    const void* fn = decode_fn(d.resid_bf16 != 0, nv, trace != nullptr);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaLaunchCooperativeKernel(fn, dim3(G), dim3(DEC_THREADS), args, (size_t)smem, s);
    return e;
}

// ---- decode without any device allocation ---------------------------------------------------------
// Some callers cannot allocate device memory when they run a decode step: an engine whose device
// memory is entirely handed out by its own arena after start-up (hoard itself sizes its expert slot
// pool to the VRAM budget), or a step loop that must not call cudaMalloc (it can synchronise the
// device, and a failure in the middle of a step has no recovery). For them the
// persistent decode kernel can take its scratch (h, the block maxima of h, the router accumulators and
// the grid-barrier words) from this fixed file-scope device array instead of a context's scratch.
// Every GPU that loads this library holds the array until the process exits.
constexpr int NOALLOC_MAX_K = 16;       // expert positions per token (routed + shared)
constexpr int NOALLOC_MAX_I = 1024;     // expert intermediate size
constexpr int NOALLOC_MAX_E = 512;      // experts per layer
constexpr size_t NOALLOC_H_BYTES = (size_t)NOALLOC_MAX_K * NOALLOC_MAX_I * 4;                  // 64 KiB
constexpr size_t NOALLOC_AMAX_BYTES = 2 * NOALLOC_MAX_K * (NOALLOC_MAX_I / QK) * 4;           // 512 B
constexpr size_t NOALLOC_RACC_BYTES = (size_t)2 * RACC_COPIES * (NOALLOC_MAX_E + 2) * 8;       // 32,896 B
constexpr size_t NOALLOC_SYNC_BYTES = 8704;          // error word, barrier words, h block counters (one line each)
constexpr size_t NOALLOC_ZERO_BYTES = NOALLOC_AMAX_BYTES + NOALLOC_RACC_BYTES + NOALLOC_SYNC_BYTES;
constexpr size_t NOALLOC_BYTES = NOALLOC_H_BYTES + NOALLOC_ZERO_BYTES;                         // ~105 KiB
static __device__ __align__(256) unsigned char g_decode_scratch[NOALLOC_BYTES];

// Device address of g_decode_scratch on the current device. In host code the array's name is only a
// host-side stand-in, so the address is looked up with that device current; the lookup also loads the
// module that holds the array. A context resolves it once, when it is created.
cudaError_t decode_static_address(void** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    *out = p;
    return cudaSuccess;
}

bool decode_static_fits(const Dims& d, int KK) {
    return KK <= NOALLOC_MAX_K && d.I <= NOALLOC_MAX_I && d.E <= NOALLOC_MAX_E;
}

size_t decode_static_error_offset() { return NOALLOC_H_BYTES + NOALLOC_AMAX_BYTES + NOALLOC_RACC_BYTES; }

cudaError_t launch_decode_static(const Dims& d, int KK, int sh_dt, const LayerWeights* lws_dev, int n_layers,
                                 void* scratch, void* x_inout, int32_t* sel_out, float* w_out, cudaStream_t s) {
    if (!decode_static_fits(d, KK) || !scratch) return cudaErrorInvalidValue;
    cudaError_t e;
    uint8_t* b = static_cast<uint8_t*>(scratch);
    Scratch sc{};
    sc.h = reinterpret_cast<float*>(b);
    sc.amax = reinterpret_cast<unsigned*>(b + NOALLOC_H_BYTES);
    sc.partials = reinterpret_cast<float*>(b + NOALLOC_H_BYTES + NOALLOC_AMAX_BYTES);
    sc.sync = reinterpret_cast<unsigned*>(b + NOALLOC_H_BYTES + NOALLOC_AMAX_BYTES + NOALLOC_RACC_BYTES);
    // the array keeps whatever the last call left: clear everything the kernel expects at zero
    // (block maxima, router accumulators, barrier counters, error word); h needs no clearing
    e = cudaMemsetAsync(b + NOALLOC_H_BYTES, 0, NOALLOC_ZERO_BYTES, s);
    if (e != cudaSuccess) return e;
    return launch_decode_persistent(d, KK, sh_dt, lws_dev, n_layers, sc, x_inout, 1, sel_out, w_out, s, nullptr);
}

}  // namespace hoard
