// kernels_stream.cu -- small-batch expert matmuls that stream each selected slot's weights from HBM
// once per call, for the grouped (exact-integer, Q8_K-activation) path.
//
// Both kernels are persistent (one CTA per SM) and split each CTA into
//   * a producer warp, whose lane 0 stages one tile of weight rows per pipeline stage with a few
//     1-D bulk copies (one per weight plane: the plane layout keeps a tile's rows contiguous),
//     completion counted on the stage's "full" mbarrier; and
//   * eight consumer warps, which wait for a stage, compute, and release it on its "empty" mbarrier.
// A tile is (slot, block of rows); a CTA takes tiles blockIdx.x, blockIdx.x + gridDim.x, ... in
// rounds of up to RT, whose metadata (slot, rows, entries) all threads load into shared memory at the
// start of the round. The Q8_K activations of a tile's first ACT entries are copied into one of three
// shared buffers by the consumers with cp.async two tiles ahead; entries beyond ACT are read from
// global memory directly.
//
// Lane mapping (fixed across rows, so a lane's activations are loaded once per tile and reused for
// every row it computes):
//   gate/up (Q4_K, H = 2048): lane = (block bb = lane/4, 32-byte group g = lane%4) of a row: the
//     lane's 32 qs bytes hold sub-blocks 2g (low nibbles) and 2g+1 (high nibbles), 64 weights, and
//     its activations are the 64 bytes at bb*256 + 64g. A warp computes 2 gate and 2 up rows and
//     reduces the four lane sums with one transposing butterfly (each lane ends with one row).
//   down (Q6_K or Q4_K, I/256 <= 4): lane = (row rq = lane/4 of the warp's 8 rows, unit q = lane%4);
//     the lane loops over the row's blocks. Q6_K unit q = 64 weights (ql 2 x 16 B, qh 16 B; the
//     ql/qh layout of q6k_unit_isum); Q4_K unit q = 32-byte group q. Shared activations are laid
//     out [piece a][unit q] so that the four units' 16-byte reads fall in distinct banks.
//
// Integer dots are exact (dp4a; the high nibbles of Q4_K are taken as 16 x nibble by an
// unsigned x signed dp4a and shifted back, exact since every term is a multiple of 16); the float
// combination per lane is that of ggml's Q4_K/Q6_K x Q8_K dot (d8 * (d * sum sc*isum - dmin * sum
// m*bsum), d8 * d6 * sum sc*(isum - 32*bsum)); lane sums are added by butterflies, so results agree
// with the oracle to f32 summation order.
#include "common.cuh"
#include "kernels.h"
#include "async_copy.cuh"

namespace hoard {
namespace {

constexpr int SW_CTAS_PER_SM = 2;                        // resident CTAs per SM (each with its own pipeline)
constexpr int SW_CONSUMERS = 8;                          // consumer warps
constexpr int SW_THREADS = 32 * (SW_CONSUMERS + 1);      // + the producer warp
constexpr int sw_smem(int ctas_per_sm) { return (ctas_per_sm == 1 ? 227 : 112) * 1024; }   // per CTA
constexpr int RT = 64;                                   // tiles per metadata round
constexpr int MAX_ACT = 16;
constexpr int SW_STATIC = RT * 16 + RT * MAX_ACT * 4 + 64;   // static shared memory of either kernel
constexpr int sw_dyn(int ctas_per_sm) { return sw_smem(ctas_per_sm) - SW_STATIC - 1024; }  // dynamic budget
constexpr int SW_DYN = sw_dyn(SW_CTAS_PER_SM);
constexpr int NAB = 3;                                   // activation buffers (staged two tiles ahead)
constexpr int GT_R = 16;                                 // gate rows (and up rows) per tile
constexpr int GT_STAGES = SW_CTAS_PER_SM == 1 ? 4 : 2;
constexpr int GT_ACT = SW_CTAS_PER_SM == 1 ? 8 : 4;      // entries staged per gate/up tile
constexpr int DT_R = 64;                                 // down rows per tile (8 warps x 8 rows)
constexpr int DT_ACT = SW_CTAS_PER_SM == 1 ? 16 : 8;     // entries staged per down tile
constexpr int TG = SW_CTAS_PER_SM == 1 ? 4 : 2;          // entries per register group
static_assert(GT_ACT <= MAX_ACT && DT_ACT <= MAX_ACT, "staged entries");
static_assert(DT_ACT % TG == 0, "token groups lie wholly inside or outside the staged entries");

__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {   // unsigned bytes of a x signed bytes of b
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint4 lds16(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ int4 ldg16i(const void* p) { return *reinterpret_cast<const int4*>(p); }

struct SlotPtrs {
    const uint8_t *g, *u, *d;
    int dt;
};
__device__ __forceinline__ SlotPtrs slot_ptrs(const LayerWeights& lw, int s) {
    SlotPtrs m;
    if (s < lw.n_slots) {
        const uint8_t* b = lw.pool + (int64_t)s * lw.slot_stride;
        m.g = b; m.u = b + lw.off_up; m.d = b + lw.off_down; m.dt = lw.down_type;
    } else {
        m.g = lw.shared; m.u = lw.shared + lw.sh_off_up; m.d = lw.shared + lw.sh_off_down; m.dt = lw.sh_down_type;
    }
    return m;
}

// Tile metadata of one round: the CTA's tiles blockIdx.x + (base + i) * gridDim.x, i < RT, loaded
// into shared memory by all threads at the start of the round (one pass of dependent loads instead of
// one per tile on every warp's critical path): slot, first row, first sorted entry, entry count, and
// the first ACT entry ids.
struct TileMeta {
    int slot, r0, start, n;
};
template <int ACT>
__device__ __forceinline__ int load_round(TileMeta* meta, int (*ent)[MAX_ACT], const int2* items, const int* offsets,
                                          const int* perm, int ntiles, int ntr, int R, int base) {
    const int G = gridDim.x;
    const int first = blockIdx.x + base * G;
    const int nr = first >= ntiles ? 0 : min(RT, (ntiles - first + G - 1) / G);
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        const int tile = first + i * G;
        TileMeta m;
        m.slot = items[tile / ntr].x;
        m.r0 = (tile % ntr) * R;
        m.start = offsets[m.slot];
        m.n = offsets[m.slot + 1] - m.start;
        meta[i] = m;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < nr * ACT; idx += blockDim.x) {
        const int i = idx / ACT, e = idx - i * ACT;
        if (e < meta[i].n) ent[i][e] = perm[meta[i].start + e];
    }
    __syncthreads();
    return nr;
}

// Scales and mins of sub-blocks 2g, 2g+1 of a Q4_K header (branch-free for the lane's fixed g).
struct Q4Scales {
    int sc0, sc1, m0, m1;
    float d, dmin;
};
struct Q4Lane {           // per-lane constants of the decode
    int sh, shA, mA, mB;
    __device__ __forceinline__ explicit Q4Lane(int g) {
        sh = 16 * (g & 1);
        const bool lo = g < 2;
        shA = lo ? 0 : 2;
        mA = lo ? 63 : 0x30;
        mB = lo ? 0 : 0xF;
    }
    __device__ __forceinline__ Q4Scales decode(const uint4& h) const {
        const uint32_t y = h.y >> sh, z = h.z >> sh, w = h.w >> sh;
        Q4Scales s;
        s.sc0 = (int)(((y >> shA) & mA) | (w & mB));
        s.sc1 = (int)(((y >> (8 + shA)) & mA) | ((w >> 8) & mB));
        s.m0 = (int)(((z >> shA) & mA) | ((w >> 4) & mB));
        s.m1 = (int)(((z >> (8 + shA)) & mA) | ((w >> 12) & mB));
        s.d = h2f(h.x);
        s.dmin = h2f(h.x >> 16);
        return s;
    }
};

// One entry's Q8_K activations for a lane's 64 weights of one block.
struct Act64 {
    int a[16];
    int bs0, bs1;
    float d8;
};
// q64: the 64 activation bytes; bs4: the 4 partial sums of 16; d8: the block scale
__device__ __forceinline__ void load_act64(Act64& A, const int8_t* q64, const int* bs4, const float* d8) {
    const int4 v0 = ldg16i(q64), v1 = ldg16i(q64 + 16), v2 = ldg16i(q64 + 32), v3 = ldg16i(q64 + 48);
    A.a[0] = v0.x; A.a[1] = v0.y; A.a[2] = v0.z; A.a[3] = v0.w;
    A.a[4] = v1.x; A.a[5] = v1.y; A.a[6] = v1.z; A.a[7] = v1.w;
    A.a[8] = v2.x; A.a[9] = v2.y; A.a[10] = v2.z; A.a[11] = v2.w;
    A.a[12] = v3.x; A.a[13] = v3.y; A.a[14] = v3.z; A.a[15] = v3.w;
    const int4 b = ldg16i(bs4);
    A.bs0 = b.x + b.y;
    A.bs1 = b.z + b.w;
    A.d8 = *d8;
}

// A Q4_K group (32 qs bytes) split into low nibbles and 16 x high nibbles.
struct Q4Group {
    uint32_t lo[8], hi[8];
    __device__ __forceinline__ void set(const uint4& w0, const uint4& w1) {
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = w[i] & 0x0F0F0F0Fu;
            hi[i] = w[i] & 0xF0F0F0F0u;
        }
    }
    __device__ __forceinline__ float dot(const Q4Scales& s, const Act64& A) const {
        int l0 = 0, l1 = 0, h0 = 0, h1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            l0 = __dp4a((int)lo[i], A.a[i], l0);
            l1 = __dp4a((int)lo[i + 4], A.a[i + 4], l1);
            h0 = dp4a_us(hi[i], A.a[i + 8], h0);
            h1 = dp4a_us(hi[i + 4], A.a[i + 12], h1);
        }
        const int slo = l0 + l1, shi = (h0 + h1) >> 4;
        const int isum = s.sc0 * slo + s.sc1 * shi;
        const int msum = s.m0 * A.bs0 + s.m1 * A.bs1;
        return A.d8 * (s.d * (float)isum - s.dmin * (float)msum);
    }
};

// ---------------------------------------------------------------------------------------------
// gate/up + SwiGLU: h[ent][i] = silu(gate_i . x_t) * (up_i . x_t) for every entry of the slot
// Stage: gate qs [R][1024] | gate hdr [R][128] | up qs [R][1024] | up hdr [R][128]
// Activation buffer entry: q [2048] | bs [128 ints] | d [8 floats]
// ---------------------------------------------------------------------------------------------
constexpr int GU_NB = 8;                                 // blocks per row (H = 2048)
constexpr int GU_QROW = GU_NB * 128, GU_HROW = GU_NB * 16;
constexpr int GU_MAT = GT_R * (GU_QROW + GU_HROW);       // one matrix's share of a stage
constexpr int GU_STAGE = 2 * GU_MAT;
constexpr int GU_AENT = QK * GU_NB + GU_NB * 16 * 4 + GU_NB * 4;   // 2592 bytes per staged entry
constexpr int GU_ABUF = GT_ACT * GU_AENT;
constexpr int GU_SMEM = GT_STAGES * GU_STAGE + NAB * GU_ABUF + 2 * GT_STAGES * 8;
static_assert(GU_SMEM <= SW_DYN, "gate/up stream shared memory");
static_assert(GU_AENT % 16 == 0, "staged entry alignment");
static_assert(GT_ACT % TG == 0, "token groups lie wholly inside or outside the staged entries");

struct GuArgs {
    LayerWeights lw;
    int I, KK;
    const int* offsets;
    const int* perm;
    const int2* items;
    const int* n_items;
    const int8_t* xq;
    const float* xd;
    const int* xbs;
    float* h;
    unsigned* err;
    unsigned long long* stamp;                           // optional {first start, last end}
};

// Consumers copy the activations of the round's tile i (its first GT_ACT entries) into `buf` and
// commit one cp.async group (an empty group past the round's last tile).
__device__ __forceinline__ void gu_stage_acts(const GuArgs& a, const TileMeta* meta, const int (*ent)[MAX_ACT], int i,
                                              int nr, uint8_t* buf, int ctid) {
    constexpr int H = QK * GU_NB;
    constexpr int PPE = GU_AENT / 16;                    // 16-byte pieces per entry
    if (i < nr) {
        const int n = min(meta[i].n, GT_ACT);
        for (int idx = ctid; idx < n * PPE; idx += 32 * SW_CONSUMERS) {
            const int e = idx / PPE, p = idx - e * PPE;
            const int t = ent[i][e] / a.KK;
            const uint8_t* src;
            if (p < H / 16) src = reinterpret_cast<const uint8_t*>(a.xq + (int64_t)t * H) + 16 * p;
            else if (p < H / 16 + H / 64) src = reinterpret_cast<const uint8_t*>(a.xbs + (int64_t)t * (H / 16)) + 16 * (p - H / 16);
            else src = reinterpret_cast<const uint8_t*>(a.xd + (int64_t)t * GU_NB) + 16 * (p - H / 16 - H / 64);
            // q pieces (16 bytes; lane L of a row reads pieces 4L..4L+3) go to unit 32 * (p % 4) + p / 4,
            // so that the eight lanes of a quarter warp always read eight distinct bank groups
            const int pos = p < H / 16 ? 32 * (p & 3) + (p >> 2) : p;
            cp_async16(buf + e * GU_AENT + 16 * pos, src);
        }
    }
    cp_async_commit();
}

// Gate/up of one tile for NT entries (a compile-time count, so that nothing is issued for absent
// entries). The lane reads its two 16-byte weight halves in the order (sw, 1 - sw), sw = bb & 1 --
// so that a quarter warp's loads fall in distinct bank groups -- and its activation pieces in the
// matching order p ^ sw.
struct GuLane {
    int lane, bb, g, sw, rr;
    bool up16, up8;
    Q4Lane ql;
    __device__ __forceinline__ explicit GuLane(int lane_, int warp) : ql(lane_ & 3) {
        lane = lane_;
        bb = lane >> 2;
        g = lane & 3;
        sw = bb & 1;
        rr = 2 * warp;
        up16 = lane & 16;
        up8 = lane & 8;
    }
};

template <int NT>
__device__ __forceinline__ void gu_group(const GuArgs& a, const GuLane& L, const uint8_t* st, const uint8_t* ab,
                                         bool staged, const int* ent_row, const TileMeta& m, int e0) {
    constexpr int H = QK * GU_NB;
    Act64 A[NT];
    int en[NT];
#pragma unroll
    for (int u = 0; u < NT; ++u) {
        const int e = e0 + u;
        if (staged) {
            en[u] = ent_row[e];
            const uint8_t* E = ab + e * GU_AENT;
            const int4 v0 = ldg16i(E + 16 * (32 * (0 ^ L.sw) + L.lane)), v1 = ldg16i(E + 16 * (32 * (1 ^ L.sw) + L.lane));
            const int4 v2 = ldg16i(E + 16 * (32 * (2 ^ L.sw) + L.lane)), v3 = ldg16i(E + 16 * (32 * (3 ^ L.sw) + L.lane));
            A[u].a[0] = v0.x; A[u].a[1] = v0.y; A[u].a[2] = v0.z; A[u].a[3] = v0.w;
            A[u].a[4] = v1.x; A[u].a[5] = v1.y; A[u].a[6] = v1.z; A[u].a[7] = v1.w;
            A[u].a[8] = v2.x; A[u].a[9] = v2.y; A[u].a[10] = v2.z; A[u].a[11] = v2.w;
            A[u].a[12] = v3.x; A[u].a[13] = v3.y; A[u].a[14] = v3.z; A[u].a[15] = v3.w;
            const int4 b = ldg16i(reinterpret_cast<const int*>(E + H) + 4 * L.lane);
            A[u].bs0 = b.x + b.y;
            A[u].bs1 = b.z + b.w;
            A[u].d8 = reinterpret_cast<const float*>(E + H + H / 4)[L.bb];
        } else {
            en[u] = a.perm[m.start + e];
            const int t = en[u] / a.KK;
            const int8_t* q64 = a.xq + (int64_t)t * H + 64 * L.lane;
            const int4 v0 = ldg16i(q64 + 16 * (0 ^ L.sw)), v1 = ldg16i(q64 + 16 * (1 ^ L.sw));
            const int4 v2 = ldg16i(q64 + 16 * (2 ^ L.sw)), v3 = ldg16i(q64 + 16 * (3 ^ L.sw));
            A[u].a[0] = v0.x; A[u].a[1] = v0.y; A[u].a[2] = v0.z; A[u].a[3] = v0.w;
            A[u].a[4] = v1.x; A[u].a[5] = v1.y; A[u].a[6] = v1.z; A[u].a[7] = v1.w;
            A[u].a[8] = v2.x; A[u].a[9] = v2.y; A[u].a[10] = v2.z; A[u].a[11] = v2.w;
            A[u].a[12] = v3.x; A[u].a[13] = v3.y; A[u].a[14] = v3.z; A[u].a[15] = v3.w;
            const int4 b = ldg16i(a.xbs + (int64_t)t * (H / 16) + 4 * L.lane);
            A[u].bs0 = b.x + b.y;
            A[u].bs1 = b.z + b.w;
            A[u].d8 = a.xd[(int64_t)t * GU_NB + L.bb];
        }
    }
    float v[4][NT];
#pragma unroll
    for (int r = 0; r < 4; ++r) {                        // gate rr, gate rr+1, up rr, up rr+1
        const uint8_t* M = st + (r >> 1) * GU_MAT;
        const uint8_t* W = M + (L.rr + (r & 1)) * GU_QROW + 32 * L.lane;
        Q4Group q;
        q.set(lds16(W + 16 * L.sw), lds16(W + 16 * (1 - L.sw)));
        const Q4Scales sc = L.ql.decode(lds16(M + GT_R * GU_QROW + (L.rr + (r & 1)) * GU_HROW + L.bb * 16));
#pragma unroll
        for (int u = 0; u < NT; ++u) v[r][u] = q.dot(sc, A[u]);
    }
#pragma unroll
    for (int u = 0; u < NT; ++u) {
        // transposing butterfly: lanes 0-7 end with gate rr, 8-15 gate rr+1, 16-23 up rr, 24-31 up rr+1
        float k0 = L.up16 ? v[2][u] : v[0][u], k1 = L.up16 ? v[3][u] : v[1][u];
        const float s0 = L.up16 ? v[0][u] : v[2][u], s1 = L.up16 ? v[1][u] : v[3][u];
        k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        float k = L.up8 ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, L.up8 ? k0 : k1, 8);
        k += __shfl_xor_sync(0xffffffffu, k, 4);
        k += __shfl_xor_sync(0xffffffffu, k, 2);
        k += __shfl_xor_sync(0xffffffffu, k, 1);
        const float hv = silu_f(k) * __shfl_xor_sync(0xffffffffu, k, 16);
        if ((L.lane & 23) == 0)                          // lanes 0 and 8: gate of rows rr, rr+1
            a.h[(int64_t)en[u] * a.I + m.r0 + L.rr + (L.lane >> 3)] = hv;
    }
}

__global__ void __launch_bounds__(SW_THREADS, SW_CTAS_PER_SM) k_gateup_sw(GuArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint8_t* abuf = sm + GT_STAGES * GU_STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(abuf + NAB * GU_ABUF);
    uint64_t* empty = full + GT_STAGES;
    __shared__ TileMeta meta[RT];
    __shared__ int ent[RT][MAX_ACT];
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntr = a.I / GT_R;
    pdl_launch_dependents();                             // the successor may be scheduled now
    if (threadIdx.x == 0) {
        for (int s = 0; s < GT_STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, SW_CONSUMERS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    __syncthreads();
    pdl_wait();                                          // the work list and activations are complete
    if (a.stamp && threadIdx.x == 0) atomicMin(a.stamp, gtimer());
    const int ntiles = *a.n_items * ntr;
    const int64_t nblk = (int64_t)a.I * GU_NB;
    const bool producer = warp == SW_CONSUMERS;
    const GuLane GL(lane, warp);                         // consumer lane constants
    int j = 0;                                           // the CTA's tile counter (stage and phase)
    int n_issued = 0;                                    // producer: tiles issued (a prefix of the CTA's tiles)
    for (int base = 0;; base += RT) {
        const int nr = load_round<GT_ACT>(meta, ent, a.items, a.offsets, a.perm, ntiles, ntr, GT_R, base);
        if (nr == 0) break;
        if (producer) {
            if (lane == 0) {
                for (int i = 0; i < nr; ++i) {
                    const int s = (j + i) % GT_STAGES;
                    if (abort_flag) continue;
                    if (j + i >= GT_STAGES && !mbar_wait(empty + s, (((j + i) / GT_STAGES) - 1) & 1)) {
                        atomicOr(a.err, 2u);
                        abort_flag = 1;
                        continue;
                    }
                    const SlotPtrs m = slot_ptrs(a.lw, meta[i].slot);
                    const int64_t r0 = meta[i].r0;
                    uint8_t* st = sm + s * GU_STAGE;
                    mbar_expect_tx(full + s, GU_STAGE);
                    bulk_g2s(st, m.g + r0 * GU_QROW, GT_R * GU_QROW, full + s);
                    bulk_g2s(st + GT_R * GU_QROW, m.g + nblk * 128 + r0 * GU_HROW, GT_R * GU_HROW, full + s);
                    bulk_g2s(st + GU_MAT, m.u + r0 * GU_QROW, GT_R * GU_QROW, full + s);
                    bulk_g2s(st + GU_MAT + GT_R * GU_QROW, m.u + nblk * 128 + r0 * GU_HROW, GT_R * GU_HROW, full + s);
                    n_issued = j + i + 1;
                }
            }
        } else {
            const int ctid = threadIdx.x;                // 0 .. 255
            gu_stage_acts(a, meta, ent, 0, nr, abuf, ctid);
            gu_stage_acts(a, meta, ent, 1, nr, abuf + GU_ABUF, ctid);
            for (int i = 0; i < nr; ++i) {
                const int s = (j + i) % GT_STAGES;
                asm volatile("cp.async.wait_group 1;" ::: "memory");   // tile i's activations are in
                named_sync(1, 32 * SW_CONSUMERS);        // ... for every thread; buffer (i+2)%3 is free
                gu_stage_acts(a, meta, ent, i + 2, nr, abuf + ((i + 2) % NAB) * GU_ABUF, ctid);
                // after a timed-out wait anywhere in the CTA the consumers keep meeting at the named
                // barrier and releasing stages, but wait for and compute nothing more
                if (abort_flag || !mbar_wait(full + s, ((j + i) / GT_STAGES) & 1)) {
                    if (!abort_flag) atomicOr(a.err, 2u);
                    abort_flag = 1;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty + s);
                    continue;
                }
                const uint8_t* st = sm + s * GU_STAGE;
                const uint8_t* ab = abuf + (i % NAB) * GU_ABUF;
                const TileMeta m = meta[i];
                for (int e0 = 0; e0 < m.n; e0 += TG) {
                    const bool staged = e0 < GT_ACT;     // groups of TG lie wholly inside or outside
                    switch (min(TG, m.n - e0)) {
                    case 1: gu_group<1>(a, GL, st, ab, staged, ent[i], m, e0); break;
                    case 2: gu_group<2>(a, GL, st, ab, staged, ent[i], m, e0); break;
                    case 3: gu_group<3>(a, GL, st, ab, staged, ent[i], m, e0); break;
                    default: gu_group<4>(a, GL, st, ab, staged, ent[i], m, e0); break;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + s);
            }
            cp_async_wait_all();
        }
        j += nr;
        __syncthreads();                                 // the next round overwrites the metadata
    }
    // drain: every stage the producer issued completes before the CTA exits
    if (producer && lane == 0) {
        for (int q = n_issued - GT_STAGES > 0 ? n_issued - GT_STAGES : 0; q < n_issued; ++q)
            if (!mbar_wait(full + q % GT_STAGES, (q / GT_STAGES) & 1)) { atomicOr(a.err, 2u); break; }
    }
    if (a.stamp && threadIdx.x == 0) atomicMax(a.stamp + 1, gtimer());
}

// ---------------------------------------------------------------------------------------------
// down: y[ent][row] = down_row . h[ent] for every entry of the slot (I/256 = NBI <= 4)
// Stage (Q6_K): ql [R][NBI*128] | qh [R][NBI*64] | sc [R][NBI*16] | d [R][NBI*2]
// Stage (Q4_K): qs [R][NBI*128] | hdr [R][NBI*16]
// Activation buffer entry: q [I] in [block][piece a][unit q] order | bs [I/16 ints] | d [4 floats]
// ---------------------------------------------------------------------------------------------
struct DnArgs {
    LayerWeights lw;
    int H, I;
    const int* offsets;
    const int* perm;
    const int2* items;
    const int* n_items;
    const int8_t* hq;
    const float* hd;
    const int* hbs;
    float* y;
    unsigned* err;
    int stages, stage_bytes, aent;
    unsigned long long* stamp;                           // optional {first start, last end}
};

// piece p (16 bytes, 0..15) of a 256-block -> its position in the unit-interleaved shared layout
__device__ __forceinline__ int dn_piece_pos(int p, bool q6) {
    if (q6) {   // Q6_K unit v = 2*h2 + r reads pieces 8*h2 + r + 2*a (a = 0..3)
        const int h2 = p >> 3, r = p & 1, aa = (p >> 1) & 3;
        return 4 * aa + 2 * h2 + r;
    }
    return 4 * (p & 3) + (p >> 2);   // Q4_K group g reads pieces 4g + a
}

__device__ __forceinline__ void dn_stage_acts(const DnArgs& a, const TileMeta* meta, const int (*ent)[MAX_ACT], int i,
                                              int nr, uint8_t* buf, int ctid) {
    if (i < nr) {
        const int nb = a.I / QK;
        const bool q6 = (meta[i].slot < a.lw.n_slots ? a.lw.down_type : a.lw.sh_down_type) == T_Q6K;
        const int n = min(meta[i].n, DT_ACT);
        const int pq = a.I / 16, pb = a.I / 64;          // 16-byte pieces of q and of bs
        const int ppe = pq + pb + nb;                    // + one 4-byte copy per block scale
        for (int idx = ctid; idx < n * ppe; idx += 32 * SW_CONSUMERS) {
            const int e = idx / ppe, p = idx - e * ppe;
            const int en = ent[i][e];
            uint8_t* E = buf + e * a.aent;
            if (p < pq) {
                const int blk = p >> 4;
                cp_async16(E + blk * QK + 16 * dn_piece_pos(p & 15, q6), a.hq + (int64_t)en * a.I + 16 * p);
            } else if (p < pq + pb) {
                cp_async16(E + a.I + 16 * (p - pq),
                           reinterpret_cast<const uint8_t*>(a.hbs + (int64_t)en * (a.I / 16)) + 16 * (p - pq));
            } else {
                cp_async4(E + a.I + a.I / 4 + 4 * (p - pq - pb), a.hd + (int64_t)en * nb + (p - pq - pb));
            }
        }
    }
    cp_async_commit();
}

struct DnLane {
    int q, row, h2, r6;
    Q4Lane ql4;
    __device__ __forceinline__ DnLane(int lane, int warp) : ql4(lane & 3) {
        q = lane & 3;
        row = 8 * warp + (lane >> 2);                    // row within the tile
        h2 = q >> 1;                                     // Q6_K unit q = 2*h2 + r6
        r6 = q & 1;
    }
};

// Down rows of one tile for NT entries (a compile-time count): the lane's row, unit q of every block.
template <int NT>
__device__ __forceinline__ void dn_group(const DnArgs& a, const DnLane& L, const uint8_t* st, const uint8_t* ab, bool q6,
                                         bool staged, const int* ent_row, const TileMeta& m, int e0) {
    const int nb = a.I / QK, nbk = DT_R * nb;
    int en[NT];
    const uint8_t* E[NT];
#pragma unroll
    for (int u = 0; u < NT; ++u) {
        en[u] = staged ? ent_row[e0 + u] : a.perm[m.start + e0 + u];
        E[u] = ab + (e0 + u) * a.aent;
    }
    float acc[NT];
#pragma unroll
    for (int u = 0; u < NT; ++u) acc[u] = 0.f;
    for (int bb = 0; bb < nb; ++bb) {
        const int blk = L.row * nb + bb;
        if (q6) {
            const uint4 Aw = lds16(st + blk * 128 + 64 * L.h2 + 16 * L.r6);
            const uint4 Bw = lds16(st + blk * 128 + 64 * L.h2 + 32 + 16 * L.r6);
            const uint4 Cw = lds16(st + nbk * 128 + blk * 64 + 32 * L.h2 + 16 * L.r6);
            const uint4 Sw = lds16(st + nbk * 192 + blk * 16);
            const float d6 = h2f(*reinterpret_cast<const uint16_t*>(st + nbk * 208 + blk * 2));
            // the unit's four 16-weight groups aa = 0..3 use scales sc[8*h2 + r6 + 2*aa]
            const uint32_t s01 = L.h2 ? Sw.z : Sw.x, s23 = L.h2 ? Sw.w : Sw.y;
            const int sh = 8 * L.r6;
            const int sc0 = (int)(int8_t)(s01 >> sh), sc1 = (int)(int8_t)(s01 >> (sh + 16));
            const int sc2 = (int)(int8_t)(s23 >> sh), sc3 = (int)(int8_t)(s23 >> (sh + 16));
            uint32_t qv[4][4];
            const uint32_t Aa[4] = {Aw.x, Aw.y, Aw.z, Aw.w}, Ba[4] = {Bw.x, Bw.y, Bw.z, Bw.w};
            const uint32_t Ca[4] = {Cw.x, Cw.y, Cw.z, Cw.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                qv[0][k] = (Aa[k] & 0x0F0F0F0Fu) | ((Ca[k] << 4) & 0x30303030u);
                qv[1][k] = (Ba[k] & 0x0F0F0F0Fu) | ((Ca[k] << 2) & 0x30303030u);
                qv[2][k] = ((Aa[k] >> 4) & 0x0F0F0F0Fu) | (Ca[k] & 0x30303030u);
                qv[3][k] = ((Ba[k] >> 4) & 0x0F0F0F0Fu) | ((Ca[k] >> 2) & 0x30303030u);
            }
#pragma unroll
            for (int u = 0; u < NT; ++u) {
                int x[4][4];
                const int* bsb;
                float d8;
                if (staged) {                            // the unit's piece aa at 64*aa + 16*q
                    const int8_t* xb = reinterpret_cast<const int8_t*>(E[u] + bb * QK + 16 * L.q);
#pragma unroll
                    for (int aa = 0; aa < 4; ++aa) {
                        const int4 v = ldg16i(xb + 64 * aa);
                        x[aa][0] = v.x; x[aa][1] = v.y; x[aa][2] = v.z; x[aa][3] = v.w;
                    }
                    bsb = reinterpret_cast<const int*>(E[u] + a.I) + bb * 16 + 8 * L.h2;
                    d8 = reinterpret_cast<const float*>(E[u] + a.I + a.I / 4)[bb];
                } else {                                 // global: piece aa at 128*h2 + 16*r6 + 32*aa
                    const int8_t* xb = a.hq + (int64_t)en[u] * a.I + bb * QK + 128 * L.h2 + 16 * L.r6;
#pragma unroll
                    for (int aa = 0; aa < 4; ++aa) {
                        const int4 v = ldg16i(xb + 32 * aa);
                        x[aa][0] = v.x; x[aa][1] = v.y; x[aa][2] = v.z; x[aa][3] = v.w;
                    }
                    bsb = a.hbs + (int64_t)en[u] * (a.I / 16) + bb * 16 + 8 * L.h2;
                    d8 = a.hd[(int64_t)en[u] * nb + bb];
                }
                // partial sums of 16 of the groups aa = 0..3: ints r6, r6 + 2, r6 + 4, r6 + 6
                const int4 b0 = ldg16i(bsb), b1 = ldg16i(bsb + 4);
                const int bs0 = L.r6 ? b0.y : b0.x, bs1 = L.r6 ? b0.w : b0.z;
                const int bs2 = L.r6 ? b1.y : b1.x, bs3 = L.r6 ? b1.w : b1.z;
                int sa[4] = {0, 0, 0, 0};
#pragma unroll
                for (int aa = 0; aa < 4; ++aa)
#pragma unroll
                    for (int k = 0; k < 4; ++k) sa[aa] = __dp4a((int)qv[aa][k], x[aa][k], sa[aa]);
                const int is = sc0 * (sa[0] - 32 * bs0) + sc1 * (sa[1] - 32 * bs1) + sc2 * (sa[2] - 32 * bs2) +
                               sc3 * (sa[3] - 32 * bs3);
                acc[u] += d8 * d6 * (float)is;
            }
        } else {
            Q4Group gq;
            gq.set(lds16(st + blk * 128 + 32 * L.q), lds16(st + blk * 128 + 32 * L.q + 16));
            const Q4Scales sc = L.ql4.decode(lds16(st + nbk * 128 + blk * 16));
#pragma unroll
            for (int u = 0; u < NT; ++u) {
                Act64 A;
                if (staged) {                            // piece aa at 64*aa + 16*q
                    const int8_t* xb = reinterpret_cast<const int8_t*>(E[u] + bb * QK + 16 * L.q);
                    const int4 v0 = ldg16i(xb), v1 = ldg16i(xb + 64), v2 = ldg16i(xb + 128), v3 = ldg16i(xb + 192);
                    A.a[0] = v0.x; A.a[1] = v0.y; A.a[2] = v0.z; A.a[3] = v0.w;
                    A.a[4] = v1.x; A.a[5] = v1.y; A.a[6] = v1.z; A.a[7] = v1.w;
                    A.a[8] = v2.x; A.a[9] = v2.y; A.a[10] = v2.z; A.a[11] = v2.w;
                    A.a[12] = v3.x; A.a[13] = v3.y; A.a[14] = v3.z; A.a[15] = v3.w;
                    const int4 b = ldg16i(reinterpret_cast<const int*>(E[u] + a.I) + bb * 16 + 4 * L.q);
                    A.bs0 = b.x + b.y;
                    A.bs1 = b.z + b.w;
                    A.d8 = reinterpret_cast<const float*>(E[u] + a.I + a.I / 4)[bb];
                } else {
                    load_act64(A, a.hq + (int64_t)en[u] * a.I + bb * QK + 64 * L.q,
                               a.hbs + (int64_t)en[u] * (a.I / 16) + bb * 16 + 4 * L.q, a.hd + (int64_t)en[u] * nb + bb);
                }
                acc[u] += gq.dot(sc, A);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < NT; ++u) {
        float f = acc[u];
        f += __shfl_xor_sync(0xffffffffu, f, 1);
        f += __shfl_xor_sync(0xffffffffu, f, 2);
        if (L.q == 0) a.y[(int64_t)en[u] * a.H + m.r0 + L.row] = f;
    }
}

__global__ void __launch_bounds__(SW_THREADS, SW_CTAS_PER_SM) k_down_sw(DnArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int S = a.stages;
    uint8_t* abuf = sm + S * a.stage_bytes;
    const int abuf_bytes = DT_ACT * a.aent;
    uint64_t* full = reinterpret_cast<uint64_t*>(abuf + NAB * abuf_bytes);
    uint64_t* empty = full + S;
    __shared__ TileMeta meta[RT];
    __shared__ int ent[RT][MAX_ACT];
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = a.I / QK;
    const int ntr = a.H / DT_R;
    pdl_launch_dependents();                             // the successor may be scheduled now
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, SW_CONSUMERS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_flag = 0;
    }
    __syncthreads();
    pdl_wait();                                          // the work list and activations are complete
    if (a.stamp && threadIdx.x == 0) atomicMin(a.stamp, gtimer());
    const int ntiles = *a.n_items * ntr;
    const int64_t nblk = (int64_t)a.H * nb;
    const bool producer = warp == SW_CONSUMERS;
    const DnLane DL(lane, warp);
    const int nbk = DT_R * nb;                           // blocks in a tile
    int j = 0;
    int n_issued = 0;
    for (int base = 0;; base += RT) {
        const int nr = load_round<DT_ACT>(meta, ent, a.items, a.offsets, a.perm, ntiles, ntr, DT_R, base);
        if (nr == 0) break;
        if (producer) {
            if (lane == 0) {
                for (int i = 0; i < nr; ++i) {
                    const int s = (j + i) % S;
                    if (abort_flag) continue;
                    if (j + i >= S && !mbar_wait(empty + s, (((j + i) / S) - 1) & 1)) {
                        atomicOr(a.err, 2u);
                        abort_flag = 1;
                        continue;
                    }
                    const SlotPtrs m = slot_ptrs(a.lw, meta[i].slot);
                    uint8_t* st = sm + s * a.stage_bytes;
                    const int64_t b0 = (int64_t)meta[i].r0 * nb;
                    if (m.dt == T_Q6K) {
                        mbar_expect_tx(full + s, (unsigned)nbk * 210u);
                        bulk_g2s(st, m.d + b0 * 128, nbk * 128, full + s);
                        bulk_g2s(st + nbk * 128, m.d + nblk * 128 + b0 * 64, nbk * 64, full + s);
                        bulk_g2s(st + nbk * 192, m.d + nblk * 192 + b0 * 16, nbk * 16, full + s);
                        bulk_g2s(st + nbk * 208, m.d + nblk * 208 + b0 * 2, nbk * 2, full + s);
                    } else {
                        mbar_expect_tx(full + s, (unsigned)nbk * 144u);
                        bulk_g2s(st, m.d + b0 * 128, nbk * 128, full + s);
                        bulk_g2s(st + nbk * 128, m.d + nblk * 128 + b0 * 16, nbk * 16, full + s);
                    }
                    n_issued = j + i + 1;
                }
            }
        } else {
            const int ctid = threadIdx.x;
            dn_stage_acts(a, meta, ent, 0, nr, abuf, ctid);
            dn_stage_acts(a, meta, ent, 1, nr, abuf + abuf_bytes, ctid);
            for (int i = 0; i < nr; ++i) {
                const int s = (j + i) % S;
                asm volatile("cp.async.wait_group 1;" ::: "memory");
                named_sync(1, 32 * SW_CONSUMERS);
                dn_stage_acts(a, meta, ent, i + 2, nr, abuf + ((i + 2) % NAB) * abuf_bytes, ctid);
                if (abort_flag || !mbar_wait(full + s, ((j + i) / S) & 1)) {
                    if (!abort_flag) atomicOr(a.err, 2u);
                    abort_flag = 1;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty + s);
                    continue;
                }
                const uint8_t* st = sm + s * a.stage_bytes;
                const uint8_t* ab = abuf + (i % NAB) * abuf_bytes;
                const TileMeta m = meta[i];
                const bool q6 = (m.slot < a.lw.n_slots ? a.lw.down_type : a.lw.sh_down_type) == T_Q6K;
                for (int e0 = 0; e0 < m.n; e0 += TG) {
                    const bool staged = e0 < DT_ACT;     // groups of TG lie wholly inside or outside
                    switch (min(TG, m.n - e0)) {
                    case 1: dn_group<1>(a, DL, st, ab, q6, staged, ent[i], m, e0); break;
                    case 2: dn_group<2>(a, DL, st, ab, q6, staged, ent[i], m, e0); break;
                    case 3: dn_group<3>(a, DL, st, ab, q6, staged, ent[i], m, e0); break;
                    default: dn_group<4>(a, DL, st, ab, q6, staged, ent[i], m, e0); break;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + s);
            }
            cp_async_wait_all();
        }
        j += nr;
        __syncthreads();
    }
    if (producer && lane == 0) {
        for (int qq = n_issued - S > 0 ? n_issued - S : 0; qq < n_issued; ++qq)
            if (!mbar_wait(full + qq % S, (qq / S) & 1)) { atomicOr(a.err, 2u); break; }
    }
    if (a.stamp && threadIdx.x == 0) atomicMax(a.stamp + 1, gtimer());
}

int sw_grid(int ctas_per_sm = SW_CTAS_PER_SM) {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    return sms[dev] * ctas_per_sm;
}

}  // namespace

bool gateup_sw_supported(const Dims& d, const LayerWeights& lw) {
    if (d.H != QK * GU_NB || d.I % GT_R != 0) return false;
    if (lw.gate_type != T_Q4K || lw.up_type != T_Q4K) return false;
    if (lw.shared && (lw.sh_gate_type != T_Q4K || lw.sh_up_type != T_Q4K)) return false;
    return true;
}

bool down_sw_supported(const Dims& d, const LayerWeights& lw) {
    const int nb = d.I / QK;
    if (nb < 1 || nb > 4 || d.I % QK != 0 || d.H % DT_R != 0) return false;
    auto ok = [](int t) { return t == T_Q4K || t == T_Q6K; };
    if (!ok(lw.down_type) || (lw.shared && !ok(lw.sh_down_type))) return false;
    return true;
}

cudaError_t launch_gateup_sw(const Dims& d, const LayerWeights& lw, const Scratch& sc, int KK, cudaStream_t s,
                             unsigned long long* stamp) {
    static_assert(GU_SMEM % 8 == 0, "mbarrier alignment");
    cudaError_t e = cudaFuncSetAttribute(k_gateup_sw, cudaFuncAttributeMaxDynamicSharedMemorySize, GU_SMEM);
    if (e != cudaSuccess) return e;
    GuArgs a{lw, d.I, KK, sc.offsets, sc.perm, sc.items, sc.n_items, sc.fx_q, sc.fx_d, sc.fx_bs, sc.h, sc.sync, stamp};
    return launch_pdl(k_gateup_sw, sw_grid(), SW_THREADS, GU_SMEM, s, a);
}

cudaError_t launch_down_sw(const Dims& d, const LayerWeights& lw, const Scratch& sc, cudaStream_t s,
                           unsigned long long* stamp) {
    const int nb = d.I / QK;
    DnArgs a{lw, d.H, d.I, sc.offsets, sc.perm, sc.items, sc.n_items, sc.h_q, sc.h_d, sc.h_bs, sc.y, sc.sync, 0, 0, 0, stamp};
    a.stage_bytes = DT_R * nb * 210;                     // sized for Q6_K (Q4_K tiles use 144 per block)
    a.aent = d.I + d.I / 4 + 16;
    const int fixed = NAB * DT_ACT * a.aent;
    // SW_CTAS_PER_SM CTAs per SM where two pipeline stages fit their share of shared memory (I <= 768
    // with two CTAs), else one CTA per SM with the whole of it
    int per_sm = SW_CTAS_PER_SM;
    a.stages = (sw_dyn(per_sm) - fixed - 2 * 4 * 8) / a.stage_bytes;
    if (a.stages < 2 && per_sm > 1) {
        per_sm = 1;
        a.stages = (sw_dyn(1) - fixed - 2 * 4 * 8) / a.stage_bytes;
    }
    if (a.stages > 4) a.stages = 4;
    if (a.stages < 2) return cudaErrorInvalidValue;
    const int smem = a.stages * a.stage_bytes + fixed + 2 * a.stages * 8;
    cudaError_t e = cudaFuncSetAttribute(k_down_sw, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_down_sw, sw_grid(per_sm), SW_THREADS, smem, s, a);
}

}  // namespace hoard
