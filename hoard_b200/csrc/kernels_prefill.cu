// kernels_prefill.cu -- token-sorted grouped expert GEMM on the 5th-generation tensor cores, for the
// prefill / batched path (hoard's mul_mat_id form, src/run_specloop.cpp:125-140, src/run_m1.cpp:93-108).
//
// After routing, the (token, j) entries are counting-sorted by pool slot (k_dispatch). A work item is
// (slot, 128-entry M tile, 256-wide N block). One persistent CTA per SM runs items with three roles:
//   warp 0      one thread issues tcgen05.mma (kind::f16, M=128, N=256, K=16) with f32 accumulators
//               in tensor memory (TMEM);
//   warps 1-4   gather the A rows (f16 activations, one row per sorted entry) into 128B-swizzled
//               shared memory with cp.async, zero-filling the rows past the slot's entries;
//   warps 5-12  dequantise the B rows (Q4_K / Q6_K expert weights, one row per thread) to f16 in
//               registers and store them 128B-swizzled into shared memory; after the K loop of an item
//               they are the epilogue, reading the accumulators with tcgen05.ld.
// gate/up (MODE 0): gate and up accumulators (128 x 256 f32 each) fill all 512 TMEM columns; the
//   epilogue forms h = silu(g) * u and quantises each row's 256 values -- one Q8_K block of h, as
//   ggml's CPU backend quantises the down projection's input -- storing q * d as f16.
// down (MODE 1): one accumulator; the epilogue writes each entry's 256 output columns (f32) to the
//   per-entry buffer that the deterministic combine (k_combine) sums in expert order j.
// A operands are Q8_K-dequantised activations (q * d rounded once to f16) and B operands the
// dequantised weights rounded to f16, accumulated in f32: ggml's quantised matmul up to f16 rounding
// of the two operands (f16 rather than bf16: same tensor-core rate, three more mantissa bits).
// Every wait is bounded by %globaltimer; on expiry the CTA records an error bit, skips all further
// work, waits (bounded) for its own tensor-core and copy operations and frees its tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <cuda_fp16.h>

namespace hoard {

namespace {

constexpr int TC_THREADS = 416;           // 13 warps
constexpr int TC_M = 128;                 // rows of an M tile (UMMA M)
constexpr int TC_N = 256;                 // columns of an N block (UMMA N)
constexpr int TC_KC = 64;                 // K per pipeline stage: one 128-byte f16 row segment
constexpr int A_THREADS = 128;            // warps 1-4
constexpr int B_THREADS = 256;            // warps 5-12
constexpr int A_TID0 = 32, B_TID0 = 160;
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned su32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t* b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_test(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(su32(b)), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
// Bounded wait for the phase with this parity. Returns false at once when the CTA has given up, and
// gives up (sets the flag) after TC_WAIT_NS.
__device__ __forceinline__ bool bar_wait(uint64_t* b, unsigned parity, volatile int* abort_flag) {
    if (*abort_flag) return false;
    if (bar_test(b, parity)) return true;
    const unsigned long long t0 = gtime();
    while (!bar_test(b, parity)) {
        if (*abort_flag) return false;
        if (gtime() - t0 > TC_WAIT_NS) { *abort_flag = 1; return false; }
    }
    return true;
}
// Bounded wait that ignores the give-up flag (used to drain in-flight work before exit).
__device__ __forceinline__ void bar_drain(uint64_t* b, unsigned parity) {
    const unsigned long long t0 = gtime();
    while (!bar_test(b, parity) && gtime() - t0 < TC_WAIT_NS) {}
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, unsigned src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor of a K-major, 128B-swizzled operand tile (rows of 128 bytes, 8-row
// atoms of 1024 bytes, tile base 1024-byte aligned): start >> 4, leading offset 1 (unused by swizzled
// K-major layouts), stride offset 1024 B between 8-row atoms, version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    const uint64_t start = (su32(tile) >> 4) & 0x3FFFu;
    return start | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: D f32 (bits 4-5 = 1), A and B f16 (bits 7-9, 10-12 = 0), both K-major
// (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(TC_IDESC), "r"(accumulate)
        : "memory");
}
// arrives on the mbarrier once every tcgen05 operation this thread issued before it has completed
__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
                 : "memory");
}

// 32 TMEM lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantisation of one 64-weight segment of a weight row to 64 f16 (8 x 16 bytes) ----------
// 0x6400 | q is the f16 value 1024 + q exactly (q < 1024); subtracting 1024 recovers q exactly.
__device__ __forceinline__ __half2 h2bits(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ uint32_t bits_h2(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

template <int TYPE> struct Seg;

// Q4_K segment g (0..3) of a block = qs bytes [32g, 32g+32): low nibbles are weights [64g, 64g+32)
// (sub-block 2g), high nibbles weights [64g+32, 64g+64) (sub-block 2g+1). w = d*sc*q - dmin*m.
template <> struct Seg<T_Q4K> {
    uint4 q0, q1, hdr;
    __device__ __forceinline__ void load(const uint8_t* base, int64_t nblk_total, int64_t blk, int g) {
        const uint8_t* qs = base + blk * 128 + 32 * g;
        q0 = ld16(qs);
        q1 = ld16(qs + 16);
        hdr = ld16(base + nblk_total * 128 + blk * 16);
    }
    __device__ __forceinline__ void dequant(int g, uint4 out[8]) const {
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
        int sc0, m0, sc1, m1;
        q4k_scale_min(hdr, 2 * g, sc0, m0);
        q4k_scale_min(hdr, 2 * g + 1, sc1, m1);
        const __half2 k1024 = __float2half2_rn(1024.f);
        const __half2 dl = __float2half2_rn(d * (float)sc0), ml = __float2half2_rn(-dmin * (float)m0);
        const __half2 dh = __float2half2_rn(d * (float)sc1), mh = __float2half2_rn(-dmin * (float)m1);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // word i = qs bytes 4i..4i+3: weights 4i..4i+3 (low nibbles), 32+4i..32+4i+3 (high)
            const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
            uint32_t* lc = reinterpret_cast<uint32_t*>(&out[i >> 1]) + 2 * (i & 1);
            uint32_t* hc = reinterpret_cast<uint32_t*>(&out[4 + (i >> 1)]) + 2 * (i & 1);
            lc[0] = bits_h2(__hfma2(__hsub2(h2bits(__byte_perm(lo, 0x64646464u, 0x4140)), k1024), dl, ml));
            lc[1] = bits_h2(__hfma2(__hsub2(h2bits(__byte_perm(lo, 0x64646464u, 0x4342)), k1024), dl, ml));
            hc[0] = bits_h2(__hfma2(__hsub2(h2bits(__byte_perm(hi, 0x64646464u, 0x4140)), k1024), dh, mh));
            hc[1] = bits_h2(__hfma2(__hsub2(h2bits(__byte_perm(hi, 0x64646464u, 0x4342)), k1024), dh, mh));
        }
    }
};

// Q6_K segment s (0..3) = weights [64s, 64s+64) of the block = runs a = 2(s&1), 2(s&1)+1 of half
// h2 = s/2. Run a, element l (0..31): low bits from ql[64h2 + 32(a&1) + l] (low nibble for a < 2,
// high for a >= 2), high bits = bits 2a..2a+1 of qh[32h2 + l], scale sc[8h2 + 2a + l/16];
// w = d * sc * (q - 32).
template <> struct Seg<T_Q6K> {
    uint4 la0, la1, lb0, lb1, h0, h1, sc;
    unsigned short d;
    __device__ __forceinline__ void load(const uint8_t* base, int64_t nblk_total, int64_t blk, int s) {
        const int h2 = s >> 1;
        const uint8_t* ql = base + blk * 128 + 64 * h2;
        la0 = ld16(ql);
        la1 = ld16(ql + 16);
        lb0 = ld16(ql + 32);
        lb1 = ld16(ql + 48);
        const uint8_t* qh = base + nblk_total * 128 + blk * 64 + 32 * h2;
        h0 = ld16(qh);
        h1 = ld16(qh + 16);
        sc = ld16(base + nblk_total * 192 + blk * 16);
        d = *reinterpret_cast<const unsigned short*>(base + nblk_total * 208 + blk * 2);
    }
    __device__ __forceinline__ void dequant(int s, uint4 out[8]) const {
        const int h2 = s >> 1, a0 = 2 * (s & 1);
        const float df = __half2float(__ushort_as_half(d));
        const __half2 k1056 = __float2half2_rn(1056.f);   // 1024 + 32
        const uint32_t qhw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int a = a0 + r;
            const uint4& p0 = (a & 1) ? lb0 : la0;
            const uint4& p1 = (a & 1) ? lb1 : la1;
            const uint32_t qlw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            const int nib = a >= 2 ? 4 : 0;
            const __half2 s0 = __float2half2_rn(df * (float)sbyte(sc, 8 * h2 + 2 * a));
            const __half2 s1 = __float2half2_rn(df * (float)sbyte(sc, 8 * h2 + 2 * a + 1));
#pragma unroll
            for (int i = 0; i < 8; ++i) {   // elements l = 4i..4i+3 -> chunk 4r + i/2
                const uint32_t q = ((qlw[i] >> nib) & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * a)) & 0x03030303u) << 4);
                const __half2 scl = i < 4 ? s0 : s1;
                uint32_t* c = reinterpret_cast<uint32_t*>(&out[4 * r + (i >> 1)]) + 2 * (i & 1);
                c[0] = bits_h2(__hmul2(__hsub2(h2bits(__byte_perm(q, 0x64646464u, 0x4140)), k1056), scl));
                c[1] = bits_h2(__hmul2(__hsub2(h2bits(__byte_perm(q, 0x64646464u, 0x4342)), k1056), scl));
            }
        }
    }
};

// 64 f16 of row r into a 128B-swizzled tile: 16-byte chunk c of the row lands at chunk c ^ (r % 8)
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int r, const uint4 v[8]) {
    uint8_t* row = tile + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = v[c];
}

}  // namespace

struct TcArgs {
    LayerWeights lw;
    int H, I, KK;
    const int* offsets;     // [NS+1] sorted-entry offset of each slot
    const int* perm;        // sorted position -> entry id t*KK + j
    const int2* items;      // (slot, M tile) per M tile
    const int* n_items;     // device count of M tiles (N blocks are expanded in the kernel)
    const __half* A;        // MODE 0: Q8_K-dequantised activations [T][H]; MODE 1: h [P][I] (sorted)
    __half* hq;             // MODE 0 output [P][I] (sorted order)
    float* y;               // MODE 1 output [entries][H] by entry id
    unsigned* err;
};

template <int MODE, int TYPE>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc_experts(TcArgs a) {
    constexpr int NMAT = MODE == 0 ? 2 : 1;
    constexpr int STAGES = MODE == 0 ? 2 : 3;
    constexpr int A_BYTES = TC_M * 128;                    // 16 KiB
    constexpr int B_BYTES = TC_N * 128;                    // 32 KiB per matrix
    constexpr int STAGE_BYTES = A_BYTES + NMAT * B_BYTES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full_bar[STAGES], empty_bar[STAGES], acc_full, acc_empty, done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    __shared__ float s_amax[2][TC_M];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = MODE == 0 ? a.H : a.I;                   // reduction length
    const int NOUT = MODE == 0 ? a.I : a.H;                // output rows of the weight matrix
    const int KC = K / TC_KC;
    const int NBLK = NOUT / TC_N;
    const int nbK = K / QK;
    const int64_t nblk_total = (int64_t)NOUT * nbK;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&full_bar[s], A_THREADS + B_THREADS);
            bar_init(&empty_bar[s], 1);
        }
        bar_init(&acc_full, 1);
        bar_init(&acc_empty, B_THREADS);
        bar_init(&done_bar, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&s_tmem)),
                     "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int n_items = *a.n_items * NBLK;

    int item_no = 0;   // items this CTA has run; stage counter = item_no * KC + kc in every role
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++item_no) {
        const int2 it = a.items[item / NBLK];
        const int nb_out = item - (item / NBLK) * NBLK;
        const int slot = it.x;
        const int row0 = a.offsets[slot] + it.y * TC_M;
        const int nrows = min(TC_M, a.offsets[slot + 1] - row0);
        const uint32_t it0 = (uint32_t)item_no * (uint32_t)KC;

        if (warp == 0) {
            // ---------------- MMA issuer ----------------
            if (lane == 0) {
                bool ok = item_no == 0 || bar_wait(&acc_empty, (item_no - 1) & 1, &s_abort);
                tc_fence_after();
                for (int kc = 0; kc < KC && ok; ++kc) {
                    const uint32_t st_it = it0 + kc;
                    const int s = st_it % STAGES;
                    if (!bar_wait(&full_bar[s], (st_it / STAGES) & 1, &s_abort)) { ok = false; break; }
                    fence_async_smem();
                    tc_fence_after();
                    const uint8_t* st = smem + s * STAGE_BYTES;
                    const uint64_t ad = sw128_desc(st);
                    const uint64_t bd0 = sw128_desc(st + A_BYTES);
                    const uint64_t bd1 = sw128_desc(st + A_BYTES + B_BYTES);
#pragma unroll
                    for (int ks = 0; ks < TC_KC / 16; ++ks) {   // +32 bytes of K = +2 in the descriptor
                        const uint32_t acc = (kc > 0 || ks > 0) ? 1u : 0u;
                        umma_f16(tmem, ad + 2 * ks, bd0 + 2 * ks, acc);
                        if (MODE == 0) umma_f16(tmem + TC_N, ad + 2 * ks, bd1 + 2 * ks, acc);
                    }
                    umma_commit(&empty_bar[s]);      // stage s is free once these MMAs have read it
                }
                if (ok) umma_commit(&acc_full);      // accumulators complete
            }
            __syncwarp();
        } else if (warp < 5) {
            // ---------------- A gather: thread = (16-byte chunk c, rows rg, rg+16, ...) ----------------
            const int t = tid - A_TID0;
            const int c = t & 7, rg = t >> 3;
            const __half* src[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = rg + 16 * i;
                src[i] = nullptr;
                if (r < nrows) {
                    const int sp = row0 + r;
                    src[i] = MODE == 0 ? a.A + (int64_t)(a.perm[sp] / a.KK) * a.H : a.A + (int64_t)sp * a.I;
                }
            }
            for (int kc = 0; kc < KC; ++kc) {
                const uint32_t st_it = it0 + kc;
                const int s = st_it % STAGES;
                const uint32_t round = st_it / STAGES;
                if (round > 0 && !bar_wait(&empty_bar[s], (round - 1) & 1, &s_abort)) break;
                if (s_abort) break;
                uint8_t* tile = smem + s * STAGE_BYTES;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = rg + 16 * i;
                    const void* g = src[i] ? (const void*)(src[i] + kc * TC_KC + c * 8) : (const void*)a.A;
                    cp_async16(tile + r * 128 + ((c ^ (r & 7)) << 4), g, src[i] ? 16u : 0u);
                }
                cp_async_arrive_noinc(&full_bar[s]);
            }
        } else {
            // ---------------- B dequant (256 threads), then the epilogue ----------------
            const int r = tid - B_TID0;                          // B row within the N block
            const int64_t n = (int64_t)nb_out * TC_N + r;        // weight row
            const bool sh = slot >= a.lw.n_slots;
            const uint8_t* base = sh ? a.lw.shared : a.lw.pool + (int64_t)slot * a.lw.slot_stride;
            const uint8_t* m0 = MODE == 0 ? base : base + (sh ? a.lw.sh_off_down : a.lw.off_down);
            const uint8_t* m1 = base + (sh ? a.lw.sh_off_up : a.lw.off_up);
            Seg<TYPE> nx0, nx1;
            nx0.load(m0, nblk_total, n * nbK, 0);
            if (MODE == 0) nx1.load(m1, nblk_total, n * nbK, 0);
            for (int kc = 0; kc < KC; ++kc) {
                const uint32_t st_it = it0 + kc;
                const int s = st_it % STAGES;
                const uint32_t round = st_it / STAGES;
                const Seg<TYPE> cur0 = nx0, cur1 = nx1;
                if (kc + 1 < KC) {                               // prefetch the next segment's bytes
                    const int64_t blk = n * nbK + ((kc + 1) >> 2);
                    nx0.load(m0, nblk_total, blk, (kc + 1) & 3);
                    if (MODE == 0) nx1.load(m1, nblk_total, blk, (kc + 1) & 3);
                }
                uint4 v[8];
                cur0.dequant(kc & 3, v);
                if (round > 0 && !bar_wait(&empty_bar[s], (round - 1) & 1, &s_abort)) break;
                if (s_abort) break;
                uint8_t* tile = smem + s * STAGE_BYTES + A_BYTES;
                store_row_sw128(tile, r, v);
                if (MODE == 0) {
                    cur1.dequant(kc & 3, v);
                    store_row_sw128(tile + B_BYTES, r, v);
                }
                fence_async_smem();
                bar_arrive(&full_bar[s]);
            }
            // ---- epilogue: warp % 4 selects the TMEM lane quarter, (warp - 5) / 4 the column half ----
            const bool ok = __all_sync(0xFFFFFFFFu, bar_wait(&acc_full, item_no & 1, &s_abort));
            const int q = warp & 3, half = (warp - 5) >> 2;
            const int m = 32 * q + lane;                          // accumulator row = tile row
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
            const bool valid = m < nrows;
            if (ok) tc_fence_after();
            if (MODE == 0) {
                float amax = 0.f;
                float g[32], u[32];
                if (ok) {
#pragma unroll 1
                    for (int cc = 0; cc < 4; ++cc) {
                        const int col = 128 * half + 32 * cc;
                        tmem_ld32(lane_base + col, g);
                        tmem_ld32(lane_base + TC_N + col, u);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            amax = fmaxf(amax, fabsf(__fdividef(g[i], 1.0f + __expf(-g[i])) * u[i]));
                    }
                }
                s_amax[half][m] = amax;
                asm volatile("bar.sync 1, 256;" ::: "memory");
                amax = fmaxf(s_amax[0][m], s_amax[1][m]);
                const float iscale = amax != 0.f ? 127.f / amax : 0.f;
                const float d8 = amax != 0.f ? 1.f / iscale : 0.f;
                if (ok) {
#pragma unroll 1
                    for (int cc = 0; cc < 4; ++cc) {
                        const int col = 128 * half + 32 * cc;
                        tmem_ld32(lane_base + col, g);
                        tmem_ld32(lane_base + TC_N + col, u);
                        uint32_t pk[16];
#pragma unroll
                        for (int i = 0; i < 32; i += 2) {
                            const float h0 = __fdividef(g[i], 1.0f + __expf(-g[i])) * u[i];
                            const float h1 = __fdividef(g[i + 1], 1.0f + __expf(-g[i + 1])) * u[i + 1];
                            const int q0 = min(127, __float2int_rn(iscale * h0));
                            const int q1 = min(127, __float2int_rn(iscale * h1));
                            pk[i >> 1] = bits_h2(__floats2half2_rn((float)q0 * d8, (float)q1 * d8));
                        }
                        if (valid) {
                            uint4* dst = reinterpret_cast<uint4*>(a.hq + (int64_t)(row0 + m) * a.I +
                                                                  (int64_t)nb_out * TC_N + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
                        }
                    }
                }
                asm volatile("bar.sync 1, 256;" ::: "memory");   // s_amax is reused by the next item
            } else if (ok) {
                const int entry = valid ? a.perm[row0 + m] : 0;
                float v[32];
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    const int col = 128 * half + 32 * cc;
                    tmem_ld32(lane_base + col, v);
                    if (valid) {
                        float4* dst = reinterpret_cast<float4*>(a.y + (int64_t)entry * a.H + (int64_t)nb_out * TC_N + col);
#pragma unroll
                        for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    }
                }
            }
            tc_fence_before();
            bar_arrive(&acc_empty);
        }
    }
    // ---- teardown: drain this CTA's tensor-core ops and copies, then free the tensor memory ----
    if (warp == 0 && lane == 0) {
        umma_commit(&done_bar);
        bar_drain(&done_bar, 0);
    }
    if (warp >= 1 && warp < 5) asm volatile("cp.async.wait_all;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    if (s_abort && tid == 0) atomicOr(a.err, 2u);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// Work list: one (slot, M tile) item per 128 sorted entries of each slot.
__global__ void k_tc_items(const int* __restrict__ offsets, int NS, int2* __restrict__ items, int* __restrict__ n_items,
                           int max_items) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int n = 0;
    for (int s = 0; s < NS; ++s) {
        const int cnt = offsets[s + 1] - offsets[s];
        for (int mt = 0; mt * TC_M < cnt && n < max_items; ++mt) items[n++] = make_int2(s, mt);
    }
    *n_items = n;
}

// ggml's Q8_K of rows [R][K] (256-value blocks, iscale = 127 / max|x|, round to nearest even, clamp
// 127), written back as f16(q * d): the activation operand of the tensor-core GEMMs.
__global__ void __launch_bounds__(256) k_q8_to_f16(const float* __restrict__ x, int K, __half* __restrict__ out) {
    __shared__ float red[8];
    const int nseg = K / QK;
    const int64_t r = blockIdx.x / nseg;
    const int seg = (int)(blockIdx.x - r * nseg);
    const float v = x[r * K + seg * QK + threadIdx.x];
    float am = warp_max(fabsf(v));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
    __syncthreads();
    am = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) am = fmaxf(am, red[i]);
    float o = 0.f;
    if (am != 0.f) {
        const float iscale = 127.f / am;
        const int q = min(127, __float2int_rn(iscale * v));
        o = (float)q * (1.f / iscale);
    }
    out[r * K + seg * QK + threadIdx.x] = __float2half_rn(o);
}

namespace {

int tc_grid() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

constexpr size_t tc_smem(int mode) {
    return (mode == 0 ? 2 * ((size_t)TC_M * 128 + 2 * (size_t)TC_N * 128)
                      : 3 * ((size_t)TC_M * 128 + (size_t)TC_N * 128)) +
           1024;   // + slack to align the tiles to the 1024-byte swizzle atoms
}

template <int MODE, int TYPE>
cudaError_t launch_tc(const TcArgs& a, cudaStream_t s) {
    static unsigned long long attr_set = 0;   // devices on which the shared-memory limit was raised
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(attr_set >> dev & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_tc_experts<MODE, TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc_smem(MODE));
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set |= 1ull << dev;
    }
    k_tc_experts<MODE, TYPE><<<tc_grid(), TC_THREADS, tc_smem(MODE), s>>>(a);
    return cudaGetLastError();
}

}  // namespace

bool tc_supported(const Dims& d, const LayerWeights& lw) {
    if (d.H % TC_N || d.I % TC_N) return false;
    auto q = [](int t) { return t == T_Q4K || t == T_Q6K; };
    if (!q(lw.gate_type) || lw.up_type != lw.gate_type || !q(lw.down_type)) return false;
    if (lw.shared && (lw.sh_gate_type != lw.gate_type || lw.sh_up_type != lw.up_type ||
                      lw.sh_down_type != lw.down_type))
        return false;
    return true;
}

int64_t tc_max_items(int T, int KK, int n_slots) { return ((int64_t)T * KK + TC_M - 1) / TC_M + n_slots + 1; }

cudaError_t launch_experts_tc(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                              const int32_t* slot_of_sel, const float* w, void* x_inout, int T, cudaStream_t s,
                              int* launches) {
    const bool shared = lw.shared != nullptr;
    const int KK = d.k + (shared ? 1 : 0);
    const int NS = lw.n_slots + (shared ? 1 : 0);
    int nl = 0;
    cudaError_t e;
    // 1. ggml's Q8_K of fx, as f16 (q * d) rows
    k_q8_to_f16<<<(unsigned)((d.H / QK) * T), 256, 0, s>>>(fx, d.H, reinterpret_cast<__half*>(sc.xq16));
    ++nl;
    if (shared) {
        if ((e = launch_shared_gate(fx, lw.sh_gate_inp, d.H, T, sc.sh_gate, s)) != cudaSuccess) return e;
        ++nl;
    }
    // 2. counting sort of the entries by slot, and the (slot, M tile) work list
    if ((e = launch_dispatch(slot_of_sel, T, d.k, KK, lw.n_slots, sc, s)) != cudaSuccess) return e;
    ++nl;
    k_tc_items<<<1, 32, 0, s>>>(sc.offsets, NS, sc.items, sc.n_items, (int)tc_max_items(T, KK, lw.n_slots));
    ++nl;
    // 3. gate/up + SwiGLU + Q8_K(h); 4. down
    TcArgs a{};
    a.lw = lw;
    a.H = d.H;
    a.I = d.I;
    a.KK = KK;
    a.offsets = sc.offsets;
    a.perm = sc.perm;
    a.items = sc.items;
    a.n_items = sc.n_items;
    a.err = sc.sync;
    a.A = reinterpret_cast<const __half*>(sc.xq16);
    a.hq = reinterpret_cast<__half*>(sc.hq16);
    e = lw.gate_type == T_Q4K ? launch_tc<0, T_Q4K>(a, s) : launch_tc<0, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    ++nl;
    a.A = reinterpret_cast<const __half*>(sc.hq16);
    a.y = sc.y;
    e = lw.down_type == T_Q4K ? launch_tc<1, T_Q4K>(a, s) : launch_tc<1, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    ++nl;
    // 5. weighted combine into the residual, j ascending (shared with the grouped path)
    if ((e = launch_combine(d, sc, w, x_inout, T, KK, s)) != cudaSuccess) return e;
    ++nl;
    if (launches) *launches += nl;
    return cudaSuccess;
}

}  // namespace hoard
