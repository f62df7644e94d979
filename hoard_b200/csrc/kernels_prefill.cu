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
// The file also holds the router GEMM of large batches on the same tensor cores (k_router_tc).
#include "common.cuh"
#include "kernels.h"

#include <cuda_fp16.h>

namespace hoard {

namespace {

// warps: 0 MMA issuer, 1-4 A gather, 5-12 B dequant (+ the gate/up epilogue), 13-16 down epilogue
constexpr int tc_threads(int mode) { return mode == 0 ? 416 : 544; }
constexpr int EPI_THREADS = 128;          // down epilogue warps 13-16
constexpr int EPI_TID0 = 416;
constexpr int TC_M = 128;                 // rows of an M tile (UMMA M)
constexpr int TC_N = 256;                 // columns of an N block (UMMA N)
constexpr int TC_KC = 64;                 // K per pipeline stage: one 128-byte f16 row segment
constexpr int A_THREADS = 128;            // warps 1-4
constexpr int B_THREADS = 256;            // warps 5-12
constexpr int A_TID0 = 32, B_TID0 = 160;
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;
// phase stamps (%globaltimer) of the first CTAs' first two items: 0 MMA saw the stage full, 1 MMA
// committed it, 2 B-row 0 starts dequantising, 3 B-row 0 saw the stage empty, 4 B-row 0 arrived,
// 5 A-thread 0 saw the stage empty, 6 A-thread 0 issued its copies; stage 0 / 1 of slot 7 =
// epilogue start / end.
constexpr int TC_TRACE_CTAS = 4, TC_TRACE_ITEMS = 2, TC_TRACE_STAGES = 32, TC_TRACE_SLOTS = 8;

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
// non-blocking probe of the phase with this parity
__device__ __forceinline__ bool bar_peek(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(su32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait for the phase with this parity. Returns false when the CTA has given up, and gives up
// (sets the flag) after TC_WAIT_NS.
__device__ __forceinline__ bool bar_wait(uint64_t* b, unsigned parity, volatile int* abort_flag) {
    if (bar_test(b, parity)) return !*abort_flag;
    if (*abort_flag) return false;
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

// A B thread owns one weight row. Per 64-weight segment (one pipeline stage) the row's quantised
// bytes are copied with cp.async into a shared-memory ring several stages ahead of use (chunk-major:
// 16-byte chunk c of row r at c * 4096 + r * 16, so a warp's reads are conflict-free); the per-block
// scale words are read into registers one block (four stages) ahead.
template <int TYPE> struct Seg;

// Q4_K segment g (0..3) of a block = qs bytes [32g, 32g+32): low nibbles are weights [64g, 64g+32)
// (sub-block 2g), high nibbles weights [64g+32, 64g+64) (sub-block 2g+1). w = d*sc*q - dmin*m.
template <> struct Seg<T_Q4K> {
    static constexpr int RAW_CH = 2;                       // 16-byte chunks per row and stage
    struct Hdr { uint4 h; };
    uint4 q0, q1;
    static __device__ __forceinline__ Hdr load_hdr(const uint8_t* base, int64_t nblk_total, int64_t blk) {
        return Hdr{ld16(base + nblk_total * 128 + blk * 16)};
    }
    static __device__ __forceinline__ void issue(uint8_t* ring, int r, const uint8_t* base, int64_t nblk_total,
                                                 int64_t blk, int g) {
        (void)nblk_total;
        const uint8_t* qs = base + blk * 128 + 32 * g;
        cp_async16(ring + r * 16, qs, 16u);
        cp_async16(ring + 4096 + r * 16, qs + 16, 16u);
    }
    __device__ __forceinline__ void read(const uint8_t* ring, int r) {
        q0 = *reinterpret_cast<const uint4*>(ring + r * 16);
        q1 = *reinterpret_cast<const uint4*>(ring + 4096 + r * 16);
    }
    __device__ __forceinline__ void dequant(int g, const Hdr& hd, uint4 out[8]) const {
        const uint4& hdr = hd.h;
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
    static constexpr int RAW_CH = 6;                       // ql 64 bytes + qh 32 bytes
    struct Hdr { uint4 sc; unsigned short d; };
    uint4 la0, la1, lb0, lb1, h0, h1;
    static __device__ __forceinline__ Hdr load_hdr(const uint8_t* base, int64_t nblk_total, int64_t blk) {
        Hdr h;
        h.sc = ld16(base + nblk_total * 192 + blk * 16);
        h.d = *reinterpret_cast<const unsigned short*>(base + nblk_total * 208 + blk * 2);
        return h;
    }
    static __device__ __forceinline__ void issue(uint8_t* ring, int r, const uint8_t* base, int64_t nblk_total,
                                                 int64_t blk, int s) {
        const int h2 = s >> 1;
        const uint8_t* ql = base + blk * 128 + 64 * h2;
        const uint8_t* qh = base + nblk_total * 128 + blk * 64 + 32 * h2;
#pragma unroll
        for (int c = 0; c < 4; ++c) cp_async16(ring + c * 4096 + r * 16, ql + 16 * c, 16u);
        cp_async16(ring + 4 * 4096 + r * 16, qh, 16u);
        cp_async16(ring + 5 * 4096 + r * 16, qh + 16, 16u);
    }
    __device__ __forceinline__ void read(const uint8_t* ring, int r) {
        la0 = *reinterpret_cast<const uint4*>(ring + r * 16);
        la1 = *reinterpret_cast<const uint4*>(ring + 4096 + r * 16);
        lb0 = *reinterpret_cast<const uint4*>(ring + 2 * 4096 + r * 16);
        lb1 = *reinterpret_cast<const uint4*>(ring + 3 * 4096 + r * 16);
        h0 = *reinterpret_cast<const uint4*>(ring + 4 * 4096 + r * 16);
        h1 = *reinterpret_cast<const uint4*>(ring + 5 * 4096 + r * 16);
    }
    __device__ __forceinline__ void dequant(int s, const Hdr& hd, uint4 out[8]) const {
        const int h2 = s >> 1, a0 = 2 * (s & 1);
        const float df = __half2float(__ushort_as_half(hd.d));
        const __half2 k1056 = __float2half2_rn(1056.f);   // 1024 + 32
        const uint32_t qhw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int a = a0 + r;
            const uint4& p0 = (a & 1) ? lb0 : la0;
            const uint4& p1 = (a & 1) ? lb1 : la1;
            const uint32_t qlw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            const int nib = a >= 2 ? 4 : 0;
            const __half2 s0 = __float2half2_rn(df * (float)sbyte(hd.sc, 8 * h2 + 2 * a));
            const __half2 s1 = __float2half2_rn(df * (float)sbyte(hd.sc, 8 * h2 + 2 * a + 1));
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

// Shared-memory plan of one CTA: an A ring (f16 activation tiles, 16 KiB per stage), a B ring
// (dequantised f16 weight tiles, 32 KiB per matrix and stage) and the raw-byte ring of the B rows.
// A has its own, deeper ring because its tiles come from L2 with ~1.3 us of latency under load,
// while a stage of MMAs takes ~0.3-0.6 us.
struct TcCfg {
    int a, b, raw;   // stages of the A ring, the B ring, the raw-byte ring
};
constexpr int TC_A_BYTES = TC_M * 128;
constexpr int tc_b_bytes(int mode) { return (mode == 0 ? 2 : 1) * TC_N * 128; }
constexpr int tc_raw_bytes(int mode, int type) { return (mode == 0 ? 2 : 1) * (type == T_Q4K ? 2 : 6) * 4096; }
constexpr int TC_SMEM_BUDGET = 225 * 1024 - 1024;          // dynamic shared memory per CTA, less alignment slack
constexpr int EPI_ROW = 36;                                 // floats per row of a warp's 32 x 32 transpose tile
constexpr int tc_epi_bytes(int mode) { return mode == 1 ? 4 * 32 * EPI_ROW * 4 : 0; }
constexpr int tc_raw_fit(int mode, int type, int a, int b) {
    return (TC_SMEM_BUDGET - tc_epi_bytes(mode) - a * TC_A_BYTES - b * tc_b_bytes(mode)) / tc_raw_bytes(mode, type) > 4
               ? 4
               : (TC_SMEM_BUDGET - tc_epi_bytes(mode) - a * TC_A_BYTES - b * tc_b_bytes(mode)) / tc_raw_bytes(mode, type);
}
// deepest A ring first, then three B stages if the raw ring still gets three, else two
constexpr TcCfg tc_cfg(int mode, int type) {
    for (int a = 4; a >= 2; --a) {
        if (tc_raw_fit(mode, type, a, 3) >= 3) return TcCfg{a, 3, tc_raw_fit(mode, type, a, 3)};
        if (tc_raw_fit(mode, type, a, 2) >= 1) return TcCfg{a, 2, tc_raw_fit(mode, type, a, 2)};
    }
    return TcCfg{0, 0, 0};
}
constexpr size_t tc_smem(int mode, int type) {
    return (size_t)tc_cfg(mode, type).a * TC_A_BYTES + (size_t)tc_cfg(mode, type).b * tc_b_bytes(mode) +
           (size_t)tc_cfg(mode, type).raw * tc_raw_bytes(mode, type) + tc_epi_bytes(mode) + 1024;   // + alignment slack
}
static_assert(tc_cfg(0, T_Q4K).a >= 2 && tc_cfg(0, T_Q6K).a >= 2 && tc_cfg(1, T_Q4K).a >= 2 &&
                  tc_cfg(1, T_Q6K).a >= 2, "shared-memory plan");

// 64 f16 of row r into a 128B-swizzled tile: 16-byte chunk c of the row lands at chunk c ^ (r % 8)
__device__ __forceinline__ void store_row_sw128(uint8_t* tile, int r, const uint4 v[8]) {
    uint8_t* row = tile + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = v[c];
}

}  // namespace

struct TcArgs {
    int grid;               // CTAs of the launch
    LayerWeights lw;
    int H, I, KK;
    const int* offsets;     // [NS+1] sorted-entry offset of each slot
    const int* perm;        // sorted position -> entry id t*KK + j
    const int2* items;      // (slot, M tile) per M tile
    const int* n_items;     // device count of M tiles (N blocks are expanded in the kernel)
    const __half* A;        // MODE 0: Q8_K-dequantised activations [T][H]; MODE 1: h [P][I] (sorted)
    const int* a_row;       // MODE 0, optional: A row of each entry id (else entry id / KK)
    __half* hq;             // MODE 0 output [P][I] (sorted order)
    __half* y;              // MODE 1 output [entries][H] by entry id, f16 (clamped to the f16 range)
    // MODE 1 over peer memory (y_peer != null): entry r is row i = r % y_cap of source s = r / y_cap's
    // region, and its output goes to rank s's yback row y_start[s] + i (block base y_peer[s] + y_off)
    uint8_t* const* y_peer;
    int64_t y_off;
    const int* y_start;
    int y_cap;
    unsigned* err;
    unsigned long long* trace;   // optional stamps [cta < TC_TRACE_CTAS][item < 2][stage < 32][TC_TRACE_SLOTS]
};

template <int MODE, int TYPE>
__global__ void __launch_bounds__(tc_threads(MODE), 1) k_tc_experts(TcArgs a) {
    constexpr int NMAT = MODE == 0 ? 2 : 1;
    constexpr TcCfg CFG = tc_cfg(MODE, TYPE);
    constexpr int AST = CFG.a, BST = CFG.b;
    constexpr int A_BYTES = TC_M * 128;                    // 16 KiB
    constexpr int B_BYTES = TC_N * 128;                    // 32 KiB per matrix
    constexpr int BSTAGE_BYTES = NMAT * B_BYTES;
    constexpr int RAW_MAT = Seg<TYPE>::RAW_CH * 4096;      // raw bytes of one matrix per stage
    constexpr int RAW_BYTES = NMAT * RAW_MAT;
    constexpr int RAWD = CFG.raw;                          // stages of raw bytes in flight
    extern __shared__ uint8_t smem_raw[];
    // accumulators: gate/up uses all 512 TMEM columns (one buffer); down double-buffers 2 x 256 columns
    constexpr int NACC = MODE == 0 ? 1 : 2;
    __shared__ uint64_t full_a[AST], empty_a[AST], full_b[BST], empty_b[BST], acc_full[NACC], acc_empty[NACC], done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    __shared__ float s_amax[2][TC_M];

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* ring_a = smem;                                // [AST][A_BYTES]
    uint8_t* ring_b = smem + AST * A_BYTES;                // [BST][NMAT][B_BYTES]
    uint8_t* ring = ring_b + BST * BSTAGE_BYTES;           // [RAWD][RAW_BYTES]
    float* epi_tile = reinterpret_cast<float*>(ring + RAWD * RAW_BYTES);   // down epilogue: [4 warps][32][EPI_ROW]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = MODE == 0 ? a.H : a.I;                   // reduction length
    const int NOUT = MODE == 0 ? a.I : a.H;                // output rows of the weight matrix
    const int KC = K / TC_KC;
    const int NBLK = NOUT / TC_N;
    const int nbK = K / QK;
    const int64_t nblk_total = (int64_t)NOUT * nbK;

    if (tid == 0) {
        for (int s = 0; s < AST; ++s) {
            bar_init(&full_a[s], A_THREADS);
            bar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < BST; ++s) {
            bar_init(&full_b[s], B_THREADS);
            bar_init(&empty_b[s], 1);
        }
        for (int i = 0; i < NACC; ++i) {
            bar_init(&acc_full[i], 1);
            bar_init(&acc_empty[i], MODE == 0 ? B_THREADS : EPI_THREADS);
        }
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
    unsigned long long* trc = a.trace && blockIdx.x < TC_TRACE_CTAS
                                  ? a.trace + (int64_t)blockIdx.x * TC_TRACE_ITEMS * TC_TRACE_STAGES * TC_TRACE_SLOTS
                                  : nullptr;
#define TC_STAMP(item_no_, kc_, slot_)                                                                     \
    do {                                                                                                   \
        if (trc && (item_no_) < TC_TRACE_ITEMS && (kc_) < TC_TRACE_STAGES)                                 \
            trc[((item_no_) * TC_TRACE_STAGES + (kc_)) * TC_TRACE_SLOTS + (slot_)] = gtime();              \
    } while (0)

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
                // this item's accumulator buffer must have been drained by the epilogue of its last user
                const int buf = item_no % NACC, use = item_no / NACC;
                const uint32_t dacc = tmem + (uint32_t)(buf * TC_N);
                bool ok = use == 0 || bar_wait(&acc_empty[buf], (use - 1) & 1, &s_abort);
                tc_fence_after();
                bool ready = false;                  // this stage's barriers were seen complete by the last probe
                for (int kc = 0; kc < KC && ok; ++kc) {
                    const uint32_t st_it = it0 + kc;
                    const int sa = st_it % AST, sb = st_it % BST;
                    if (!ready && (!bar_wait(&full_a[sa], (st_it / AST) & 1, &s_abort) ||
                                   !bar_wait(&full_b[sb], (st_it / BST) & 1, &s_abort))) { ok = false; break; }
                    TC_STAMP(item_no, kc, 0);
                    fence_async_smem();
                    tc_fence_after();
                    // probe the next stage now, so that the probes' latency overlaps this stage's MMAs
                    // rather than following them (measured: ~0.3 us of idle tensor pipe per stage otherwise)
                    const uint32_t nx = st_it + 1;
                    ready = kc + 1 < KC && bar_peek(&full_a[nx % AST], (nx / AST) & 1) &&
                            bar_peek(&full_b[nx % BST], (nx / BST) & 1);
                    const uint64_t ad = sw128_desc(ring_a + sa * A_BYTES);
                    const uint64_t bd0 = sw128_desc(ring_b + sb * BSTAGE_BYTES);
                    const uint64_t bd1 = sw128_desc(ring_b + sb * BSTAGE_BYTES + B_BYTES);
#pragma unroll
                    for (int ks = 0; ks < TC_KC / 16; ++ks) {   // +32 bytes of K = +2 in the descriptor
                        const uint32_t acc = (kc > 0 || ks > 0) ? 1u : 0u;
                        umma_f16(dacc, ad + 2 * ks, bd0 + 2 * ks, acc);
                        if (MODE == 0) umma_f16(tmem + TC_N, ad + 2 * ks, bd1 + 2 * ks, acc);
                    }
                    umma_commit(&empty_a[sa]);       // the stages are free once these MMAs have read them
                    umma_commit(&empty_b[sb]);
                    TC_STAMP(item_no, kc, 1);
                }
                if (ok) umma_commit(&acc_full[buf]); // accumulators complete
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
                    src[i] = MODE == 0 ? a.A + (int64_t)(a.a_row ? a.a_row[a.perm[sp]] : a.perm[sp] / a.KK) * a.H
                                         : a.A + (int64_t)sp * a.I;
                }
            }
            for (int kc = 0; kc < KC; ++kc) {
                const uint32_t st_it = it0 + kc;
                const int s = st_it % AST;
                const uint32_t round = st_it / AST;
                if (round > 0 && !bar_wait(&empty_a[s], (round - 1) & 1, &s_abort)) break;
                if (s_abort) break;
                if (t == 0) TC_STAMP(item_no, kc, 5);
                uint8_t* tile = ring_a + s * A_BYTES;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = rg + 16 * i;
                    const void* g = src[i] ? (const void*)(src[i] + kc * TC_KC + c * 8) : (const void*)a.A;
                    cp_async16(tile + r * 128 + ((c ^ (r & 7)) << 4), g, src[i] ? 16u : 0u);
                }
                cp_async_arrive_noinc(&full_a[s]);
                if (t == 0) TC_STAMP(item_no, kc, 6);
            }
        } else if (MODE == 1 && warp >= EPI_TID0 / 32) {
            // ---------------- down epilogue (128 threads): TMEM -> y rows, one accumulator row each -----
            const int buf = item_no % NACC, use = item_no / NACC;
            const bool ok = __all_sync(0xFFFFFFFFu, bar_wait(&acc_full[buf], use & 1, &s_abort));
            if (tid == EPI_TID0) TC_STAMP(item_no, 0, 7);
            const int q = warp & 3;
            const int m = 32 * q + lane;                          // accumulator row = tile row
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * TC_N);
            const bool valid = m < nrows;
            if (ok) {
                tc_fence_after();
                // each 32 x 32 chunk (lane = row) goes through a padded shared tile so that a store
                // instruction writes four whole 128-byte row segments instead of 32 scattered 16 bytes
                const int entry = valid ? a.perm[row0 + m] : -1;
                __half* yrow = nullptr;                             // this lane's output row
                if (entry >= 0) {
                    if (a.y_peer) {
                        const int src = entry / a.y_cap, i = entry - src * a.y_cap;
                        const int at = a.y_start[src] + i;
                        if (at >= 0 && at < a.y_cap)
                            yrow = reinterpret_cast<__half*>(a.y_peer[src] + a.y_off) + (int64_t)at * a.H;
                        else
                            atomicOr(a.err, 1u);
                    } else {
                        yrow = a.y + (int64_t)entry * a.H;
                    }
                }
                float* tile = epi_tile + (warp & 3) * 32 * EPI_ROW;
                const int rsub = lane >> 3, c4 = lane & 7;          // read phase: row 4i + rsub, float4 c4
                float v[32];
#pragma unroll 1
                for (int cc = 0; cc < TC_N / 32; ++cc) {
                    tmem_ld32(lane_base + 32 * cc, v);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<float4*>(tile + lane * EPI_ROW + 4 * i) =
                            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rr = 4 * i + rsub;
                        __half* dst = reinterpret_cast<__half*>(
                            __shfl_sync(0xFFFFFFFFu, reinterpret_cast<unsigned long long>(yrow), rr));
                        const float4 val = *reinterpret_cast<const float4*>(tile + rr * EPI_ROW + 4 * c4);
                        const float lim = 65504.f;
                        const uint2 hv = make_uint2(
                            bits_h2(__floats2half2_rn(fminf(fmaxf(val.x, -lim), lim), fminf(fmaxf(val.y, -lim), lim))),
                            bits_h2(__floats2half2_rn(fminf(fmaxf(val.z, -lim), lim), fminf(fmaxf(val.w, -lim), lim))));
                        if (dst) *reinterpret_cast<uint2*>(dst + (int64_t)nb_out * TC_N + 32 * cc + 4 * c4) = hv;
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            bar_arrive(&acc_empty[buf]);
            if (tid == EPI_TID0) TC_STAMP(item_no, 1, 7);
        } else {
            // ---------------- B dequant (256 threads), then the gate/up epilogue ----------------
            const int r = tid - B_TID0;                          // B row within the N block
            // this row's weight matrices (m0 gate or down, m1 up) and first block for item `itm`
            auto row_of = [&](int itm, const uint8_t*& m0_, const uint8_t*& m1_, int64_t& rb_) {
                const int2 itx = a.items[itm / NBLK];
                const int sl = itx.x;
                const int64_t nrow = (int64_t)(itm - (itm / NBLK) * NBLK) * TC_N + r;
                const bool shx = sl >= a.lw.n_slots;
                const uint8_t* bs = shx ? a.lw.shared : a.lw.pool + (int64_t)sl * a.lw.slot_stride;
                m0_ = MODE == 0 ? bs : bs + (shx ? a.lw.sh_off_down : a.lw.off_down);
                m1_ = bs + (shx ? a.lw.sh_off_up : a.lw.off_up);
                rb_ = nrow * nbK;
            };
            const uint8_t *m0, *m1;
            int64_t row_blk;
            row_of(item, m0, m1, row_blk);
            const int next = item + gridDim.x;                   // this CTA's next item, if any
            const uint8_t *m0n = m0, *m1n = m1;
            int64_t row_blk_n = row_blk;
            if (next < n_items) row_of(next, m0n, m1n, row_blk_n);
            // raw bytes of stage kc (one commit group, ring slot by the CTA's stage counter); stages past
            // this item's last are the next item's first ones, so a new item starts on bytes in flight
            auto issue = [&](int kc) {
                uint8_t* slot_p = ring + ((it0 + kc) % RAWD) * RAW_BYTES;
                if (kc < KC) {
                    Seg<TYPE>::issue(slot_p, r, m0, nblk_total, row_blk + (kc >> 2), kc & 3);
                    if (MODE == 0) Seg<TYPE>::issue(slot_p + RAW_MAT, r, m1, nblk_total, row_blk + (kc >> 2), kc & 3);
                } else if (next < n_items) {
                    const int kn = kc - KC;
                    Seg<TYPE>::issue(slot_p, r, m0n, nblk_total, row_blk_n + (kn >> 2), kn & 3);
                    if (MODE == 0) Seg<TYPE>::issue(slot_p + RAW_MAT, r, m1n, nblk_total, row_blk_n + (kn >> 2), kn & 3);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
            };
            if (item_no == 0) {                                  // later items' first stages were issued by the previous one
#pragma unroll
                for (int j = 0; j < RAWD; ++j) issue(j);
            }
            typename Seg<TYPE>::Hdr h0c = Seg<TYPE>::load_hdr(m0, nblk_total, row_blk), h0n = h0c;
            typename Seg<TYPE>::Hdr h1c = h0c, h1n = h0c;
            if (MODE == 0) h1c = h1n = Seg<TYPE>::load_hdr(m1, nblk_total, row_blk);
            if (nbK > 1) {
                h0n = Seg<TYPE>::load_hdr(m0, nblk_total, row_blk + 1);
                if (MODE == 0) h1n = Seg<TYPE>::load_hdr(m1, nblk_total, row_blk + 1);
            }
            for (int kc = 0; kc < KC; ++kc) {
                const uint32_t st_it = it0 + kc;
                const int s = st_it % BST;
                const uint32_t round = st_it / BST;
                if (kc > 0 && (kc & 3) == 0) {                   // next block: rotate the scale words
                    h0c = h0n;
                    h1c = h1n;
                    const int nb_next = (kc >> 2) + 1;
                    if (nb_next < nbK) {
                        h0n = Seg<TYPE>::load_hdr(m0, nblk_total, row_blk + nb_next);
                        if (MODE == 0) h1n = Seg<TYPE>::load_hdr(m1, nblk_total, row_blk + nb_next);
                    }
                }
                asm volatile("cp.async.wait_group %0;" ::"n"(RAWD - 1) : "memory");
                if (r == 0) TC_STAMP(item_no, kc, 2);
                const uint8_t* slot_p = ring + ((it0 + kc) % RAWD) * RAW_BYTES;
                Seg<TYPE> sg;
                sg.read(slot_p, r);
                uint4 v[8];
                sg.dequant(kc & 3, h0c, v);
                if (round > 0 && !bar_wait(&empty_b[s], (round - 1) & 1, &s_abort)) break;
                if (s_abort) break;
                if (r == 0) TC_STAMP(item_no, kc, 3);
                uint8_t* tile = ring_b + s * BSTAGE_BYTES;
                store_row_sw128(tile, r, v);
                if (MODE == 0) {
                    sg.read(slot_p + RAW_MAT, r);
                    sg.dequant(kc & 3, h1c, v);
                    store_row_sw128(tile + B_BYTES, r, v);
                }
                fence_async_smem();
                bar_arrive(&full_b[s]);
                if (r == 0) TC_STAMP(item_no, kc, 4);
                issue(kc + RAWD);                                // refill this ring slot (its bytes are consumed)
            }
            if (MODE == 1) continue;
            // ---- gate/up epilogue: warp % 4 selects the TMEM lane quarter, (warp - 5) / 4 the column half ----
            const bool ok = __all_sync(0xFFFFFFFFu, bar_wait(&acc_full[0], item_no & 1, &s_abort));
            if (r == 0) TC_STAMP(item_no, 0, 7);
            const int q = warp & 3, half = (warp - 5) >> 2;
            const int m = 32 * q + lane;                          // accumulator row = tile row
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
            const bool valid = m < nrows;
            if (ok) tc_fence_after();
            {
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
            }
            tc_fence_before();
            bar_arrive(&acc_empty[0]);
            if (r == 0) TC_STAMP(item_no, 1, 7);
        }
    }
#undef TC_STAMP
    // ---- teardown: drain this CTA's tensor-core ops and copies, then free the tensor memory ----
    if (warp == 0 && lane == 0) {
        umma_commit(&done_bar);
        bar_drain(&done_bar, 0);
    }
    if (warp >= 1) asm volatile("cp.async.wait_all;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    if (s_abort && tid == 0) atomicOr(a.err, 2u);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// ggml's Q8_K of rows [R][K] (256-value blocks, iscale = 127 / max|x|, round to nearest even, clamp
// 127), written back as f16(q * d): the activation operand of the tensor-core GEMMs. One warp per
// 256-value block (8 values per lane), eight blocks per CTA.
__global__ void __launch_bounds__(256) k_q8_to_f16(const float* __restrict__ x, int64_t nblocks, __half* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const float4* src = reinterpret_cast<const float4*>(x + b * QK) + 2 * lane;
    const float4 v0 = src[0], v1 = src[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
    am = warp_max(am);
    const float iscale = am != 0.f ? 127.f / am : 0.f;
    const float d = am != 0.f ? 1.f / iscale : 0.f;
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q0 = min(127, __float2int_rn(iscale * v[2 * i])), q1 = min(127, __float2int_rn(iscale * v[2 * i + 1]));
        pk[i] = bits_h2(__floats2half2_rn((float)q0 * d, (float)q1 * d));
    }
    reinterpret_cast<uint4*>(out + b * QK)[lane] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// ---------------------------------------------------------------------------------------------
// Router logits of large batches on the tensor cores (tcgen05 kind::tf32), f32-accurate by a
// three-term split: x = x_hi + x_lo and w = w_hi + w_lo with x_hi = x truncated to tf32 and x_lo =
// x - x_hi (exact in f32, read by the tensor core truncated to tf32); x . w is taken as
// x_hi.w_hi + x_hi.w_lo + x_lo.w_hi with f32 accumulation in tensor memory (the dropped x_lo.w_lo
// and the truncation of the low parts are ~2^-21 of |x||w| per product). CTA (128-token tile,
// N-expert tile, K split z): warp 0's lane 0 issues the MMAs (M = 128, N, K = 8; three per K step);
// warps 1-8 load the stage's 32-value K segments of the 128 token rows of fx and the N expert rows of
// the router as 16-byte pieces (eight lanes per row, so a warp's loads cover whole 128-byte lines: a
// row per thread saturated the L1 tag stage, 87 % of L1TEX throughput for 13 % tensor-pipe activity),
// split them and store the hi and lo parts 128B-swizzled; warps 1-4 then read the accumulator rows and
// write the split's partial logits (double) in the layout k_route_topk sums: part[z][t][e].
// ---------------------------------------------------------------------------------------------
namespace {

constexpr int RT_M = 128;                  // tokens per tile (UMMA M)
constexpr int RT_NMAX = 128;               // experts per tile (UMMA N: a multiple of 16)
constexpr int RT_STAGES = 3;
constexpr int RT_THREADS = 288;
constexpr int RT_A_BYTES = RT_M * 128;     // one 128-row x 32-value f32 tile (hi or lo)
constexpr int RT_B_BYTES = RT_NMAX * 128;
constexpr int RT_STAGE = 2 * RT_A_BYTES + 2 * RT_B_BYTES;
constexpr size_t RT_SMEM = (size_t)RT_STAGES * RT_STAGE + 1024;

// the tf32 value the tensor core reads from an f32 word: the low 13 mantissa bits dropped
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

}  // namespace

struct RouterTcArgs {
    const float* fx;       // [T][H]
    const float* w;        // [E][H]
    int T, H, E, N, klen;  // N experts per tile (multiple of 16, <= RT_NMAX); klen K per split (multiple of 32)
    double* part;          // [splits][T][E]
    unsigned* err;
};

__global__ void __launch_bounds__(RT_THREADS, 1) k_router_tc(const RouterTcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[RT_STAGES], empty[RT_STAGES], done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * RT_M, e0 = blockIdx.y * a.N, k0 = blockIdx.z * a.klen;
    const int KS = a.klen / 32;
    if (tid == 0) {
        for (int s = 0; s < RT_STAGES; ++s) {
            bar_init(&full[s], RT_THREADS - 32);
            bar_init(&empty[s], 1);
        }
        bar_init(&done_bar, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&s_tmem)),
                     "r"(RT_NMAX) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // D f32 (bits 4-5 = 1), A and B tf32 (bits 7-9, 10-12 = 2), both K-major, N >> 3, M >> 4
    const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(a.N >> 3) << 17) | ((uint32_t)(RT_M >> 4) << 24);
    if (warp == 0) {
        if (lane == 0) {
            for (int kc = 0; kc < KS; ++kc) {
                const int s = kc % RT_STAGES;
                if (!bar_wait(&full[s], (kc / RT_STAGES) & 1, &s_abort)) break;
                fence_async_smem();
                tc_fence_after();
                const uint8_t* st = smem + s * RT_STAGE;
                const uint64_t ahi = sw128_desc(st), alo = sw128_desc(st + RT_A_BYTES);
                const uint64_t bhi = sw128_desc(st + 2 * RT_A_BYTES), blo = sw128_desc(st + 2 * RT_A_BYTES + RT_B_BYTES);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {           // K = 8 per MMA: +32 bytes = +2 in the descriptor
                    umma_tf32(tmem, ahi + 2 * ks, bhi + 2 * ks, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                    umma_tf32(tmem, ahi + 2 * ks, blo + 2 * ks, idesc, 1u);
                    umma_tf32(tmem, alo + 2 * ks, bhi + 2 * ks, idesc, 1u);
                }
                umma_commit(&empty[s]);                  // the stage is free once these MMAs have read it
            }
            umma_commit(&done_bar);                      // the accumulators are complete
        }
        __syncwarp();
    } else {
        // 16-byte pieces: piece idx = p + 256 j (j < 8) is chunk idx % 8 of row idx / 8 (rows 0-127 the
        // token rows of fx, 128-255 the expert rows of the router), so that a warp's loads cover four
        // whole 128-byte row segments
        const int p = tid - 32;
        const float* src[8];
        bool valid[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int idx = p + 256 * j, row = idx >> 3, c = idx & 7;
            const bool is_a = row < RT_M;
            const int rr = is_a ? row : row - RT_M;
            valid[j] = is_a ? t0 + rr < a.T : (rr < a.N && e0 + rr < a.E);
            src[j] = (is_a ? a.fx + (int64_t)(t0 + rr) * a.H : a.w + (int64_t)(e0 + rr) * a.H) + k0 + 4 * c;
        }
        float4 nxt[8];
        auto load = [&](int kc) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                nxt[j] = valid[j] ? __ldg(reinterpret_cast<const float4*>(src[j] + 32 * kc)) : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        load(0);
        for (int kc = 0; kc < KS; ++kc) {
            const int s = kc % RT_STAGES;
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = nxt[j];
            if (kc + 1 < KS) load(kc + 1);               // the next segment in flight during this one
            if (kc >= RT_STAGES && !bar_wait(&empty[s], ((kc / RT_STAGES) - 1) & 1, &s_abort)) break;
            if (s_abort) break;
            uint8_t* st = smem + s * RT_STAGE;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int idx = p + 256 * j, row = idx >> 3, c = idx & 7;
                const bool is_a = row < RT_M;
                const int rr = is_a ? row : row - RT_M;
                if (!is_a && rr >= a.N) continue;            // expert rows past the tile are not read
                // hi = x with the mantissa bits below tf32 cleared; lo = x - hi (exact in f32), of which
                // the tensor core reads the leading 11 bits
                const float h0 = tf32_trunc(v[j].x), h1 = tf32_trunc(v[j].y), h2 = tf32_trunc(v[j].z),
                            h3 = tf32_trunc(v[j].w);
                const uint4 hi = make_uint4(__float_as_uint(h0), __float_as_uint(h1), __float_as_uint(h2), __float_as_uint(h3));
                const uint4 lo = make_uint4(__float_as_uint(v[j].x - h0), __float_as_uint(v[j].y - h1),
                                            __float_as_uint(v[j].z - h2), __float_as_uint(v[j].w - h3));
                uint8_t* th = st + (is_a ? 0 : 2 * RT_A_BYTES);
                const int part_bytes = is_a ? RT_A_BYTES : RT_B_BYTES;
                const int off = rr * 128 + ((c ^ (rr & 7)) << 4);    // 128B swizzle
                *reinterpret_cast<uint4*>(th + off) = hi;
                *reinterpret_cast<uint4*>(th + part_bytes + off) = lo;
            }
            fence_async_smem();
            bar_arrive(&full[s]);
        }
    }
    // epilogue: warps 1-4 read the accumulator rows (warp w reaches TMEM lanes 32 * (w % 4) ..)
    if (warp >= 1 && warp <= 4) {
        const bool ok = __all_sync(0xFFFFFFFFu, bar_wait(&done_bar, 0, &s_abort));
        if (ok) {
            tc_fence_after();
            const int q = warp & 3, m = 32 * q + lane, t = t0 + m;
            const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
            double* dst = a.part + ((int64_t)blockIdx.z * a.T + t) * a.E + e0;
            float v[32];
            for (int cc = 0; cc * 32 < a.N; ++cc) {
                tmem_ld32(lane_base + 32 * cc, v);
                if (t < a.T) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int col = 32 * cc + i;
                        if (col < a.N && e0 + col < a.E) dst[col] = (double)v[i];
                    }
                }
            }
        }
    }
    // teardown: the MMAs have completed (or the CTA gave up and drains them), then free the tensor memory
    if (warp == 0 && lane == 0) bar_drain(&done_bar, 0);
    tc_fence_before();
    __syncthreads();
    if (s_abort && tid == 0) atomicOr(a.err, 2u);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(RT_NMAX) : "memory");
    }
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

template <int MODE, int TYPE>
cudaError_t launch_tc(const TcArgs& a, cudaStream_t s) {
    static unsigned long long attr_set = 0;   // devices on which the shared-memory limit was raised
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(attr_set >> dev & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_tc_experts<MODE, TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc_smem(MODE, TYPE));
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set |= 1ull << dev;
    }
    k_tc_experts<MODE, TYPE><<<a.grid, tc_threads(MODE), tc_smem(MODE, TYPE), s>>>(a);
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

cudaError_t launch_router_tc(const float* fx, const float* w_router, int T, int H, int E, int ksplit, double* part,
                             unsigned* err, cudaStream_t s) {
    if (T <= 0 || E <= 0 || H % (32 * ksplit) != 0) return cudaErrorInvalidValue;
    static unsigned long long attr_set = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(attr_set >> dev & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_router_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RT_SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set |= 1ull << dev;
    }
    RouterTcArgs a{fx, w_router, T, H, E, 0, H / ksplit, part, err};
    a.N = E >= RT_NMAX ? RT_NMAX : ((E + 15) / 16) * 16;
    const dim3 grid((T + RT_M - 1) / RT_M, (E + a.N - 1) / a.N, ksplit);
    k_router_tc<<<grid, RT_THREADS, RT_SMEM, s>>>(a);
    return cudaGetLastError();
}

// Expert FFN of R rows that arrive already quantised (Q8_K q*d as f16, [R][H]), each bound to one
// pool slot: the expert-parallel receive side. y_out[r] (f16 [R][H]) is row r's expert output.
cudaError_t launch_experts_tc_rows(const Dims& d, const LayerWeights& lw, const Scratch& sc, const uint16_t* rows,
                                   const int32_t* slot_of_row, int R, uint16_t* y_out, cudaStream_t s, int* launches) {
    int nl = 0;
    cudaError_t e;
    if ((e = launch_dispatch(slot_of_row, R, 1, 1, lw.n_slots, sc, TC_M, s, &nl)) != cudaSuccess) return e;
    TcArgs a{};
    a.grid = d.gemm_ctas > 0 && d.gemm_ctas < tc_grid() ? d.gemm_ctas : tc_grid();
    a.lw = lw;
    a.lw.shared = nullptr;           // rows name their slot; a shared expert is not dispatched
    a.H = d.H;
    a.I = d.I;
    a.KK = 1;
    a.offsets = sc.offsets;
    a.perm = sc.perm;
    a.items = sc.items;
    a.n_items = sc.n_items;
    a.err = sc.sync;
    a.A = reinterpret_cast<const __half*>(rows);
    a.hq = reinterpret_cast<__half*>(sc.hq16);
    e = lw.gate_type == T_Q4K ? launch_tc<0, T_Q4K>(a, s) : launch_tc<0, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    a.A = reinterpret_cast<const __half*>(sc.hq16);
    a.y = reinterpret_cast<__half*>(y_out);
    e = lw.down_type == T_Q4K ? launch_tc<1, T_Q4K>(a, s) : launch_tc<1, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    if (launches) *launches += nl + 2;
    return cudaSuccess;
}

// Expert-parallel receive side over peer memory: the G regions of this rank's block hold the entries
// that every source sent (count[s] of them in region s), each tagged with its expert id and the row of
// its token in region s of `rows`.
__global__ void __launch_bounds__(256) k_p2p_rx_slots(const uint8_t* __restrict__ block, P2PLayout L, int G, int cap,
                                                      int cap_rows, int e_lo, int epr, int slot_base, int n_slots,
                                                      unsigned* err, int* __restrict__ slots, int* __restrict__ arow) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= (int64_t)G * cap) return;
    const int src = (int)(r / cap), i = (int)(r - (int64_t)src * cap);
    const int* count = reinterpret_cast<const int*>(block + L.count);
    const int32_t* expert = reinterpret_cast<const int32_t*>(block + L.expert);
    const int32_t* row_of = reinterpret_cast<const int32_t*>(block + L.row_of);
    int sl = -1, ar = 0;
    if (!(*(volatile unsigned*)err & 2u) && i < count[src]) {
        const int ex = expert[r], ro = row_of[r];
        if (ex >= e_lo && ex < e_lo + epr && ex - e_lo + slot_base < n_slots && ro >= 0 && ro < cap_rows) {
            sl = ex - e_lo + slot_base;
            ar = src * cap_rows + ro;
        } else {
            atomicOr(err, 1u);
        }
    }
    slots[r] = sl;
    arow[r] = ar;
}

cudaError_t launch_p2p_experts(const Dims& d, const LayerWeights& lw, const Scratch& sc, const P2PSend& p,
                               const uint8_t* block, int slot_base, int* slots, int* arow, cudaStream_t s,
                               int* launches) {
    const int64_t n = (int64_t)p.G * p.cap;
    k_p2p_rx_slots<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(block, p.L, p.G, p.cap, p.cap_rows, p.rank * p.epr,
                                                                p.epr, slot_base, lw.n_slots, sc.sync, slots, arow);
    int nl = 1;
    cudaError_t e;
    if ((e = launch_dispatch(slots, (int)n, 1, 1, lw.n_slots, sc, TC_M, s, &nl, true)) != cudaSuccess) return e;
    TcArgs a{};
    a.grid = d.gemm_ctas > 0 && d.gemm_ctas < tc_grid() ? d.gemm_ctas : tc_grid();
    a.lw = lw;
    a.lw.shared = nullptr;
    a.H = d.H;
    a.I = d.I;
    a.KK = 1;
    a.offsets = sc.offsets;
    a.perm = sc.perm;
    a.items = sc.items;
    a.n_items = sc.n_items;
    a.err = sc.sync;
    a.A = reinterpret_cast<const __half*>(block + p.L.rows);
    a.a_row = arow;
    a.hq = reinterpret_cast<__half*>(sc.hq16);
    e = lw.gate_type == T_Q4K ? launch_tc<0, T_Q4K>(a, s) : launch_tc<0, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    a.A = reinterpret_cast<const __half*>(sc.hq16);
    a.a_row = nullptr;
    a.y_peer = p.peer;
    a.y_off = p.L.yback;
    a.y_start = reinterpret_cast<const int*>(block + p.L.start);
    a.y_cap = p.cap;
    e = lw.down_type == T_Q4K ? launch_tc<1, T_Q4K>(a, s) : launch_tc<1, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    if (launches) *launches += nl + 2;
    return cudaSuccess;
}

// Q8_K-dequantised f16 rows of fx ([T][H]); used by the expert-parallel send side.
cudaError_t launch_q8_rows(const float* fx, int T, int H, uint16_t* out, cudaStream_t s) {
    const int64_t nq = (int64_t)T * (H / QK);
    k_q8_to_f16<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(fx, nq, reinterpret_cast<__half*>(out));
    return cudaGetLastError();
}

int64_t tc_trace_elems() { return (int64_t)2 * TC_TRACE_CTAS * TC_TRACE_ITEMS * TC_TRACE_STAGES * TC_TRACE_SLOTS; }

cudaError_t launch_experts_tc(const Dims& d, const LayerWeights& lw, const Scratch& sc, const float* fx,
                              const int32_t* slot_of_sel, const float* w, void* x_inout, int T, cudaStream_t s,
                              int* launches, unsigned long long* trace) {
    const bool shared = lw.shared != nullptr;
    const int KK = d.k + (shared ? 1 : 0);
    int nl = 0;
    cudaError_t e;
    // 1. ggml's Q8_K of fx, as f16 (q * d) rows
    const int64_t nq = (int64_t)T * (d.H / QK);
    k_q8_to_f16<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(fx, nq, reinterpret_cast<__half*>(sc.xq16));
    ++nl;
    if (shared) {
        if ((e = launch_shared_gate(fx, lw.sh_gate_inp, d.H, T, sc.sh_gate, s)) != cudaSuccess) return e;
        ++nl;
    }
    // 2. counting sort of the entries by slot, and the (slot, M tile) work list
    if ((e = launch_dispatch(slot_of_sel, T, d.k, KK, lw.n_slots, sc, TC_M, s, &nl)) != cudaSuccess) return e;
    // 3. gate/up + SwiGLU + Q8_K(h); 4. down
    TcArgs a{};
    a.grid = d.gemm_ctas > 0 && d.gemm_ctas < tc_grid() ? d.gemm_ctas : tc_grid();
    a.lw = lw;
    a.H = d.H;
    a.I = d.I;
    a.KK = KK;
    a.offsets = sc.offsets;
    a.perm = sc.perm;
    a.items = sc.items;
    a.n_items = sc.n_items;
    a.err = sc.sync;
    a.trace = trace;
    a.A = reinterpret_cast<const __half*>(sc.xq16);
    a.hq = reinterpret_cast<__half*>(sc.hq16);
    e = lw.gate_type == T_Q4K ? launch_tc<0, T_Q4K>(a, s) : launch_tc<0, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    ++nl;
    a.A = reinterpret_cast<const __half*>(sc.hq16);
    a.y = reinterpret_cast<__half*>(sc.y);      // f16 rows in the f32 scratch
    if (trace) a.trace = trace + tc_trace_elems() / 2;
    e = lw.down_type == T_Q4K ? launch_tc<1, T_Q4K>(a, s) : launch_tc<1, T_Q6K>(a, s);
    if (e != cudaSuccess) return e;
    ++nl;
    // 5. weighted combine into the residual, j ascending (shared with the grouped path)
    if ((e = launch_combine(d, sc, w, x_inout, T, KK, s, true)) != cudaSuccess) return e;
    ++nl;
    if (launches) *launches += nl;
    return cudaSuccess;
}

}  // namespace hoard
