// common.cuh -- device-side formats and arithmetic shared by every hoard_b200 kernel.
//
// Expert weights live in the HBM pool in a *plane* layout, re-laid from the GGUF block bytes at
// upload time so that every warp-wide 16-byte load is aligned and coalesced:
//
//   Q4_K matrix [N rows][nb blocks of 256 weights]:
//     qs  plane: N*nb*128 bytes at offset 0             (block (n,b) at (n*nb+b)*128, GGUF order)
//     hdr plane: N*nb*16  bytes at offset N*nb*128      (fp16 d, fp16 dmin, 12 B packed scales/mins)
//   Q6_K matrix:
//     ql  plane: N*nb*128 at 0; qh plane: N*nb*64 at N*nb*128; sc plane: N*nb*16 (int8) at
//     N*nb*192; d plane: N*nb fp16 at N*nb*208.
// Total bytes equal the GGUF bytes (144 / 210 per block); nothing is dequantised in memory.
//
// Activations follow ggml's CPU quantized mul_mat: each 256-value segment of an f32 activation
// row is quantized to Q8_K (d = 1/(127/amax), q = rne(x*127/amax), plus 16-value sums), and the
// weight . activation dot is an exact integer dot per sub-block, scaled by the fp16 factors.
// The sign convention (amax instead of ggml's signed max) negates q and d together, which leaves
// every product d*q, and so every dot, bit-identical.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace hoard {

// ---- programmatic dependent launch (the decode harness's chains of small kernels) ----------------
// A kernel launched by launch_pdl may be scheduled while the previous kernel of its stream still runs:
// it first lets its own successor be scheduled (launch_dependents), then waits until its predecessor has
// completed and its memory is visible (wait), before it reads or writes anything. With a predecessor
// that was not launched this way, or with a plain launch, both instructions return at once.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
    pdl_launch_dependents();
    pdl_wait();
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr int QK = 256;
enum : int { T_F32 = 0, T_F16 = 1, T_Q4K = 12, T_Q6K = 14, T_BF16 = 30 };

__host__ __device__ inline int block_bytes(int type) { return type == T_Q4K ? 144 : (type == T_Q6K ? 210 : 0); }
__host__ __device__ inline int64_t mat_bytes(int type, int64_t n, int64_t k) { return n * (k / QK) * block_bytes(type); }

// Units: the piece of a row one lane handles in one step.
//   Q4_K unit = 16 qs bytes = 32 weights (8 units per block);
//   Q6_K unit = 32 ql + 16 qh bytes = 64 weights (4 units per block).
__host__ __device__ inline int units_per_block(int type) { return type == T_Q4K ? 8 : 4; }

// ---- loads ----------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ int4 ld16s(const void* p) { return *reinterpret_cast<const int4*>(p); }
// weights are streamed once per call: keep them out of L1
__device__ __forceinline__ uint4 ld16_stream(const void* p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// ---- Q8_K activation row view -----------------------------------------------------------------
struct ActRow {
    const int8_t* q;   // [K]
    const float* d;    // [K/256]
    const int* bs;     // [K/16] sums of 16 consecutive q
};

// ---- Q4_K ---------------------------------------------------------------------------------------
struct Q4KPlanes {
    const uint8_t* qs;
    const uint8_t* hdr;
    __device__ __forceinline__ Q4KPlanes(const uint8_t* base, int64_t nblk_total)
        : qs(base), hdr(base + nblk_total * 128) {}
};

// 6-bit (scale, min) of sub-block j from the header words (w1,w2,w3 = scale bytes 0..11).
__device__ __forceinline__ void q4k_scale_min(const uint4& h, int j, int& sc, int& m) {
    const int jj = j & 3;
    const uint32_t b0 = (h.y >> (8 * jj)) & 0xFF;   // scales[jj]
    const uint32_t b4 = (h.z >> (8 * jj)) & 0xFF;   // scales[jj+4]
    if (j < 4) {
        sc = b0 & 63;
        m = b4 & 63;
    } else {
        const uint32_t b8 = (h.w >> (8 * jj)) & 0xFF;  // scales[jj+8]
        sc = (b8 & 0xF) | ((b0 >> 6) << 4);
        m = (b8 >> 4) | ((b4 >> 6) << 4);
    }
}

// Integer part of one Q4_K unit: unit c8 (0..7) of a block = qs bytes [16*c8, 16*c8+16):
// low nibbles are elements 64g+16hh+[0,16) (sub-block 2g), high nibbles 64g+32+16hh+[0,16)
// (sub-block 2g+1), with g = c8/2, hh = c8%2.  a_blk points at the activation's 256-segment.
__device__ __forceinline__ float q4k_unit_dot(const uint4& w, const uint4& h, int c8, const int8_t* a_blk,
                                              const int* bs_blk, float d8) {
    const int g = c8 >> 1, hh = c8 & 1;
    const int4 alo = ld16s(a_blk + 64 * g + 16 * hh);
    const int4 ahi = ld16s(a_blk + 64 * g + 32 + 16 * hh);
    int slo = __dp4a((int)(w.x & 0x0F0F0F0Fu), alo.x, 0);
    slo = __dp4a((int)(w.y & 0x0F0F0F0Fu), alo.y, slo);
    slo = __dp4a((int)(w.z & 0x0F0F0F0Fu), alo.z, slo);
    slo = __dp4a((int)(w.w & 0x0F0F0F0Fu), alo.w, slo);
    int shi = __dp4a((int)((w.x >> 4) & 0x0F0F0F0Fu), ahi.x, 0);
    shi = __dp4a((int)((w.y >> 4) & 0x0F0F0F0Fu), ahi.y, shi);
    shi = __dp4a((int)((w.z >> 4) & 0x0F0F0F0Fu), ahi.z, shi);
    shi = __dp4a((int)((w.w >> 4) & 0x0F0F0F0Fu), ahi.w, shi);
    int sc0, m0, sc1, m1;
    q4k_scale_min(h, 2 * g, sc0, m0);
    q4k_scale_min(h, 2 * g + 1, sc1, m1);
    const int bs0 = bs_blk[4 * g + hh], bs1 = bs_blk[4 * g + 2 + hh];
    const float d = h2f(h.x), dmin = h2f(h.x >> 16);
    return d8 * (d * (float)(sc0 * slo + sc1 * shi) - dmin * (float)(m0 * bs0 + m1 * bs1));
}

// ---- Q6_K ---------------------------------------------------------------------------------------
struct Q6KPlanes {
    const uint8_t* ql;
    const uint8_t* qh;
    const uint8_t* sc;
    const uint8_t* d;
    __device__ __forceinline__ Q6KPlanes(const uint8_t* base, int64_t nblk_total)
        : ql(base), qh(base + nblk_total * 128), sc(base + nblk_total * 192), d(base + nblk_total * 208) {}
};

__device__ __forceinline__ int sbyte(const uint4& v, int i) {  // signed byte i (0..15) of a 16-byte vector
    const uint32_t w = (i < 4) ? v.x : (i < 8) ? v.y : (i < 12) ? v.z : v.w;
    return (int)(int8_t)((w >> (8 * (i & 3))) & 0xFF);
}

// Integer part of one Q6_K unit v (0..3) of a block: h2 = v/2 picks the 128-weight half, r = v%2
// the 16-byte run. A = ql[64h2+16r..], B = ql[64h2+32+16r..], C = qh[32h2+16r..] give the four
// 16-weight groups 128h2 + 32a + 16r + [0,16), a = 0..3, with int8 scales sc[8h2 + r + 2a].
// sum (q-32)*x = sum q*x - 32*sum x, and sum x over a 16-group is the Q8_K partial sum.
__device__ __forceinline__ int q6k_unit_isum(const uint4& A, const uint4& B, const uint4& C, const uint4& S,
                                             int v, const int8_t* a_blk, const int* bs_blk) {
    const int h2 = v >> 1, r = v & 1;
    const int8_t* a0 = a_blk + 128 * h2 + 16 * r;
    const int4 x0 = ld16s(a0), x1 = ld16s(a0 + 32), x2 = ld16s(a0 + 64), x3 = ld16s(a0 + 96);
    const uint32_t Aw[4] = {A.x, A.y, A.z, A.w};
    const uint32_t Bw[4] = {B.x, B.y, B.z, B.w};
    const uint32_t Cw[4] = {C.x, C.y, C.z, C.w};
    const int xa0[4] = {x0.x, x0.y, x0.z, x0.w}, xa1[4] = {x1.x, x1.y, x1.z, x1.w};
    const int xa2[4] = {x2.x, x2.y, x2.z, x2.w}, xa3[4] = {x3.x, x3.y, x3.z, x3.w};
    int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t q0 = (Aw[i] & 0x0F0F0F0Fu) | ((Cw[i] << 4) & 0x30303030u);
        const uint32_t q1 = (Bw[i] & 0x0F0F0F0Fu) | ((Cw[i] << 2) & 0x30303030u);
        const uint32_t q2 = ((Aw[i] >> 4) & 0x0F0F0F0Fu) | (Cw[i] & 0x30303030u);
        const uint32_t q3 = ((Bw[i] >> 4) & 0x0F0F0F0Fu) | ((Cw[i] >> 2) & 0x30303030u);
        s0 = __dp4a((int)q0, xa0[i], s0);
        s1 = __dp4a((int)q1, xa1[i], s1);
        s2 = __dp4a((int)q2, xa2[i], s2);
        s3 = __dp4a((int)q3, xa3[i], s3);
    }
    const int g0 = 8 * h2 + r;
    s0 -= 32 * bs_blk[g0];
    s1 -= 32 * bs_blk[g0 + 2];
    s2 -= 32 * bs_blk[g0 + 4];
    s3 -= 32 * bs_blk[g0 + 6];
    return sbyte(S, g0) * s0 + sbyte(S, g0 + 2) * s1 + sbyte(S, g0 + 4) * s2 + sbyte(S, g0 + 6) * s3;
}

// ---- one lane's share of a quantized row . Q8_K activation ---------------------------------------
// Row `n` of a plane-layout matrix (N rows, nb blocks); this lane takes units u = lane, lane+32, ...
// Units are taken two at a time with both units' weight loads issued before either is used (the
// sum keeps the unit order).
template <int TYPE> struct RowUnit;
template <> struct RowUnit<T_Q4K> {
    uint4 w, h;
    int b, c8;
    __device__ __forceinline__ void load(const uint8_t* base, int64_t nblk_total, int64_t row, int nb, int u) {
        b = u >> 3;
        c8 = u & 7;
        const int64_t blk = row * nb + b;
        const Q4KPlanes p(base, nblk_total);
        w = ld16_stream(p.qs + blk * 128 + 16 * c8);
        h = ld16(p.hdr + blk * 16);
    }
    __device__ __forceinline__ float dot(const ActRow& a) const {
        return q4k_unit_dot(w, h, c8, a.q + QK * b, a.bs + 16 * b, a.d[b]);
    }
};
template <> struct RowUnit<T_Q6K> {
    uint4 A, B, C, S;
    float d6;
    int b, v;
    __device__ __forceinline__ void load(const uint8_t* base, int64_t nblk_total, int64_t row, int nb, int u) {
        b = u >> 2;
        v = u & 3;
        const int h2 = v >> 1, r = v & 1;
        const int64_t blk = row * nb + b;
        const Q6KPlanes p(base, nblk_total);
        A = ld16_stream(p.ql + blk * 128 + 64 * h2 + 16 * r);
        B = ld16_stream(p.ql + blk * 128 + 64 * h2 + 32 + 16 * r);
        C = ld16_stream(p.qh + blk * 64 + 32 * h2 + 16 * r);
        S = ld16(p.sc + blk * 16);
        d6 = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p.d + blk * 2)));
    }
    __device__ __forceinline__ float dot(const ActRow& a) const {
        const int is = q6k_unit_isum(A, B, C, S, v, a.q + QK * b, a.bs + 16 * b);
        return a.d[b] * d6 * (float)is;
    }
};

template <int TYPE>
__device__ __forceinline__ float row_dot_lane(const uint8_t* base, int64_t nblk_total, int64_t row, int nb,
                                              const ActRow& a, int lane) {
    float acc = 0.f;
    const int nunits = nb * (TYPE == T_Q4K ? 8 : 4);
    int u = lane;
    for (; u + 32 < nunits; u += 64) {
        RowUnit<TYPE> x0, x1;
        x0.load(base, nblk_total, row, nb, u);
        x1.load(base, nblk_total, row, nb, u + 32);
        acc += x0.dot(a);
        acc += x1.dot(a);
    }
    if (u < nunits) {
        RowUnit<TYPE> x0;
        x0.load(base, nblk_total, row, nb, u);
        acc += x0.dot(a);
    }
    return acc;
}

// ---- reductions --------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

template <typename R> __device__ __forceinline__ float to_f32(R v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename R> __device__ __forceinline__ R from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

}  // namespace hoard
