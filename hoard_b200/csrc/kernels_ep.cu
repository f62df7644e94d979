// kernels_ep.cu -- the send side of expert-parallel batched tokens (C4: experts [g*E/G, (g+1)*E/G) on
// rank g, tokens data-parallel): the (token, j) entries of a rank's routing are counting-sorted by
// destination rank and their Q8_K-dequantised f16 activation rows gathered into one send buffer, so
// one all-to-all (counts first, then rows) moves them. pos_of_entry[t*k + j] is the entry's row in the
// send buffer; the expert outputs come back in the same order and the combine reads them through it.
// The order of entries within one destination is arbitrary: every row is computed independently.
#include "common.cuh"
#include "kernels.h"

namespace hoard {

namespace {

constexpr int EP_MAX_RANKS = 64;
constexpr int EP_CHUNK = 2048;     // entries per CTA of the count / scatter kernels

__global__ void __launch_bounds__(256) k_ep_count(const int32_t* __restrict__ sel, int n, int n_ranks, int epr,
                                                  int* __restrict__ counts, unsigned* err) {
    __shared__ int hist[EP_MAX_RANKS];
    for (int i = threadIdx.x; i < n_ranks; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int e0 = blockIdx.x * EP_CHUNK, e1 = min(n, e0 + EP_CHUNK);
    for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
        const int ex = sel[e];
        if (ex < 0 || ex >= n_ranks * epr) { atomicOr(err, 1u); continue; }
        atomicAdd(&hist[ex / epr], 1);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n_ranks; i += blockDim.x)
        if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

__global__ void k_ep_offsets(const int* __restrict__ counts, int n_ranks, int* __restrict__ cursor) {
    if (threadIdx.x != 0) return;
    int acc = 0;
    for (int i = 0; i < n_ranks; ++i) {
        cursor[i] = acc;
        acc += counts[i];
    }
}

__global__ void __launch_bounds__(256) k_ep_scatter(const int32_t* __restrict__ sel, int n, int n_ranks, int epr,
                                                    int* __restrict__ cursor, int* __restrict__ pos_of_entry,
                                                    int32_t* __restrict__ send_expert) {
    const int lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * EP_CHUNK, e1 = min(n, e0 + EP_CHUNK);
    for (int base = e0; base < e1; base += blockDim.x) {
        const int e = base + threadIdx.x;
        int dest = -1, ex = -1;
        if (e < e1) {
            ex = sel[e];
            dest = (ex < 0 || ex >= n_ranks * epr) ? -1 : ex / epr;
        }
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, dest);
        const int leader = __ffs(peers) - 1;
        int p = 0;
        if (lane == leader && dest >= 0) p = atomicAdd(&cursor[dest], __popc(peers));
        p = __shfl_sync(0xFFFFFFFFu, p, leader);
        if (e < e1) {
            if (dest >= 0) {
                const int pos = p + __popc(peers & ((1u << lane) - 1u));
                pos_of_entry[e] = pos;
                send_expert[pos] = ex;
            } else {
                pos_of_entry[e] = -1;
            }
        }
    }
}

// one warp per entry: its token's f16 row (H * 2 bytes) into the entry's send row
__global__ void __launch_bounds__(256) k_ep_gather(const uint16_t* __restrict__ xq, int n, int k, int H,
                                                   const int* __restrict__ pos_of_entry, uint16_t* __restrict__ rows) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (e >= n) return;
    const int pos = pos_of_entry[e];
    if (pos < 0) return;
    const uint4* src = reinterpret_cast<const uint4*>(xq + (int64_t)(e / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(rows + (int64_t)pos * H);
    for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

}  // namespace

cudaError_t launch_ep_pack(const int32_t* sel, int T, int k, int n_ranks, int experts_per_rank, const uint16_t* xq,
                           int H, int* counts, int* cursor, int* pos_of_entry, int32_t* send_expert,
                           uint16_t* send_rows, unsigned* err, cudaStream_t s, int* launches) {
    if (n_ranks < 1 || n_ranks > EP_MAX_RANKS) return cudaErrorInvalidValue;
    const int n = T * k;
    cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)n_ranks * sizeof(int), s);
    if (e != cudaSuccess) return e;
    const int grid = (n + EP_CHUNK - 1) / EP_CHUNK;
    k_ep_count<<<grid, 256, 0, s>>>(sel, n, n_ranks, experts_per_rank, counts, err);
    k_ep_offsets<<<1, 32, 0, s>>>(counts, n_ranks, cursor);
    k_ep_scatter<<<grid, 256, 0, s>>>(sel, n, n_ranks, experts_per_rank, cursor, pos_of_entry, send_expert);
    k_ep_gather<<<(n + 7) / 8, 256, 0, s>>>(xq, n, k, H, pos_of_entry, send_rows);
    if (launches) *launches += 4;
    return cudaGetLastError();
}

}  // namespace hoard
