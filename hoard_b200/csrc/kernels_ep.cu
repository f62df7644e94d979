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

// ---- over NVLink peer memory ----

// Exclusive prefix of the per-destination counts (this rank's send order), and both written into
// every destination's count[rank] / start[rank].
__global__ void k_p2p_meta(P2PSend p, const int* __restrict__ counts, int* __restrict__ cursor,
                           int* __restrict__ start) {
    if (threadIdx.x != 0) return;
    int acc = 0;
    for (int g = 0; g < p.G; ++g) {
        const int c = counts[g];
        cursor[g] = acc;
        start[g] = acc;
        reinterpret_cast<int*>(p.peer[g] + p.L.count)[p.rank] = c;
        reinterpret_cast<int*>(p.peer[g] + p.L.start)[p.rank] = acc;
        acc += c;
    }
}

// One warp per token (lanes j < k: its entries): send positions (warp-aggregated cursors per
// destination), each entry's expert id and token row into its destination's region `rank`; the first
// lane of each destination group takes one row of that destination's region for the token, so a token
// row crosses NVLink once per destination rank, not once per expert. Row order within a region is
// arbitrary: every entry's arithmetic is independent of its neighbours.
__global__ void __launch_bounds__(256) k_p2p_scatter(P2PSend p, const int32_t* __restrict__ sel, int T, int k,
                                                     int* __restrict__ cursor, const int* __restrict__ start,
                                                     int* __restrict__ rcursor, int* __restrict__ pos_of_entry,
                                                     int* __restrict__ rowinfo) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;                                   // whole warps
    const int64_t e = (int64_t)t * k + lane;
    int dest = -1 - lane, ex = -1;                        // absent / rejected entries: groups of one
    if (lane < k) {
        ex = sel[e];
        if (ex >= 0 && ex < p.G * p.epr) dest = ex / p.epr;
    }
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, dest);
    const int leader = __ffs(peers) - 1;
    int q = 0, rr = 0;
    if (lane == leader && dest >= 0) {
        q = atomicAdd(&cursor[dest], __popc(peers));
        rr = atomicAdd(&rcursor[dest], 1);
    }
    q = __shfl_sync(0xFFFFFFFFu, q, leader);
    rr = __shfl_sync(0xFFFFFFFFu, rr, leader);
    if (lane < k) {
        if (dest >= 0) {
            const int pos = q + __popc(peers & ((1u << lane) - 1u));
            pos_of_entry[e] = pos;
            const int64_t i = (int64_t)p.rank * p.cap + (pos - start[dest]);
            reinterpret_cast<int32_t*>(p.peer[dest] + p.L.expert)[i] = ex;
            reinterpret_cast<int32_t*>(p.peer[dest] + p.L.row_of)[i] = rr;
            rowinfo[e] = lane == leader ? rr : -1;
        } else {
            pos_of_entry[e] = -1;
            rowinfo[e] = -1;
        }
    }
}

// One warp per entry that sends its token's row (rowinfo >= 0): the f16 row into row rowinfo of the
// destination's region `rank`, 16-byte stores (512 contiguous bytes per warp instruction over NVLink).
__global__ void __launch_bounds__(256) k_p2p_gather(P2PSend p, const int32_t* __restrict__ sel,
                                                    const uint16_t* __restrict__ xq, int n, int k,
                                                    const int* __restrict__ rowinfo) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (e >= n) return;
    const int rr = rowinfo[e];
    if (rr < 0) return;
    const int dest = sel[e] / p.epr;
    const int64_t row = (int64_t)p.rank * p.cap_rows + rr;
    const uint4* src = reinterpret_cast<const uint4*>(xq + (int64_t)(e / k) * p.H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.peer[dest] + p.L.rows) + row * p.H);
    for (int i = lane; i < p.H / 8; i += 32) dst[i] = src[i];
}

__global__ void k_p2p_signal(P2PSend p, uint32_t epoch) {
    const int g = threadIdx.x;
    if (g >= p.G) return;
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(p.peer[g] + p.L.flags) + p.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
}

__global__ void k_p2p_wait(const uint8_t* block, int64_t flags_off, int G, uint32_t epoch,
                           unsigned long long timeout_ns, unsigned* err) {
    const int s = threadIdx.x;
    if (s >= G) return;
    if (*(volatile unsigned*)err & 2u) return;            // an earlier wait already gave up
    const uint32_t* f = reinterpret_cast<const uint32_t*>(block + flags_off) + s;
    unsigned long long t0 = 0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if ((int32_t)(v - epoch) >= 0) break;
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > timeout_ns) {
            atomicOr(err, 2u);
            break;
        }
        __nanosleep(200);
    }
    __threadfence_system();
}

}  // namespace

P2PLayout p2p_layout(int G, int cap, int cap_rows, int H) {
    auto al = [](int64_t v) { return (v + 255) / 256 * 256; };
    P2PLayout L{};
    L.flags = 0;
    L.count = 256;
    L.start = 512;
    L.expert = 1024;
    L.row_of = al(L.expert + (int64_t)G * cap * 4);
    L.rows = al(L.row_of + (int64_t)G * cap * 4);
    L.yback = al(L.rows + (int64_t)G * cap_rows * H * 2);
    L.bytes = al(L.yback + (int64_t)cap * H * 2);
    return L;
}

cudaError_t launch_p2p_send(const P2PSend& p, const int32_t* sel, int T, int k, const uint16_t* xq, int* counts,
                            int* cursor, int* start, int* rcursor, int* pos_of_entry, int* rowinfo, unsigned* err,
                            cudaStream_t s, int* launches) {
    if (p.G < 1 || p.G > EP_MAX_RANKS || k < 1 || k > 32 || T > p.cap_rows) return cudaErrorInvalidValue;
    const int n = T * k;
    cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)p.G * sizeof(int), s);
    if (e != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(rcursor, 0, (size_t)p.G * sizeof(int), s)) != cudaSuccess) return e;
    const int grid = (n + EP_CHUNK - 1) / EP_CHUNK;
    k_ep_count<<<grid, 256, 0, s>>>(sel, n, p.G, p.epr, counts, err);
    k_p2p_meta<<<1, 32, 0, s>>>(p, counts, cursor, start);
    k_p2p_scatter<<<(T + 7) / 8, 256, 0, s>>>(p, sel, T, k, cursor, start, rcursor, pos_of_entry, rowinfo);
    k_p2p_gather<<<(n + 7) / 8, 256, 0, s>>>(p, sel, xq, n, k, rowinfo);
    if (launches) *launches += 4;
    return cudaGetLastError();
}

cudaError_t launch_p2p_signal(const P2PSend& p, uint32_t epoch, cudaStream_t s) {
    k_p2p_signal<<<1, 64, 0, s>>>(p, epoch);
    return cudaGetLastError();
}

cudaError_t launch_p2p_wait(const uint8_t* block, const P2PLayout& L, int G, uint32_t epoch,
                            unsigned long long timeout_ns, unsigned* err, cudaStream_t s) {
    k_p2p_wait<<<1, 64, 0, s>>>(block, L.flags, G, epoch, timeout_ns, err);
    return cudaGetLastError();
}

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
