// block_ops.cuh -- CTA-wide reductions and the router's softmax + top-k, shared by the grouped
// path and the persistent decode kernel so both select experts with identical arithmetic.
#pragma once
#include "common.cuh"

namespace hoard {

// ---------------------------------------------------------------------------------------------
// block reductions (any multiple of 32 threads, <= 1024)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ double block_sum_d(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double r = 0.0;
    for (int i = 0; i < nw; ++i) r += red[i];
    return r;
}

__device__ __forceinline__ float block_max_f(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
    return r;
}

// softmax over E logits held in shared memory (in place -> probabilities), then top-k by rank:
// rank(e) = #{j : p_j > p_e} + #{j < e : p_j == p_e}, i.e. descending with ties to the lower id.
static __device__ __noinline__ void softmax_topk(float* lg, int E, int k, int renorm, int32_t* sel, float* w, double* redd,
                             float* redf, int* s_sel, float* s_w) {
    float m = -INFINITY;
    for (int e = threadIdx.x; e < E; e += blockDim.x) m = fmaxf(m, lg[e]);
    m = block_max_f(m, redf);
    double s = 0.0;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const float v = expf(lg[e] - m);
        lg[e] = v;
        s += (double)v;
    }
    s = block_sum_d(s, redd);
    const float inv = (float)(1.0 / s);
    for (int e = threadIdx.x; e < E; e += blockDim.x) lg[e] *= inv;
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const float p = lg[e];
        int rank = 0;
        for (int j = 0; j < E; ++j) {
            const float q = lg[j];
            rank += (q > p) || (q == p && j < e);
        }
        if (rank < k) { s_sel[rank] = e; s_w[rank] = p; }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (renorm) {
            float sum = 0.f;
            for (int j = 0; j < k; ++j) sum += s_w[j];
            if (sum < 6.103515625e-5f) sum = 6.103515625e-5f;
            for (int j = 0; j < k; ++j) s_w[j] /= sum;
        }
        for (int j = 0; j < k; ++j) { sel[j] = s_sel[j]; w[j] = s_w[j]; }
    }
    __syncthreads();
}

}  // namespace hoard
