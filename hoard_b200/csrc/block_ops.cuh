// block_ops.cuh -- CTA-wide reductions shared by the grouped path and the persistent decode kernel.
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

}  // namespace hoard
