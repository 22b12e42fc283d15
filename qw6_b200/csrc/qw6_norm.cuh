// qw6_norm.cuh -- qw6's RMSNorm factor on the GPU (qw6_cpu_rmsnorm,
// qw6.c:2503-2513): 1 / sqrtf(sum(x^2) / dim + 1e-6f).
#pragma once
#include <cuda_runtime.h>

namespace qw6 {

constexpr float kRmsEps = 1e-6f;  // QW6_RMS_EPS (qw6.h:67)

// Sum of v over the CTA (every thread gets it); red: blockDim.x / 32 floats
// of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
    __syncthreads();
    return t;
}

// 1 / sqrt(sum(x^2)/dim + eps) for the row x (every thread gets it).  The sum
// is a block reduction (qw6 sums sequentially; the difference is fp32
// rounding of the sum), the rest is qw6's expression with IEEE operations.
__device__ __forceinline__ float rms_inv(const float* __restrict__ x, int dim, float* red) {
    float ss = 0.f;
#pragma unroll 8
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    const float t = block_sum(ss, red);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)dim), kRmsEps)));
}

}  // namespace qw6
