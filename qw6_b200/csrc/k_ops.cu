// k_ops.cu -- routing, combine, activation, argmax and fp32 matvec kernels.
//
// Semantics follow qw6's CPU reference, which is the parity target:
//   moe_route  qw6_cpu_moe_route  qw6.c:2796-2827  (Vulkan: moe_route.comp)
//   gather     moe_gather.comp:17-29 (sum in selection order, then shared)
//   silu_mul   qw6.c:2258 with qw6_silu qw6.h:292-294 (silu_mul.comp)
//   argmax     qw6_cpu_argmax     qw6.c:2858-2863  (argmax.comp/sampling.comp
//              break ties by lane; here ties go to the lowest index like the
//              CPU path)
#include <cuda_runtime.h>

#include <cstdint>

#include "qw6_launch.h"
#include "qw6_pdl.cuh"
#include "qw6_argmax.cuh"
#include "qw6_route.cuh"

namespace qw6 {

__global__ void k_route(const float* logits, int ntok, int ne, int k, int32_t* idx, float* w) {
    pdl_grid_wait();
    const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (tok >= ntok) return;
    route_token(logits + (size_t)tok * ne, ne, k, idx + (size_t)tok * k, w + (size_t)tok * k, threadIdx.x & 31);
}

// --------------------------------------------------------------- gather --
__global__ void k_gather(const float* __restrict__ eo, const float* __restrict__ w, const float* __restrict__ sh,
                         float sw, float* __restrict__ out, int dim, int k) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    float acc = 0.f;
    for (int e = 0; e < k; e++) acc = __fadd_rn(acc, __fmul_rn(w[e], eo[(size_t)e * dim + i]));
    if (sh) acc = __fadd_rn(acc, __fmul_rn(sw, sh[i]));
    out[i] = acc;
}

// ------------------------------------------------------------- silu_mul --
__device__ __forceinline__ float silu_ref(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }

__global__ void k_silu_mul(const float* g, const float* u, float* o, int n) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) o[i] = __fmul_rn(silu_ref(g[i]), u[i]);
}

// --------------------------------------------------------------- argmax --
// (keys: qw6_argmax.cuh)
__global__ void k_argmax_partial(const float* __restrict__ x, uint32_t n, unsigned long long* __restrict__ key) {
    unsigned long long best = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long kk = argmax_key(x[i], i);
        best = kk > best ? kk : best;
    }
    best = warp_max_u64(best);
    __shared__ unsigned long long s[32];
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0;
        best = warp_max_u64(best);
        if (threadIdx.x == 0) atomicMax(key, best);
    }
}

__global__ void k_argmax_final(const float* __restrict__ x, uint32_t n, const unsigned long long* __restrict__ key,
                               uint32_t* __restrict__ out_idx, float* __restrict__ out_val) {
    uint32_t i = ~(uint32_t)(*key & 0xffffffffull);
    if (i >= n) i = 0;  // unreachable: every element contributes a non-zero key
    *out_idx = i;
    if (out_val) *out_val = x[i];
}

// keys[s*ntok + t] for s < nshards: max over shards, then (index, value).
__global__ void k_argmax_keys_reduce(const unsigned long long* __restrict__ keys, int nshards, int ntok,
                                     uint32_t* __restrict__ idx, float* __restrict__ val) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= ntok) return;
    unsigned long long k = 0;
    for (int s = 0; s < nshards; s++) {
        const unsigned long long v = keys[(size_t)s * ntok + t];
        k = v > k ? v : k;
    }
    idx[t] = argmax_key_index(k);
    if (val) val[t] = argmax_key_value(k);
}

// ------------------------------------------------------------ f32 matvec --
// One warp per row, float4 loads when the row is 16-byte aligned.
__global__ void k_matvec_f32(const float* __restrict__ w, const float* __restrict__ x, float* __restrict__ y,
                             int rows, int cols) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* wr = w + (size_t)row * cols;
    float acc = 0.f;
    if ((cols & 3) == 0 && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15u) == 0) {
        const float4* w4 = reinterpret_cast<const float4*>(wr);
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int c = lane; c < cols / 4; c += 32) {
            const float4 a = w4[c], b = x4[c];
            acc = fmaf(a.x, b.x, acc);
            acc = fmaf(a.y, b.y, acc);
            acc = fmaf(a.z, b.z, acc);
            acc = fmaf(a.w, b.w, acc);
        }
    } else {
        for (int c = lane; c < cols; c += 32) acc = fmaf(wr[c], x[c], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = acc;
}

}  // namespace qw6

using namespace qw6;

static int launched() { return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA; }

extern "C" int qw6k_moe_route(const float* logits, uint32_t ntok, uint32_t n_experts, uint32_t top_k, int32_t* idx,
                              float* w, cudaStream_t st) {
    if (!logits || !idx || !w || !ntok || !n_experts || n_experts > 256 || !top_k || top_k > 32 ||
        top_k > n_experts)
        return QW6K_ERR_ARG;
    const int wpb = 4;
    if (launch_pdl(k_route, dim3((ntok + wpb - 1) / wpb), dim3(32 * wpb), 0, st, logits, (int)ntok, (int)n_experts,
                   (int)top_k, idx, w) != cudaSuccess)
        return QW6K_ERR_CUDA;
    return launched();
}

extern "C" int qw6k_moe_gather(const float* eo, const float* w, const float* shared, float sw, float* out,
                               uint32_t dim, uint32_t top_k, cudaStream_t st) {
    if (!eo || !w || !out || !dim || !top_k) return QW6K_ERR_ARG;
    k_gather<<<(dim + 255) / 256, 256, 0, st>>>(eo, w, shared, sw, out, (int)dim, (int)top_k);
    return launched();
}

extern "C" int qw6k_silu_mul(const float* g, const float* u, float* o, uint32_t n, cudaStream_t st) {
    if (!g || !u || !o || !n) return QW6K_ERR_ARG;
    return launch_pdl(k_silu_mul, dim3((n + 255) / 256), dim3(256), 0, st, g, u, o, (int)n) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_argmax(const float* x, uint32_t n, unsigned long long* key64, uint32_t* out_idx, float* out_val,
                           cudaStream_t st) {
    if (!x || !n || !key64 || !out_idx) return QW6K_ERR_ARG;
    if (cudaMemsetAsync(key64, 0, sizeof(unsigned long long), st) != cudaSuccess) return QW6K_ERR_CUDA;
    unsigned blocks = (n + 255) / 256;
    if (blocks > 592) blocks = 592;
    k_argmax_partial<<<blocks, 256, 0, st>>>(x, n, key64);
    k_argmax_final<<<1, 1, 0, st>>>(x, n, key64, out_idx, out_val);
    return launched();
}

extern "C" int qw6k_argmax_keys_reduce(const unsigned long long* keys, uint32_t nshards, uint32_t ntok, uint32_t* idx,
                                       float* val, cudaStream_t st) {
    if (!keys || !idx || !nshards || !ntok) return QW6K_ERR_ARG;
    k_argmax_keys_reduce<<<(ntok + 127) / 128, 128, 0, st>>>(keys, (int)nshards, (int)ntok, idx, val);
    return launched();
}

extern "C" int qw6k_matvec_f32(const float* w, const float* x, float* y, uint32_t rows, uint32_t cols,
                               cudaStream_t st) {
    if (!w || !x || !y || !rows || !cols) return QW6K_ERR_ARG;
    k_matvec_f32<<<(rows + 7) / 8, 256, 0, st>>>(w, x, y, (int)rows, (int)cols);
    return launched();
}
