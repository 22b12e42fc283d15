// k_ep.cu -- expert-parallel dispatch/combine kernels for the prefill MoE.
//
// Experts are sharded contiguously: rank r owns experts [r*epr, (r+1)*epr).
// For the assignments a = t*topk + k of this rank's tokens:
//   count    per-GLOBAL-expert assignment counts and each assignment's
//            position among those of its expert (atomic order -- it decides
//            only which send row an assignment occupies, never a value);
//   pack     send row p = (exclusive prefix of the counts over experts)[e]
//            + pos[a] gets the token's bf16 row; send_pos[a] = p.  Send rows
//            are therefore sorted by global expert, which also groups them
//            by destination rank, and inside each destination's block by
//            the destination's local expert -- the receiver recovers every
//            row's expert from the exchanged per-expert counts alone;
//   expand   on the owner: row_expert of every received row from the
//            [source][local expert] count matrix;
//   combine  out[t] = sum_k w[a] * ret[send_pos[a]] (fp32 fma, slot order),
//            where ret holds the owners' unweighted bf16 expert outputs
//            returned in send-row order -- the same arithmetic, in the same
//            order, as the single-GPU prefill combine.
// The all-to-all exchanges in between go through NCCL (qw6_b200/ep.py).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qw6_launch.h"

namespace qw6 {

__global__ void k_ep_count(const int32_t* __restrict__ idx, int n, int32_t* __restrict__ cnt,
                           int32_t* __restrict__ pos) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a < n) pos[a] = atomicAdd(&cnt[idx[a]], 1);
}

// exclusive prefix of cnt[0..ne) into off[] (ne <= 256, blockDim 256)
__device__ __forceinline__ void block_prefix256(const int32_t* __restrict__ cnt, int ne, int* off) {
    __shared__ int wsum[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int v = tid < ne ? cnt[tid] : 0;
    int s = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, s, d);
        if (lane >= d) s += u;
    }
    if (lane == 31) wsum[warp] = s;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; w++) base += wsum[w];
    off[tid] = base + s - v;
    __syncthreads();
}

// one warp per assignment: 16-byte copies of the token row
__global__ void __launch_bounds__(256) k_ep_pack(const int32_t* __restrict__ idx, const int32_t* __restrict__ pos,
                                                 const int32_t* __restrict__ cnt, int n, int topk, int ne,
                                                 const __nv_bfloat16* __restrict__ x, int hidden,
                                                 __nv_bfloat16* __restrict__ send_x, int32_t* __restrict__ send_pos) {
    __shared__ int off[256];
    block_prefix256(cnt, ne, off);
    const int a = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (a >= n) return;
    const int p = off[idx[a]] + pos[a];
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(a / topk) * hidden);
    uint4* dstp = reinterpret_cast<uint4*>(send_x + (size_t)p * hidden);
    for (int i = lane; i < hidden / 8; i += 32) dstp[i] = src[i];
    if (lane == 0) send_pos[a] = p;
}

// recv_cnt[s*epr + e] rows from source s for local expert e arrive in
// (s, e) order; row_expert[r] = e of received row r.
__global__ void __launch_bounds__(256) k_ep_expand(const int32_t* __restrict__ recv_cnt, int nblk, int epr,
                                                   int32_t* __restrict__ row_expert) {
    __shared__ int off[256];
    block_prefix256(recv_cnt, nblk, off);
    const int b = blockIdx.x;  // one CTA per (source, local expert) block
    const int o = off[b], c = recv_cnt[b], e = b % epr;
    for (int i = threadIdx.x; i < c; i += blockDim.x) row_expert[o + i] = e;
}

__global__ void k_ep_combine(const __nv_bfloat16* __restrict__ ret, const float* __restrict__ w,
                             const int32_t* __restrict__ send_pos, int topk, int hidden, float* __restrict__ out) {
    const int t = blockIdx.y, f = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (f >= hidden) return;
    float o0 = 0.f, o1 = 0.f;
    for (int k = 0; k < topk; k++) {
        const size_t a = (size_t)t * topk + k;
        const float wk = w[a];
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(ret + (size_t)send_pos[a] * hidden + f);
        o0 = fmaf(wk, __bfloat162float(v.x), o0);
        o1 = fmaf(wk, __bfloat162float(v.y), o1);
    }
    *reinterpret_cast<float2*>(out + (size_t)t * hidden + f) = make_float2(o0, o1);
}

}  // namespace qw6

using namespace qw6;

extern "C" int qw6k_ep_count(const int32_t* idx, uint32_t n, uint32_t ne, int32_t* cnt, int32_t* pos,
                             cudaStream_t st) {
    if (!idx || !cnt || !pos || !n || !ne || ne > 256) return QW6K_ERR_ARG;
    if (cudaMemsetAsync(cnt, 0, ne * sizeof(int32_t), st) != cudaSuccess) return QW6K_ERR_CUDA;
    k_ep_count<<<(n + 255) / 256, 256, 0, st>>>(idx, (int)n, cnt, pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_pack(const int32_t* idx, const int32_t* pos, const int32_t* cnt, uint32_t n, uint32_t topk,
                            uint32_t ne, const void* x_bf16, uint32_t hidden, void* send_x, int32_t* send_pos,
                            cudaStream_t st) {
    if (!idx || !pos || !cnt || !x_bf16 || !send_x || !send_pos || !n || !topk || !ne || ne > 256 || !hidden ||
        hidden % 8)
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x_bf16) | reinterpret_cast<uintptr_t>(send_x)) & 15u) return QW6K_ERR_ALIGN;
    k_ep_pack<<<(n + 7) / 8, 256, 0, st>>>(idx, pos, cnt, (int)n, (int)topk, (int)ne, (const __nv_bfloat16*)x_bf16,
                                          (int)hidden, (__nv_bfloat16*)send_x, send_pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_expand(const int32_t* recv_cnt, uint32_t world, uint32_t epr, int32_t* row_expert,
                              cudaStream_t st) {
    if (!recv_cnt || !row_expert || !world || !epr || world * epr > 256) return QW6K_ERR_ARG;
    k_ep_expand<<<world * epr, 256, 0, st>>>(recv_cnt, (int)(world * epr), (int)epr, row_expert);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_combine(const void* ret_bf16, const float* w, const int32_t* send_pos, uint32_t ntok,
                               uint32_t topk, uint32_t hidden, float* out, cudaStream_t st) {
    if (!ret_bf16 || !w || !send_pos || !out || !ntok || !topk || !hidden || hidden % 2) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(ret_bf16) & 3u) || (reinterpret_cast<uintptr_t>(out) & 7u)) return QW6K_ERR_ALIGN;
    dim3 g((hidden / 2 + 255) / 256, ntok);
    k_ep_combine<<<g, 256, 0, st>>>((const __nv_bfloat16*)ret_bf16, w, send_pos, (int)topk, (int)hidden, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
