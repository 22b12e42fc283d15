// k_ep.cu -- expert-parallel dispatch/combine kernels for the prefill MoE.
//
// Experts are sharded contiguously: rank r owns experts [r*epr, (r+1)*epr).
// For the assignments (token t, slot k) of this rank's tokens:
//   count    destination rank of each assignment and its position among the
//            assignments bound for that rank (atomic order -- the position
//            decides only which send row it occupies, never a value);
//   pack     send row p = offset(dst) + pos: the token's bf16 row, its local
//            expert index and routing weight; send_pos[a] = p;
//   combine  out[t] = sum_k ret[send_pos[t*topk + k]] in slot order, where
//            ret holds the weighted expert outputs returned by the owners in
//            send-row order (deterministic: fixed order per token).
// The all-to-all exchanges between pack, the owners' grouped GEMMs and
// combine go through NCCL (qw6_b200/ep.py).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qw6_launch.h"

namespace qw6 {

__global__ void k_ep_count(const int32_t* __restrict__ idx, int n, int epr, int32_t* __restrict__ cnt,
                           int32_t* __restrict__ pos) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a < n) pos[a] = atomicAdd(&cnt[idx[a] / epr], 1);
}

// one warp per assignment: 16-byte copies of the token row
__global__ void k_ep_pack(const int32_t* __restrict__ idx, const float* __restrict__ w, const int32_t* __restrict__ pos,
                          const int32_t* __restrict__ cnt, int n, int topk, int world, int epr,
                          const __nv_bfloat16* __restrict__ x, int hidden, __nv_bfloat16* __restrict__ send_x,
                          int32_t* __restrict__ send_e, float* __restrict__ send_w, int32_t* __restrict__ send_pos) {
    __shared__ int off[64];
    if (threadIdx.x == 0) {
        int o = 0;
        for (int r = 0; r < world; r++) {
            off[r] = o;
            o += cnt[r];
        }
    }
    __syncthreads();
    const int a = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (a >= n) return;
    const int e = idx[a], dst = e / epr, p = off[dst] + pos[a];
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(a / topk) * hidden);
    uint4* dstp = reinterpret_cast<uint4*>(send_x + (size_t)p * hidden);
    for (int i = lane; i < hidden / 8; i += 32) dstp[i] = src[i];
    if (lane == 0) {
        send_e[p] = e - dst * epr;
        send_w[p] = w[a];
        send_pos[a] = p;
    }
}

__global__ void k_ep_combine(const float* __restrict__ ret, const int32_t* __restrict__ send_pos, int topk, int hidden,
                             float* __restrict__ out) {
    const int t = blockIdx.y, f = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (f >= hidden) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; k++) {
        const float4 v = *reinterpret_cast<const float4*>(ret + (size_t)send_pos[t * topk + k] * hidden + f);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    *reinterpret_cast<float4*>(out + (size_t)t * hidden + f) = acc;
}

}  // namespace qw6

using namespace qw6;

extern "C" int qw6k_ep_count(const int32_t* idx, uint32_t n, uint32_t world, uint32_t epr, int32_t* cnt, int32_t* pos,
                             cudaStream_t st) {
    if (!idx || !cnt || !pos || !n || !world || world > 64 || !epr) return QW6K_ERR_ARG;
    if (cudaMemsetAsync(cnt, 0, world * sizeof(int32_t), st) != cudaSuccess) return QW6K_ERR_CUDA;
    k_ep_count<<<(n + 255) / 256, 256, 0, st>>>(idx, (int)n, (int)epr, cnt, pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_pack(const int32_t* idx, const float* w, const int32_t* pos, const int32_t* cnt, uint32_t n,
                            uint32_t topk, uint32_t world, uint32_t epr, const void* x_bf16, uint32_t hidden,
                            void* send_x, int32_t* send_e, float* send_w, int32_t* send_pos, cudaStream_t st) {
    if (!idx || !w || !pos || !cnt || !x_bf16 || !send_x || !send_e || !send_w || !send_pos || !n || !topk ||
        !world || world > 64 || !epr || hidden % 8)
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x_bf16) | reinterpret_cast<uintptr_t>(send_x)) & 15u) return QW6K_ERR_ALIGN;
    k_ep_pack<<<(n + 7) / 8, 256, 0, st>>>(idx, w, pos, cnt, (int)n, (int)topk, (int)world, (int)epr,
                                          (const __nv_bfloat16*)x_bf16, (int)hidden, (__nv_bfloat16*)send_x, send_e,
                                          send_w, send_pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_combine(const float* ret, const int32_t* send_pos, uint32_t ntok, uint32_t topk,
                               uint32_t hidden, float* out, cudaStream_t st) {
    if (!ret || !send_pos || !out || !ntok || !topk || hidden % 4) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(ret) | reinterpret_cast<uintptr_t>(out)) & 15u) return QW6K_ERR_ALIGN;
    dim3 g((hidden / 4 + 255) / 256, ntok);
    k_ep_combine<<<g, 256, 0, st>>>(ret, send_pos, (int)topk, (int)hidden, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
