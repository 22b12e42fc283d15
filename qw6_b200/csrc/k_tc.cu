// k_tc.cu -- dense bf16 GEMM on the 5th-generation tensor cores (tcgen05,
// accumulators in TMEM): D[M x N] (fp32) = A[M x K] . B[N x K]^T, both
// operands K-major bf16.  It is the reference use of the primitives in
// qw6_tc.cuh, which the dequantizing grouped MoE GEMM builds on, and is
// exposed as qw6cu_gemm_bf16_nt.
//
// CTA = 4 warps, tile M 128 x N BN, K slabs of 64.  All threads stage both
// operands into the 128-byte-swizzled layout (two stages); thread 0 issues
// four K=16 MMAs per slab and commits them to the stage's mbarrier, which
// frees the stage two slabs later.  Waits are time-bounded (error word).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qw6_devcfg.cuh"
#include "qw6_launch.h"
#include "qw6_tc.cuh"

namespace qw6 {

template <int BN>
__global__ void __launch_bounds__(128) k_gemm_bf16_nt(const __nv_bfloat16* __restrict__ A,
                                                      const __nv_bfloat16* __restrict__ B, float* __restrict__ D,
                                                      int M, int N, int K, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = BN * 128, STAGE = A_BYTES + B_BYTES;
    __shared__ uint64_t mbar[2];
    __shared__ uint32_t tmem_base;
    __shared__ int ncommit[2];  // commits issued per stage (for the error-path drain)
    const int tid = threadIdx.x, warp = tid >> 5;
    const int m0 = blockIdx.x * 128, n0 = blockIdx.y * BN;

    if (warp == 0) tmem_alloc(&tmem_base, BN < 32 ? 32 : BN);
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_fence_init();
        ncommit[0] = ncommit[1] = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
    const int nk = K / 64;
    bool ok = true;

    for (int ks = 0; ks < nk && ok; ks++) {
        const int s = ks & 1;
        if (ks >= 2) ok = mbar_wait(&mbar[s], ((ks - 2) >> 1) & 1, err, 1);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        uint8_t* sa = smem + s * STAGE;
        uint8_t* sb = sa + A_BYTES;
        for (int i = tid; i < 128 * 8; i += 128) {
            const int r = i >> 3, c = i & 7, gr = m0 + r;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (gr < M) v = *reinterpret_cast<const uint4*>(A + (size_t)gr * K + ks * 64 + c * 8);
            *reinterpret_cast<uint4*>(sa + sw128_off(r, c)) = v;
        }
        for (int i = tid; i < BN * 8; i += 128) {
            const int r = i >> 3, c = i & 7, gr = n0 + r;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (gr < N) v = *reinterpret_cast<const uint4*>(B + (size_t)gr * K + ks * 64 + c * 8);
            *reinterpret_cast<uint4*>(sb + sw128_off(r, c)) = v;
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++)
                umma_bf16(tmem, umma_desc_sw128(a0 + 32 * k4), umma_desc_sw128(b0 + 32 * k4), idesc,
                          (ks > 0 || k4 > 0) ? 1u : 0u);
            umma_commit(&mbar[s]);
            ncommit[s]++;
        }
    }
    if (ok && nk > 0) ok = mbar_wait(&mbar[(nk - 1) & 1], ((nk - 1) >> 1) & 1, err, 2);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        const int row = m0 + warp * 32 + (tid & 31);
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
            if (row < M) {
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (n0 + c0 + j < N) D[(size_t)row * N + n0 + c0 + j] = v[j];
            }
        }
    } else {
        // a wait gave up: wait (bounded) for every committed MMA batch before freeing TMEM
        __syncthreads();
        for (int s = 0; s < 2; s++)
            if (ncommit[s] > 0) mbar_wait(&mbar[s], (ncommit[s] - 1) & 1, nullptr, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, BN < 32 ? 32 : BN);
}

template <int BN>
static int launch_gemm(const void* A, const void* B, float* D, int M, int N, int K, int* err, cudaStream_t st) {
    const size_t smem = 2 * (128 * 128 + BN * 128) + 1024;
    static DevFlags cfg;
    if (smem_optin(cfg, k_gemm_bf16_nt<BN>, (int)smem)) return QW6K_ERR_CUDA;
    dim3 grid((M + 127) / 128, (N + BN - 1) / BN);
    k_gemm_bf16_nt<BN><<<grid, 128, smem, st>>>((const __nv_bfloat16*)A, (const __nv_bfloat16*)B, D, M, N, K, err);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

}  // namespace qw6

extern "C" int qw6k_gemm_bf16_nt(const void* A, const void* B, float* D, uint32_t M, uint32_t N, uint32_t K,
                                 int* err, cudaStream_t st) {
    if (!A || !B || !D || !err || !M || !N || !K || K % 64 || M > (1u << 24) || N > (1u << 24)) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15u) return QW6K_ERR_ALIGN;
    if (N <= 64) return qw6::launch_gemm<64>(A, B, D, (int)M, (int)N, (int)K, err, st);
    if (N <= 128) return qw6::launch_gemm<128>(A, B, D, (int)M, (int)N, (int)K, err, st);
    return qw6::launch_gemm<256>(A, B, D, (int)M, (int)N, (int)K, err, st);
}
