// qw6_tc.cuh -- Blackwell (sm_100a) tensor-core building blocks: tcgen05 MMA
// with TMEM accumulators, UMMA shared-memory descriptors, mbarriers with
// time-bounded waits.
//
// Operand tiles are K-major with the 128-byte swizzle: a row (one M or N
// index) holds 64 bf16 = 128 bytes of K; 8 rows form a 1024-byte atom in
// which 16-byte chunk c of row r is stored at chunk (c ^ (r & 7)).  Atoms are
// stacked along M/N (stride 1024 B).  The MMA's K = 16 sub-steps inside one
// 64-wide K slab advance the descriptor start address by 32 bytes.
#pragma once

#include <cstdint>

namespace qw6 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of (row, 16-byte chunk) inside a SWIZZLE_128B K-major tile
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

// UMMA shared-memory matrix descriptor: K-major, SWIZZLE_128B, SBO = 1024 B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3ffffu) >> 4);  // start address >> 4   (bits 0-13)
    d |= (uint64_t)1 << 16;                      // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;           // stride byte offset  (bits 32-45)
    d |= (uint64_t)1 << 46;                      // descriptor version 0b001 (bits 46-48)
    d |= (uint64_t)2 << 61;                      // layout: SWIZZLE_128B (bits 61-63)
    return d;
}

// Instruction descriptor, kind::f16: BF16 x BF16 -> F32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4)                         // D format F32
           | (1u << 7)                       // A format BF16
           | (1u << 10)                      // B format BF16
           | ((uint32_t)(N >> 3) << 17)      // N / 8
           | ((uint32_t)(M >> 4) << 24);     // M / 16
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on an mbarrier once all prior tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mbar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy smem writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// TMEM allocation (one whole warp); the base address lands in *dst (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes
// 32*(w%4) .. +31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// ----------------------------------------------------------- mbarriers ----

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// Test phase `parity`; if it is not complete yet the thread is suspended
// (without issuing) until the phase completes or kSuspendHintNs pass.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for phase `parity` of an mbarrier, giving up after `limit_ns`: on a
// timeout the error word gets `code` and false is returned (no hang).
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// The clock is read once per 64 suspended polls (each up to kSuspendHintNs).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(b, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; n++) {
        if (mbar_try_wait(b, parity)) return true;
        if ((n & 63) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
            if (err) atomicExch(err, code);
            return false;
        }
    }
}

}  // namespace qw6
