// qw6_argmax.cuh -- packed (value, index) keys for argmax reductions.
//
// key = ordered(value) << 32 | ~index, where ordered() is an order-preserving
// float -> uint32 map, so a larger key is a larger value and, among equal
// values, a lower index: the result of qw6_cpu_argmax's strict '>' scan
// (qw6.c:2858-2863).  NaN orders as -inf except at index 0, which takes the
// maximal key (the CPU scan never moves past a NaN x[0]).  The max of keys is
// associative and commutative, so per-warp partials, atomicMax and the
// combination of row shards all give the same answer as one scan.
#pragma once

#include <cstdint>

namespace qw6 {

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i) {
    uint32_t u;
    if (isnan(v)) {
        if (i == 0) return ~0ull;
        u = 0x007fffffu;  // ordered(-inf)
    } else {
        const uint32_t b = __float_as_uint(v);
        u = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return ((unsigned long long)u << 32) | (unsigned long long)(~i);
}

__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
    if (k == ~0ull) return __uint_as_float(0x7fc00000u);
    const uint32_t u = (uint32_t)(k >> 32);
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) { return ~(uint32_t)(k & 0xffffffffull); }

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, k, o);
        k = x > k ? x : k;
    }
    return k;
}

}  // namespace qw6
