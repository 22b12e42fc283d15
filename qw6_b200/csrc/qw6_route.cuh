// qw6_route.cuh -- warp-level top-k expert selection shared by the routing
// and MoE planning kernels (semantics of qw6_cpu_moe_route, qw6.c:2796-2827).
#pragma once

#include <cstdint>

namespace qw6 {

// ---------------------------------------------------------------- route --
// One warp per token.  Lane l holds logits l, l+32, ..., so scanning its
// slots in order and keeping strict '>' finds its lowest-index maximum; the
// warp merge prefers the higher value, then the lower index.  qw6's scan
// starts from element 0 and only replaces on a strict '>', hence: a NaN at
// index 0 wins the round; any other NaN never wins (treated as -inf); when
// every remaining value is -inf, index 0 is chosen (possibly again).

__device__ __forceinline__ void route_token(const float* __restrict__ lg, int ne, int k, int32_t* __restrict__ idx,
                                            float* __restrict__ w, int lane) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = lane + 32 * i;
        v[i] = e < ne ? lg[e] : -INFINITY;
    }
    float sel[32];
    int seli[32];
    for (int r = 0; r < k; r++) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = lane + 32 * i;
            const float c = isnan(v[i]) ? -INFINITY : v[i];
            if (e < ne && (c > bv || bi == 0x7fffffff)) {
                bv = c;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        const float v0 = __shfl_sync(0xffffffffu, v[0], 0);
        if (isnan(v0)) bi = 0;
        // the winner's original value (NaN stays NaN)
        const int owner = bi & 31, slot = bi >> 5;
        float mine = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i == slot) mine = v[i];
        const float orig = __shfl_sync(0xffffffffu, mine, owner);
        if (lane == owner) {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (i == slot) v[i] = -INFINITY;
        }
        sel[r & 31] = orig;
        seli[r & 31] = bi;
    }
    if (lane == 0) {
        float mx = sel[0];
        for (int r = 1; r < k; r++)
            if (sel[r] > mx) mx = sel[r];
        float sum = 0.f;
        for (int r = 0; r < k; r++) {
            sel[r] = expf(__fsub_rn(sel[r], mx));
            sum = __fadd_rn(sum, sel[r]);
        }
        for (int r = 0; r < k; r++) {
            idx[r] = seli[r];
            w[r] = __fdiv_rn(sel[r], sum);
        }
    }
}

}  // namespace qw6
