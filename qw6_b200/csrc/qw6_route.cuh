// qw6_route.cuh -- warp-level top-k expert selection shared by the routing
// and MoE planning kernels (semantics of qw6_cpu_moe_route, qw6.c:2796-2827).
#pragma once

#include <cstdint>

namespace qw6 {

// Order-preserving map float -> uint32 (larger float, larger key).  NaN maps
// to the key of -inf: in qw6's scan a NaN never replaces the running best.
__device__ __forceinline__ uint32_t route_key(float v) {
    if (isnan(v)) v = -INFINITY;
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// One warp per token.  Lane l holds logits l, l+32, ..., l+224.  A round
// picks the largest value, lowest index on ties (qw6 starts from element 0 and
// replaces only on a strict '>'), via redux.sync: max over the lanes' local
// best keys, then min over the indices that reach it.  Special cases kept
// from the CPU scan: a NaN at index 0 wins its round; the winner is set to
// -inf, not removed, so when all remaining values are -inf index 0 is chosen
// (again).  Softmax over the selected logits as qw6 does: max-subtract, expf,
// sum in selection order, divide.
__device__ __forceinline__ void route_token(const float* lg, int ne, int k, int32_t* idx, float* w, int lane) {
    float v[8];
    uint32_t key[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = lane + 32 * i;
        v[i] = e < ne ? lg[e] : -INFINITY;
        key[i] = route_key(v[i]);
    }
    const uint32_t kNegInf = 0x007fffffu;  // route_key(-inf)
    float sel_v = 0.f;  // lane r keeps round r's value and index
    int sel_i = 0;
    bool nan0 = __shfl_sync(0xffffffffu, isnan(v[0]) ? 1 : 0, 0) != 0;  // logit 0 is NaN (until selected)
    for (int r = 0; r < k; r++) {
        uint32_t bk = 0;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = lane + 32 * i;
            if (e < ne && (key[i] > bk || bi == 0x7fffffff)) {
                bk = key[i];
                bi = e;
            }
        }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bi == 0x7fffffff ? 0u : bk);
        int win = (int)__reduce_min_sync(0xffffffffu, (bi != 0x7fffffff && bk == mk) ? (uint32_t)bi : 0xffffffffu);
        if (nan0) win = 0;
        const int owner = win & 31, slot = win >> 5;
        float mine = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i == slot) mine = v[i];
        const float orig = __shfl_sync(0xffffffffu, mine, owner);
        if (lane == owner) {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (i == slot) {
                    v[i] = -INFINITY;
                    key[i] = kNegInf;
                }
        }
        if (win == 0) nan0 = false;
        if (lane == (r & 31)) {
            sel_v = orig;
            sel_i = win;
        }
    }
    // softmax over the k selected values as qw6 computes it: the max by a
    // strict '>' scan in selection order, expf(v - max), the sum in selection
    // order, then each weight divided by the sum
    float mx = __shfl_sync(0xffffffffu, sel_v, 0);
    for (int r = 1; r < k; r++) {
        const float t = __shfl_sync(0xffffffffu, sel_v, r);
        if (t > mx) mx = t;
    }
    const float ex = expf(__fsub_rn(sel_v, mx));
    float sum = 0.f;
    for (int r = 0; r < k; r++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, r));
    if (lane < k) {
        idx[lane] = sel_i;
        w[lane] = __fdiv_rn(ex, sum);
    }
}

}  // namespace qw6
