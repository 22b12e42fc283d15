// k_moe.cu -- routed MoE FFN for decode-sized batches, entirely on device.
//
// Reference composition (qw6_apply_layer_moe, qw6.c:2246-2264):
//   route -> for each selected expert e (selection order):
//   g = Wg[e].x, u = Wu[e].x, mid = silu(g)*u, t = Wd[e].mid, out += w_e*t.
// The Vulkan pipeline runs this as a host readback of the routing plus 5
// synchronous dispatches per expert (qw6_vk.c:3357-3407).  Here there is no
// host round trip and every expert's weights are read once per layer (once
// per work item of <= 4*NQ tokens when an expert has more):
//   ntok <= 4   two launches: self-routed gate/up + silu (k_moe_small_gu),
//               then down with the slot-order combine (k_moe_small_down,
//               programmatic dependent launch: it routes and prefetches its
//               weights while gate/up runs);
//   ntok > 4    four launches: plan (route every token, group the (token,
//               slot) assignments by expert with a counting sort, cut
//               each expert's list into work items), gate/up per item,
//               down per item, slot-order combine (k_moe_plan, k_moe_gateup,
//               k_moe_down, k_moe_combine).
// Weight tile-blocks go straight from HBM into registers (16-byte coalesced
// loads of the packed layout, qw6_dev.cuh) and are multiplied with int8 MMAs.
#include <cuda_runtime.h>

#include "qw6_dev.cuh"
#include "qw6_devcfg.cuh"
#include "qw6_grids.cuh"
#include "qw6_launch.h"
#include "qw6_pdl.cuh"
#include "qw6_route.cuh"

namespace qw6 {

struct MoeArgs {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    size_t gstride, ustride, dstride;  // bytes between experts (packed layout)
    const float* logits;
    const float* x;
    float* out;
    int ntok, hidden, inter, ne, topk, chunk;
    // workspace
    int32_t* idx;
    float* w;
    int32_t* order;
    int4* items;
    int* nitems;
    float* mid;
    float* dout;
};

// ------------------------------------------------------------------ plan --
__global__ void __launch_bounds__(1024) k_moe_plan(const MoeArgs a) {
    __shared__ int cnt[256], off[257], ich[257], fill[256];
    __shared__ int sidx[4096];  // the routed expert of every assignment (ntok * topk <= 4096)
    pdl_wait();  // logits and the workspace are free to use
    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int TK = a.ntok * a.topk;
    for (int t = warp; t < a.ntok; t += nw)
        route_token(a.logits + (size_t)t * a.ne, a.ne, a.topk, a.idx + (size_t)t * a.topk, a.w + (size_t)t * a.topk,
                    lane);
    for (int e = tid; e < 256; e += blockDim.x) cnt[e] = fill[e] = 0;
    __syncthreads();
    for (int i = tid; i < TK; i += blockDim.x) {
        const int e = a.idx[i];
        sidx[i] = e;
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    // exclusive scans of the per-expert counts and chunk counts: each of the
    // first 8 warps scans 32 experts with shuffles, then the warp totals
    __shared__ int wsum[2][8];
    int v = 0, ch = 0;
    if (tid < 256) {
        v = tid < a.ne ? cnt[tid] : 0;
        ch = (v + a.chunk - 1) / a.chunk;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int pv = __shfl_up_sync(0xffffffffu, v, o), pc = __shfl_up_sync(0xffffffffu, ch, o);
            if (lane >= o) { v += pv; ch += pc; }
        }
        if (lane == 31) { wsum[0][warp] = v; wsum[1][warp] = ch; }
    }
    __syncthreads();
    if (tid < 256) {
        int bv = 0, bc = 0;
        for (int w2 = 0; w2 < warp; w2++) { bv += wsum[0][w2]; bc += wsum[1][w2]; }
        const int own = tid < a.ne ? cnt[tid] : 0;
        off[tid] = bv + v - own;                           // exclusive
        ich[tid] = bc + ch - (own + a.chunk - 1) / a.chunk;
        if (tid == 255) { off[256] = bv + v; ich[256] = bc + ch; *a.nitems = bc + ch; }
    }
    __syncthreads();
    // counting sort: an assignment's place among its expert's is the order of
    // the shared-memory atomics.  No value depends on it: every token of an
    // item is staged, multiplied (its own MMA column) and combined on its own.
    for (int i = tid; i < TK; i += blockDim.x) {
        const int e = sidx[i];
        a.order[off[e] + atomicAdd(&fill[e], 1)] = i;
    }
    for (int e = tid; e < a.ne; e += blockDim.x) {
        const int n = cnt[e];
        for (int c = 0; c * a.chunk < n; c++)
            a.items[ich[e] + c] = make_int4(e, off[e] + c * a.chunk, min(a.chunk, n - c * a.chunk), 0);
    }
}

__device__ __forceinline__ float silu_exact(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }

template <int F>
__host__ __device__ constexpr size_t tbl_bytes_of() {
    return IQLut<F>::bytes;
}

// ====================================================== small batches ====
// ntok <= 4: every CTA routes the token(s) itself (no planner launch), lists
// the distinct selected experts in ascending order, and takes expert
// items[blockIdx / mgroups].  All ntok tokens share the 4 MMA columns, so an
// expert chosen by several tokens is read once.  The down kernel is launched
// with programmatic dependent launch: it routes and prefetches its weight
// tiles while the gate/up kernel still runs, then waits for mid.

struct SmallPlan {
    int idx[32];
    float w[32];
    int items[32];      // distinct selected experts, ascending
    int slot_item[32];  // assignment (t*topk + k) -> position in items
    int nitems;
    int rowsel[4];
};

__device__ __forceinline__ void small_plan(SmallPlan* P, const MoeArgs& a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < a.ntok)
        route_token(a.logits + (size_t)warp * a.ne, a.ne, a.topk, P->idx + warp * a.topk, P->w + warp * a.topk,
                    lane);
    __syncthreads();
    if (warp == 0) {
        const int TK = a.ntok * a.topk;
        const int e = lane < TK ? P->idx[lane] : 0x7fffffff;
        bool first = lane < TK;
        for (int j = 0; j < TK; j++)
            if (j < lane && P->idx[j] == e) first = false;
        const unsigned fm = __ballot_sync(0xffffffffu, first);
        int rank = 0;
        for (int j = 0; j < TK; j++)
            if ((fm >> j) & 1u) rank += P->idx[j] < e;
        if (first) P->items[rank] = e;
        if (lane < TK) P->slot_item[lane] = rank;
        if (lane == 0) P->nitems = __popc(fm);
    }
    __syncthreads();
}

template <int F, int NBW>
__device__ __forceinline__ void small_gu_body(const MoeArgs& a) {
    extern __shared__ __align__(16) uint8_t smem[];
    using T = Tile<F, 1>;
    constexpr int TB = T::TB;
    __shared__ SmallPlan P;
    // logits and x come from the previous kernel.  The down kernel routes
    // from the same logits before its own wait, so it may start only once
    // this kernel is past its wait (the logits are then complete).
    pdl_wait();
    pdl_trigger();
    const int nbh = a.hidden / 256, ks = nbh / NBW, mpc = kWarps / ks;
    const int mgroups = (a.inter / 16) / mpc;
    const int item = blockIdx.x / mgroups, mg = blockIdx.x % mgroups;
    small_plan(&P, a);
    if (item >= P.nitems) return;
    const int e = P.items[item];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ms = warp / ks, split = warp % ks, mt = mg * mpc + ms, b0 = split * NBW;
    const uint8_t* gb = a.gate + (size_t)e * a.gstride + ((size_t)mt * nbh + b0) * TB;
    const uint8_t* ub = a.up + (size_t)e * a.ustride + ((size_t)mt * nbh + b0) * TB;
    typename T::Frag g[NBW], u[NBW];
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        T::load(g[i], gb + i * TB, lane);
        T::load(u[i], ub + i * TB, lane);
    }
    if (blockIdx.x == 0 && threadIdx.x < a.ntok * a.topk) {
        a.idx[threadIdx.x] = P.idx[threadIdx.x];
        a.w[threadIdx.x] = P.w[threadIdx.x];
    }
    uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
    XStage xs = xstage_carve(smem + tbl_bytes_of<F>(), 4, a.hidden);
    float* red = reinterpret_cast<float*>(smem + tbl_bytes_of<F>() + xstage_bytes(4, a.hidden));
    if constexpr (IsIQ<F>::value) IQLut<F>::init(tbl, grid_ptr<F>());
    xstage_fill(xs, a.x, a.hidden, a.ntok, 4, a.hidden);
    __syncthreads();
    const XView xv = xs.view();
    float ag[2][1] = {{0.f}, {0.f}}, au[2][1] = {{0.f}, {0.f}};
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        tile_dot<F, 1>(g[i], xv, b0 + i, ag, lane, tbl);
        tile_dot<F, 1>(u[i], xv, b0 + i, au, lane, tbl);
    }
    if (ks > 1) {
        float* r = red + (warp * 32 + lane) * 4;
        r[0] = ag[0][0];
        r[1] = ag[1][0];
        r[2] = au[0][0];
        r[3] = au[1][0];
        __syncthreads();
        if (split == 0) {
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
            for (int p = 0; p < ks; p++) {
                const float* rp = red + ((warp + p) * 32 + lane) * 4;
                s0 += rp[0];
                s1 += rp[1];
                s2 += rp[2];
                s3 += rp[3];
            }
            ag[0][0] = s0;
            ag[1][0] = s1;
            au[0][0] = s2;
            au[1][0] = s3;
        }
    }
    const int g8 = lane >> 2, t = lane & 3;
    if (split == 0 && t < a.ntok) {
        const float m0 = __fmul_rn(silu_exact(ag[0][0]), au[0][0]);
        const float m1 = __fmul_rn(silu_exact(ag[1][0]), au[1][0]);
        for (int k = 0; k < a.topk; k++)
            if (P.idx[t * a.topk + k] == e) {
                float* m = a.mid + (size_t)(t * a.topk + k) * a.inter + mt * 16 + g8;
                m[0] = m0;
                m[8] = m1;
            }
    }
}

// Formats whose gate/up body fits 128 registers with (almost) no spills are
// compiled for two CTAs per SM: a gate/up CTA and a down CTA (<= 128
// registers) then share an SM, so the early-launched down kernel's CTAs
// prefetch their weights beside gate/up instead of waiting for SMs to empty.
template <int F>
struct SmallGuPaired {
    static constexpr bool value = F == QW6F_IQ2_XXS || F == QW6F_Q4_K_M || F == QW6F_Q4_K_S;
};
template <int F, int NBW>
__global__ void __launch_bounds__(kThreads) k_moe_small_gu(const MoeArgs a) {
    small_gu_body<F, NBW>(a);
}
template <int F, int NBW>
__global__ void __launch_bounds__(kThreads, 2) k_moe_small_gu2(const MoeArgs a) {
    small_gu_body<F, NBW>(a);
}
template <int F, int NBW>
constexpr void (*small_gu_kernel())(MoeArgs) {
    if constexpr (SmallGuPaired<F>::value) return k_moe_small_gu2<F, NBW>;
    else return k_moe_small_gu<F, NBW>;
}

// Down projection + routing-weighted combine, one CTA per 16 output rows:
// warp w computes the rows for the selected experts items[w], items[w+8], ...
// (all ntok tokens in the MMA columns), then the CTA sums
// out[t][r] = sum_k w[t,k] * d_{e(t,k)}[t][r] in slot order k, rounded like
// qw6's `out[i] += w[e] * tmp[i]` loop (qw6.c:2263).
template <int F>
__global__ void __launch_bounds__(kThreads) k_moe_small_down(const MoeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    using T = Tile<F, 1>;
    constexpr int TB = T::TB;
    __shared__ SmallPlan P;
    __shared__ int rs[32][4];
    __shared__ float dres[32][4][16];
    pdl_trigger();
    small_plan(&P, a);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, nbi = a.inter / 256, ni = P.nitems, TK = a.ntok * a.topk;
    auto tptr = [&](int it, int b) {
        return a.down + (size_t)P.items[it] * a.dstride + ((size_t)mt * nbi + b) * TB;
    };
    typename T::Frag fa, fb;
    if (warp < ni) {  // prefetch while the gate/up kernel may still be running
        T::load(fa, tptr(warp, 0), lane);
        if (nbi > 1) T::load(fb, tptr(warp, 1), lane);
    }
    for (int i = threadIdx.x; i < ni * 4; i += blockDim.x) {
        const int it = i >> 2, t = i & 3;
        int r = -1;
        if (t < a.ntok)
            for (int k = a.topk - 1; k >= 0; k--)
                if (P.idx[t * a.topk + k] == P.items[it]) r = t * a.topk + k;
        rs[it][t] = r;
    }
    uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
    uint8_t* stage0 = smem + tbl_bytes_of<F>();
    const size_t sb = xstage_bytes(4, a.inter);
    if constexpr (IsIQ<F>::value) IQLut<F>::init(tbl, grid_ptr<F>());
    __syncthreads();
    pdl_wait();  // mid from the gate/up kernel is complete and visible
    for (int it = warp; it < ni; it += kWarps) {
        if (it != warp) {
            T::load(fa, tptr(it, 0), lane);
            if (nbi > 1) T::load(fb, tptr(it, 1), lane);
        }
        // this warp stages (quantizes) only its own expert's mid rows
        const XStage st = xstage_carve(stage0 + it * sb, 4, a.inter);
        xstage_fill_warps(st, a.mid, a.inter, a.ntok, 4, a.inter, rs[it], 1, 0, 1);
        __syncwarp();
        const XView xv = st.view();
        float acc[2][1] = {{0.f}, {0.f}};
        for (int b = 0; b < nbi; b += 2) {
            tile_dot<F, 1>(fa, xv, b, acc, lane, tbl);
            if (b + 2 < nbi) T::load(fa, tptr(it, b + 2), lane);
            if (b + 1 < nbi) {
                tile_dot<F, 1>(fb, xv, b + 1, acc, lane, tbl);
                if (b + 3 < nbi) T::load(fb, tptr(it, b + 3), lane);
            }
        }
        const int g8 = lane >> 2, t = lane & 3;
        dres[it][t][g8] = acc[0][0];
        dres[it][t][g8 + 8] = acc[1][0];
    }
    __syncthreads();
    if ((int)threadIdx.x < a.ntok * 16) {
        const int t = threadIdx.x >> 4, r = threadIdx.x & 15;
        float o = 0.f;
        for (int k = 0; k < a.topk; k++) {
            const int s = t * a.topk + k;
            o = __fadd_rn(o, __fmul_rn(P.w[s], dres[P.slot_item[s]][t][r]));
        }
        a.out[(size_t)t * a.hidden + mt * 16 + r] = o;
    }
    (void)TK;
}

// ==================================================== planned batches ====
// ntok > 4: the planner grouped the assignments by expert into work items
// (expert, <= 4*NQ of its assignments); gate/up runs per (item, 16-row tile)
// with one warp per K block (gate and up tile-blocks loaded straight into
// registers), down per (item, 8/ks 16-row tiles of hidden) with ks warps per
// tile (two K blocks each), and k_moe_combine sums the slots in order.
template <int F, int NQ, int NBW>
__global__ void __launch_bounds__(kThreads) k_moe_gateup(const MoeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    using T = Tile<F, NQ>;
    constexpr int TB = T::TB;
    const int ks = a.hidden / 256 / NBW, mpc = kWarps / ks;
    const int mgroups = (a.inter / 16) / mpc;
    const int item = blockIdx.x / mgroups, mg = blockIdx.x % mgroups;
    if (item >= *a.nitems) return;
    const int4 it = a.items[item];
    const int e = it.x, cnt = it.z;
    const int32_t* sel = a.order + it.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ms = warp / ks, split = warp % ks, mt = mg * mpc + ms, nbh = a.hidden / 256, b0 = split * NBW;

    const uint8_t* gb = a.gate + (size_t)e * a.gstride + ((size_t)mt * nbh + b0) * TB;
    const uint8_t* ub = a.up + (size_t)e * a.ustride + ((size_t)mt * nbh + b0) * TB;
    typename T::Frag g[NBW], u[NBW];
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        T::load(g[i], gb + i * TB, lane);
        T::load(u[i], ub + i * TB, lane);
    }

    uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
    XStage xs = xstage_carve(smem + tbl_bytes_of<F>(), 4 * NQ, a.hidden);
    float* red = reinterpret_cast<float*>(smem + tbl_bytes_of<F>() + xstage_bytes(4 * NQ, a.hidden));
    if constexpr (IsIQ<F>::value) IQLut<F>::init(tbl, grid_ptr<F>());
    xstage_fill(xs, a.x, a.hidden, cnt, 4 * NQ, a.hidden, sel, a.topk);
    __syncthreads();
    const XView xv = xs.view();

    float ag[2][NQ], au[2][NQ];
#pragma unroll
    for (int q = 0; q < NQ; q++) ag[0][q] = ag[1][q] = au[0][q] = au[1][q] = 0.f;
#pragma unroll
    for (int i = 0; i < NBW; i++) {
        tile_dot<F, NQ>(g[i], xv, b0 + i, ag, lane, tbl);
        tile_dot<F, NQ>(u[i], xv, b0 + i, au, lane, tbl);
    }

    if (ks > 1) {
        float* r = red + (warp * 32 + lane) * 4 * NQ;
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            r[4 * q + 0] = ag[0][q];
            r[4 * q + 1] = ag[1][q];
            r[4 * q + 2] = au[0][q];
            r[4 * q + 3] = au[1][q];
        }
        __syncthreads();
        if (split == 0) {
#pragma unroll
            for (int q = 0; q < NQ; q++) {
                float s[4] = {0.f, 0.f, 0.f, 0.f};
                for (int p = 0; p < ks; p++) {
                    const float* rp = red + ((warp + p) * 32 + lane) * 4 * NQ + 4 * q;
                    s[0] += rp[0];
                    s[1] += rp[1];
                    s[2] += rp[2];
                    s[3] += rp[3];
                }
                ag[0][q] = s[0];
                ag[1][q] = s[1];
                au[0][q] = s[2];
                au[1][q] = s[3];
            }
        }
    }
    if (split == 0) {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const int j = 4 * q + t;
            if (j < cnt) {
                float* m = a.mid + (size_t)sel[j] * a.inter + mt * 16 + g;
                m[0] = __fmul_rn(silu_exact(ag[0][q]), au[0][q]);
                m[8] = __fmul_rn(silu_exact(ag[1][q]), au[1][q]);
            }
        }
    }
}

// ------------------------------------------------------------------ down --
template <int F, int NQ>
__global__ void __launch_bounds__(kThreads) k_moe_down(const MoeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    using T = Tile<F, NQ>;
    constexpr int TB = T::TB;
    const int ks = a.inter / 512, mpc = kWarps / ks;
    const int mgroups = (a.hidden / 16) / mpc;
    const int item = blockIdx.x / mgroups, mg = blockIdx.x % mgroups;
    if (item >= *a.nitems) return;
    const int4 it = a.items[item];
    const int e = it.x, cnt = it.z;
    const int32_t* sel = a.order + it.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ms = warp / ks, split = warp % ks, mt = mg * mpc + ms, nbi = a.inter / 256, b0 = split * 2;

    const uint8_t* db = a.down + (size_t)e * a.dstride + ((size_t)mt * nbi + b0) * TB;
    typename T::Frag d0, d1;
    T::load(d0, db, lane);
    T::load(d1, db + TB, lane);

    uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
    XStage xs = xstage_carve(smem + tbl_bytes_of<F>(), 4 * NQ, a.inter);
    float* red = reinterpret_cast<float*>(smem + tbl_bytes_of<F>() + xstage_bytes(4 * NQ, a.inter));
    if constexpr (IsIQ<F>::value) IQLut<F>::init(tbl, grid_ptr<F>());
    xstage_fill(xs, a.mid, a.inter, cnt, 4 * NQ, a.inter, sel, 1);
    __syncthreads();
    const XView xv = xs.view();

    float acc[2][NQ];
#pragma unroll
    for (int q = 0; q < NQ; q++) acc[0][q] = acc[1][q] = 0.f;
    tile_dot<F, NQ>(d0, xv, b0, acc, lane, tbl);
    tile_dot<F, NQ>(d1, xv, b0 + 1, acc, lane, tbl);

    if (ks > 1) {
        float* r = red + (warp * 32 + lane) * 2 * NQ;
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            r[2 * q] = acc[0][q];
            r[2 * q + 1] = acc[1][q];
        }
        __syncthreads();
        if (split == 0) {
#pragma unroll
            for (int q = 0; q < NQ; q++) {
                float s0 = 0.f, s1 = 0.f;
                for (int p = 0; p < ks; p++) {
                    s0 += red[((warp + p) * 32 + lane) * 2 * NQ + 2 * q];
                    s1 += red[((warp + p) * 32 + lane) * 2 * NQ + 2 * q + 1];
                }
                acc[0][q] = s0;
                acc[1][q] = s1;
            }
        }
    }
    if (split == 0) {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const int j = 4 * q + t;
            if (j < cnt) {
                float* o = a.dout + (size_t)sel[j] * a.hidden + mt * 16 + g;
                o[0] = acc[0][q];
                o[8] = acc[1][q];
            }
        }
    }
}


// --------------------------------------------------------------- combine --
__global__ void k_moe_combine(const MoeArgs a) {
    pdl_wait();
    const int t = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.hidden) return;
    float acc = 0.f;
    for (int k = 0; k < a.topk; k++) {
        const int s = t * a.topk + k;
        acc = __fadd_rn(acc, __fmul_rn(a.w[s], a.dout[(size_t)s * a.hidden + i]));
    }
    a.out[(size_t)t * a.hidden + i] = acc;
}

// -------------------------------------------------------------- launcher --

#define QW6_MOE_DISPATCH(quant, FN, NQ, ...)                  \
    switch (quant) {                                          \
    case QW6F_Q4_K_M:                                         \
    case QW6F_Q4_K_S: return FN<QW6F_Q4_K_M, NQ>(__VA_ARGS__); \
    case QW6F_Q5_K: return FN<QW6F_Q5_K, NQ>(__VA_ARGS__);     \
    case QW6F_Q6_K: return FN<QW6F_Q6_K, NQ>(__VA_ARGS__);     \
    case QW6F_IQ2_XXS: return FN<QW6F_IQ2_XXS, NQ>(__VA_ARGS__); \
    case QW6F_IQ2_S: return FN<QW6F_IQ2_S, NQ>(__VA_ARGS__);   \
    case QW6F_IQ3_S: return FN<QW6F_IQ3_S, NQ>(__VA_ARGS__);   \
    default: return QW6K_ERR_QUANT;                           \
    }

template <typename Kern>
static int launch_ex(Kern k, int grid, int block, size_t smem, bool pdl, cudaStream_t st, const MoeArgs& a) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, a) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

// K blocks per warp of the small-batch gate/up kernel: two (half the CTAs,
// so the early-launched down kernel's CTAs find room) when there are >= 8.
static int nbw_of(int nb) { return nb >= 8 ? 2 : 1; }

template <int F, int NBW>
static int launch_small_gu(const MoeArgs& a, cudaStream_t st) {
    const size_t smem = tbl_bytes_of<F>() + xstage_bytes(4, a.hidden) + (size_t)kThreads * 4 * 4;
    static DevFlags cfg;
    if (smem_optin(cfg, small_gu_kernel<F, NBW>(), 200 * 1024)) return QW6K_ERR_CUDA;
    const int ks = a.hidden / 256 / NBW, mgroups = (a.inter / 16) / (kWarps / ks);
    return launch_ex(small_gu_kernel<F, NBW>(), a.ntok * a.topk * mgroups, kThreads, smem, true, st, a);
}

template <int F>
static size_t small_down_smem(const MoeArgs& a) {
    return tbl_bytes_of<F>() + (size_t)a.ntok * a.topk * xstage_bytes(4, a.inter);
}

template <int F, int NBW>
static int launch_small_down(const MoeArgs& a, cudaStream_t st) {
    const size_t smem = small_down_smem<F>(a);
    if (smem > 180 * 1024) return QW6K_ERR_ARG;
    static DevFlags cfg;
    if (smem_optin(cfg, k_moe_small_down<F>, 200 * 1024)) return QW6K_ERR_CUDA;
    return launch_ex(k_moe_small_down<F>, a.hidden / 16, kThreads, smem, true, st, a);
}

template <int F, int NQ>
static size_t gu_smem(int hidden) {
    return tbl_bytes_of<F>() + xstage_bytes(4 * NQ, hidden) + (size_t)kThreads * 4 * NQ * 4;
}

template <int F, int NQ>
static int launch_gateup(const MoeArgs& a, int max_items, cudaStream_t st) {
    const size_t smem = gu_smem<F, NQ>(a.hidden);
    if (smem > 200 * 1024) return QW6K_ERR_ARG;
    // one K block of gate and up per warp (two when hidden has more than 8)
    const int nbh = a.hidden / 256, nbw = nbh > kWarps ? 2 : 1;
    static DevFlags cfg1, cfg2;
    if (smem_optin(nbw == 1 ? cfg1 : cfg2, nbw == 1 ? k_moe_gateup<F, NQ, 1> : k_moe_gateup<F, NQ, 2>, 200 * 1024))
        return QW6K_ERR_CUDA;
    const int mgroups = (a.inter / 16) / (kWarps / (nbh / nbw));
    if (nbw == 1) k_moe_gateup<F, NQ, 1><<<max_items * mgroups, kThreads, smem, st>>>(a);
    else k_moe_gateup<F, NQ, 2><<<max_items * mgroups, kThreads, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

template <int F, int NQ>
static int launch_down(const MoeArgs& a, int max_items, cudaStream_t st) {
    const size_t smem = gu_smem<F, NQ>(a.inter);
    if (smem > 200 * 1024) return QW6K_ERR_ARG;
    static DevFlags cfg;
    if (smem_optin(cfg, k_moe_down<F, NQ>, 200 * 1024)) return QW6K_ERR_CUDA;
    const int mgroups = (a.hidden / 16) / (kWarps / (a.inter / 512));
    k_moe_down<F, NQ><<<max_items * mgroups, kThreads, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

static int gateup_any(uint32_t q, int nq, const MoeArgs& a, int mi, cudaStream_t st) {
    if (nq == 1) { QW6_MOE_DISPATCH(q, launch_gateup, 1, a, mi, st) }
    QW6_MOE_DISPATCH(q, launch_gateup, 2, a, mi, st)
}
static int down_any(uint32_t q, int nq, const MoeArgs& a, int mi, cudaStream_t st) {
    if (nq == 1) { QW6_MOE_DISPATCH(q, launch_down, 1, a, mi, st) }
    QW6_MOE_DISPATCH(q, launch_down, 2, a, mi, st)
}

static int small_gu_any(uint32_t q, const MoeArgs& a, cudaStream_t st) {
    if (nbw_of(a.hidden / 256) == 1) { QW6_MOE_DISPATCH(q, launch_small_gu, 1, a, st) }
    QW6_MOE_DISPATCH(q, launch_small_gu, 2, a, st)
}
static int small_down_any(uint32_t q, const MoeArgs& a, cudaStream_t st) {
    QW6_MOE_DISPATCH(q, launch_small_down, 1, a, st)
}

// Set up every kernel of the decode paths on the current device (function
// attributes, which also loads them), so that later calls only launch.
template <int F>
static int dec_setup_one() {
    static DevFlags c1, c2, c3, c4, c5, c6;
    int rc = smem_optin(c1, small_gu_kernel<F, 1>(), 200 * 1024);
    rc |= smem_optin(c2, k_moe_small_down<F>, 200 * 1024);
    static DevFlags c9;
    rc |= smem_optin(c9, small_gu_kernel<F, 2>(), 200 * 1024);
    static DevFlags c7, c8;
    rc |= smem_optin(c3, k_moe_gateup<F, 1, 1>, 200 * 1024);
    rc |= smem_optin(c4, k_moe_gateup<F, 2, 1>, 200 * 1024);
    rc |= smem_optin(c7, k_moe_gateup<F, 1, 2>, 200 * 1024);
    rc |= smem_optin(c8, k_moe_gateup<F, 2, 2>, 200 * 1024);
    rc |= smem_optin(c5, k_moe_down<F, 1>, 200 * 1024);
    rc |= smem_optin(c6, k_moe_down<F, 2>, 200 * 1024);
    cudaFuncAttributes fa;
    rc |= cudaFuncGetAttributes(&fa, k_moe_plan) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
    rc |= cudaFuncGetAttributes(&fa, k_moe_combine) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
    return rc ? QW6K_ERR_CUDA : 0;
}

}  // namespace qw6

using namespace qw6;

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static int moe_items_max(uint32_t ntok, uint32_t ne, uint32_t topk, uint32_t chunk) {
    const uint32_t tk = ntok * topk;
    return (int)((tk < ne ? tk : ne) + tk / chunk + 1);
}

// Assignments per work item of the planned path: 4 (one MMA n-tile) while
// experts average at most 3 assignments (config 2: 512 over 256), else 8.
// An item's tile-blocks are decoded once for all its tokens, so a larger
// chunk shares the (instruction-bound) IQ / K decode among more tokens, but
// costs a second n-tile of MMAs and activation staging for every item,
// mostly empty when experts see ~2 tokens.
static uint32_t moe_chunk(uint32_t ntok, uint32_t ne, uint32_t topk) {
    return (ntok <= 4 || (uint64_t)ntok * topk <= 3ull * ne) ? 4u : 8u;
}

extern "C" size_t qw6k_moe_ws_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t ne, uint32_t topk) {
    const size_t tk = (size_t)ntok * topk;
    const int mi = moe_items_max(ntok, ne, topk, moe_chunk(ntok, ne, topk));
    return al256(tk * 4) * 3 + al256((size_t)mi * 16) + 256 + al256(tk * inter * 4) + al256(tk * hidden * 4);
}

static bool moe_small(const qw6k_moe_desc* d) {
    if (d->ntok > 4 || d->ntok * d->topk > 32) return false;
    const int nbh = (int)d->hidden / 256;
    const int ksh = nbh / nbw_of(nbh);
    if (ksh > 8 || (d->inter / 16) % (kWarps / ksh)) return false;
    const size_t lut = d->dq == QW6F_IQ2_XXS ? IQLut<QW6F_IQ2_XXS>::bytes
                       : d->dq == QW6F_IQ2_S ? IQLut<QW6F_IQ2_S>::bytes
                       : d->dq == QW6F_IQ3_S ? IQLut<QW6F_IQ3_S>::bytes : 0;
    return (size_t)d->ntok * d->topk * xstage_bytes(4, (int)d->inter) + lut <= 180 * 1024;
}

static int moe_args(const qw6k_moe_desc* d, MoeArgs& a) {
    if (!d || !d->gate || !d->up || !d->down || !d->logits || !d->x || !d->out || !d->ws || !d->ntok || !d->ne ||
        d->ne > 256 || !d->topk || d->topk > 32 || d->topk > d->ne || (size_t)d->ntok * d->topk > 4096)
        return QW6K_ERR_ARG;
    const uint32_t nbh = d->hidden / 256, nbi = d->inter / 256;
    if (!nbh || !nbi || d->hidden % 256 || d->inter % 256 || nbh > 16 || nbi > 16 || d->hidden > 4096)
        return QW6K_ERR_ARG;
    if (!moe_small(d) && (d->hidden % 512 || d->inter % 512)) return QW6K_ERR_ARG;  // the planned kernels' K split
    if (d->ws_bytes < qw6k_moe_ws_bytes(d->ntok, d->hidden, d->inter, d->ne, d->topk)) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(d->x) | reinterpret_cast<uintptr_t>(d->gate) |
         reinterpret_cast<uintptr_t>(d->up) | reinterpret_cast<uintptr_t>(d->down) | d->gstride | d->ustride |
         d->dstride) & 15u)
        return QW6K_ERR_ALIGN;
    a.gate = (const uint8_t*)d->gate;
    a.up = (const uint8_t*)d->up;
    a.down = (const uint8_t*)d->down;
    a.gstride = d->gstride;
    a.ustride = d->ustride;
    a.dstride = d->dstride;
    a.logits = d->logits;
    a.x = d->x;
    a.out = d->out;
    a.ntok = (int)d->ntok;
    a.hidden = (int)d->hidden;
    a.inter = (int)d->inter;
    a.ne = (int)d->ne;
    a.topk = (int)d->topk;
    a.chunk = (int)moe_chunk(d->ntok, d->ne, d->topk);
    const size_t tk = (size_t)d->ntok * d->topk;
    const int mi = moe_items_max(d->ntok, d->ne, d->topk, (uint32_t)a.chunk);
    uint8_t* p = (uint8_t*)d->ws;
    a.idx = (int32_t*)p; p += al256(tk * 4);
    a.w = (float*)p; p += al256(tk * 4);
    a.order = (int32_t*)p; p += al256(tk * 4);
    a.items = (int4*)p; p += al256((size_t)mi * 16);
    a.nitems = (int*)p; p += 256;
    a.mid = (float*)p; p += al256(tk * d->inter * 4);
    a.dout = (float*)p;
    return 0;
}


/* Configure (and load) every decode kernel of every format on the current
 * device. */
extern "C" int qw6k_moe_decode_setup(void) {
    int rc = dec_setup_one<QW6F_Q4_K_M>();
    rc |= dec_setup_one<QW6F_Q5_K>();
    rc |= dec_setup_one<QW6F_Q6_K>();
    rc |= dec_setup_one<QW6F_IQ2_XXS>();
    rc |= dec_setup_one<QW6F_IQ2_S>();
    rc |= dec_setup_one<QW6F_IQ3_S>();
    return rc ? QW6K_ERR_CUDA : 0;
}

extern "C" int qw6k_moe_check(const qw6k_moe_desc* d) {
    MoeArgs a;
    return moe_args(d, a);
}

/* Number of launches of one layer and the kind of launch i
 * (0 plan, 1 gate/up, 2 down, 3 combine). */
extern "C" int qw6k_moe_nphases(const qw6k_moe_desc* d) { return moe_small(d) ? 2 : 4; }
extern "C" int qw6k_moe_phase_kind(const qw6k_moe_desc* d, int phase) {
    return moe_small(d) ? phase + 1 : phase;
}

extern "C" int qw6k_moe_phase(const qw6k_moe_desc* d, int phase, cudaStream_t st) {
    MoeArgs a;
    const int rc = moe_args(d, a);
    if (rc) return rc;
    if (moe_small(d)) {
        switch (phase) {
        case 0:
            return small_gu_any(d->gq, a, st);
        case 1:
            return small_down_any(d->dq, a, st);
        default:
            return QW6K_ERR_ARG;
        }
    }
    const int mi = moe_items_max(d->ntok, d->ne, d->topk, (uint32_t)a.chunk);
    const int nq = a.chunk / 4;
    switch (phase) {
    case 0:
        return launch_pdl(k_moe_plan, dim3(1), dim3(1024), 0, st, a) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
    case 1:
        return gateup_any(d->gq, nq, a, mi, st);
    case 2:
        return down_any(d->dq, nq, a, mi, st);
    case 3:
        return launch_pdl(k_moe_combine, dim3((d->hidden + 255) / 256, d->ntok), dim3(256), 0, st, a) == cudaSuccess
                   ? 0
                   : QW6K_ERR_CUDA;
    default:
        return QW6K_ERR_ARG;
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
