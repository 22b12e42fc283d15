// k_prefill.cu -- routed MoE FFN for prefill-sized batches on the tcgen05
// tensor cores (config 3: 4096 tokens, 256 experts, top-8).
//
// Composition as qw6_apply_layer_moe (qw6.c:2246-2264) per token, computed as
// grouped GEMMs over the tokens routed to each expert:
//   plan   route (qw6.c:2796-2827), count per expert, offsets, scatter the
//          (token, slot) assignments into expert order; work item = one
//          expert x up to 256 of its assignments;
//   gemm1  per (item, 128-row feature tile): A = gate and up rows of the
//          expert, dequantized from the packed Q4_K tiles to bf16 straight
//          into the 128B-swizzled shared layout; B = the item's token rows of
//          X (bf16, gathered); two TMEM accumulators (D^T: features x tokens);
//          epilogue H[assignment][feature] = bf16(silu(g) * u);
//   gemm2  per (item, 128-row tile of hidden): A = down rows (Q6_K -> bf16),
//          B = the item's H rows; epilogue out[token] += w * D (fp32 atomics,
//          so the order of the 8 slot contributions is not fixed).
// Numerics: bf16 operands with fp32 accumulation; within 2e-2 of the fp32
// CPU composition (the prefill tolerance).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "qw6_dev.cuh"
#include "qw6_devcfg.cuh"
#include "qw6_launch.h"
#include "qw6_pdl.cuh"
#include "qw6_route.cuh"
#include "qw6_tc.cuh"

namespace qw6 {

constexpr int kPfChunk = 256;  // max tokens of one work item (MMA N)

struct PfArgs {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    size_t gstride, ustride, dstride;
    const float* logits;
    const __nv_bfloat16* x;
    float* out;
    int ntok, hidden, inter, ne, topk;
    int32_t* idx;
    float* w;
    int32_t* pos;
    int32_t* cnt;
    int32_t* off;
    int4* items;
    int* nitems;
    int32_t* order;
    __nv_bfloat16* h;     // [TK][inter]  silu(gate)*up per assignment
    __nv_bfloat16* dout;  // [TK][hidden] expert output per assignment
    const int32_t* slot_row;    // sorted mode: x row of each slot (null: identity)
    int slot_stride;            // element stride of slot_row / slot_dst
    uint8_t* const* out_peers;  // push mode: outputs go to other GPUs (see qw6k_moe_desc)
    size_t out_off;
    const int32_t* slot_dst;
    int out_rows;
    int* err;
};

// ------------------------------------------------------------------ plan --
// Exclusive scans of the per-expert counts and of their 256-token chunks,
// and the work-item list; run by one CTA of 256 threads (ne <= 256).
__device__ __forceinline__ void pf_offsets_cta(const PfArgs& a) {
    __shared__ int wsum[2][8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int own = tid < a.ne ? __ldcg(a.cnt + tid) : 0;
    int v = own, ch = (own + kPfChunk - 1) / kPfChunk;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int pv = __shfl_up_sync(0xffffffffu, v, o), pc = __shfl_up_sync(0xffffffffu, ch, o);
        if (lane >= o) {
            v += pv;
            ch += pc;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = v;
        wsum[1][warp] = ch;
    }
    __syncthreads();
    int bv = 0, bc = 0;
    for (int w2 = 0; w2 < warp; w2++) {
        bv += wsum[0][w2];
        bc += wsum[1][w2];
    }
    const int o0 = bv + v - own, c0 = bc + ch - (own + kPfChunk - 1) / kPfChunk;
    if (tid < a.ne) a.off[tid] = o0;
    if (tid == 255) *a.nitems = bc + ch;
    __syncthreads();
    if (tid < a.ne)
        for (int c = 0; c * kPfChunk < own; c++)
            a.items[c0 + c] = make_int4(tid, o0 + c * kPfChunk, min(kPfChunk, own - c * kPfChunk), 0);
}

// The CTA that finishes last (all counts are in: every CTA fences its
// atomics before it takes a ticket) runs the scans.  a.nitems[1] is the
// ticket counter, zeroed before the launch.
__device__ __forceinline__ void pf_offsets_if_last(const PfArgs& a) {
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(a.nitems + 1, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (last) {
        __threadfence();
        pf_offsets_cta(a);
    }
}

// Route every token (a warp each, qw6.c:2796-2827), count its assignments per
// expert (their positions within the expert: the order of the atomics, which
// the results do not depend on), and, in the last CTA, the offsets.
__global__ void __launch_bounds__(256) k_pf_route_count(const PfArgs a) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t < a.ntok) {
        route_token(a.logits + (size_t)t * a.ne, a.ne, a.topk, a.idx + (size_t)t * a.topk, a.w + (size_t)t * a.topk,
                    lane);
        if (lane < a.topk) {  // the lane reads back the index it wrote
            const int i = t * a.topk + lane;
            a.pos[i] = atomicAdd(&a.cnt[a.idx[i]], 1);
        }
    }
    pf_offsets_if_last(a);
}

// Rows mode (routing given per row): the counts and positions, then the offsets.
__global__ void __launch_bounds__(256) k_pf_count(const PfArgs a) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.ntok * a.topk) a.pos[i] = atomicAdd(&a.cnt[a.idx[i]], 1);
    pf_offsets_if_last(a);
}

// Sorted mode (counts given): the offsets alone.
__global__ void __launch_bounds__(256) k_pf_offsets(const PfArgs a) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    pf_offsets_cta(a);
}

__global__ void k_pf_scatter(const PfArgs a) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.ntok * a.topk) a.order[a.off[a.idx[i]] + a.pos[i]] = i;
}

// ------------------------------------------------------ A-tile producers --
// A lane fills rows (16*mi + g, 16*mi + g + 8) of a 128 x 64 bf16 A tile
// (one K slab) from the packed tile-block; it covers K [8t, 8t+8) of both
// 32-halves of the slab, i.e. swizzle chunks t and 4 + t.  Loading (into
// registers) and dequantizing/storing are split so that the loads of later
// slabs are in flight while slab k is dequantized.
//
// Dequantization works on bf16 pairs.  Two small unsigned values (< 128) are
// placed in the low bytes of the two 16-bit halves of a word with one prmt
// whose second source supplies 0x43 high bytes: 0x43vv is bf16 128 + v
// exactly.  The bias is then removed exactly inside a bf16x2 add or fma:
//   Q4_K scale  bf16(d*sc)   = fma(128 + sc, d_b, -128 d_b)   (one rounding)
//        min    bf16(-dm*m)  = fma(128 + m, -dm_b, 128 dm_b)
//        weight fma(128 + q - 128, scale, min)                 (one rounding)
//   Q6_K weight (128 + q - 160) * bf16(d*sc)                   (one rounding)
// with d_b, dm_b the super-block's fp16 d, dmin rounded to bf16.  A weight
// carries at most three bf16 roundings (relative error < 2^-7.4), inside
// the bf16 prefill tolerance.

constexpr uint32_t kBf16Hi = 0x43434343u;  // prmt source of the 0x43 high bytes
// bytes p0, p1 of w -> halves (0x43 p0, 0x43 p1): bf16 (128 + w.b[p0], 128 + w.b[p1])
template <int P0, int P1>
__device__ __forceinline__ uint32_t bf16_pair(uint32_t w) {
    return prmt(w, kBf16Hi, (uint32_t)(P0 | (4 << 4) | (P1 << 8) | (4 << 12)));
}
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __nv_bfloat162 bf2_of(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }

template <int F>
struct ASlab;  // one lane's quant bytes of one K slab (both row halves)
template <int F>
struct AHdr;   // one lane's per-row header of one super-block (both row halves)

// Q4_K: slab c of a super-block holds sub-blocks 2c (low nibbles of
// qs[32c..32c+32)) and 2c+1 (high nibbles).  The header is unpacked once per
// super-block: 6-bit scales/mins of sub-blocks 0-3 and 4-7 as byte words
// (qw6_get_scale_min_k4, qw6.c:1480-1490) and the bf16 constants.
template <>
struct AHdr<QW6F_Q4_K_M> {
    uint4 h[2];  // raw: d | dmin << 16, words S0, S1, S2
    uint32_t sc_lo[2], sc_hi[2], mn_lo[2], mn_hi[2];
    __nv_bfloat162 d2[2], nd128[2], ndm2[2], dm128[2];
    __device__ __forceinline__ void load(const uint8_t* tb, int lane) {
#pragma unroll
        for (int rh = 0; rh < 2; rh++) h[rh] = ldg128(tb + ((lane >> 2) + 8 * rh) * 16);
    }
    __device__ __forceinline__ void unpack() {
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            const uint32_t S0 = h[rh].y, S1 = h[rh].z, S2 = h[rh].w;
            sc_lo[rh] = S0 & 0x3f3f3f3fu;
            mn_lo[rh] = S1 & 0x3f3f3f3fu;
            sc_hi[rh] = (S2 & 0x0f0f0f0fu) | ((S0 >> 2) & 0x30303030u);
            mn_hi[rh] = ((S2 >> 4) & 0x0f0f0f0fu) | ((S1 >> 2) & 0x30303030u);
            const float d = f16f(h[rh].x), dmin = f16f(h[rh].x >> 16);
            d2[rh] = __float2bfloat162_rn(d);
            nd128[rh] = __float2bfloat162_rn(-128.f * d);
            ndm2[rh] = __float2bfloat162_rn(-dmin);
            dm128[rh] = __float2bfloat162_rn(128.f * dmin);
        }
    }
};
template <>
struct ASlab<QW6F_Q4_K_M> {
    static constexpr bool kPairShared = false;  // every slab has its own bytes
    uint2 q[2];
    template <int C>
    __device__ __forceinline__ void load(const uint8_t* tb, int lane) {
#pragma unroll
        for (int rh = 0; rh < 2; rh++) q[rh] = ldg64(tb + 256 + ((rh * 2 + (C >> 1)) * 32 + lane) * 16 + (C & 1) * 8);
    }
    template <int C>
    __device__ __forceinline__ void store(uint8_t* sa, const AHdr<QW6F_Q4_K_M>& hd, int mi, int lane) const {
        const int g = lane >> 2, t = lane & 3;
        const __nv_bfloat162 m128 = __floats2bfloat162_rn(-128.f, -128.f);
        constexpr int j0 = (2 * C) & 3, j1 = (2 * C + 1) & 3;
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            const uint32_t SC = C < 2 ? hd.sc_lo[rh] : hd.sc_hi[rh], MN = C < 2 ? hd.mn_lo[rh] : hd.mn_hi[rh];
            const __nv_bfloat162 dl = __hfma2(bf2_of(bf16_pair<j0, j0>(SC)), hd.d2[rh], hd.nd128[rh]);
            const __nv_bfloat162 dh = __hfma2(bf2_of(bf16_pair<j1, j1>(SC)), hd.d2[rh], hd.nd128[rh]);
            const __nv_bfloat162 ml = __hfma2(bf2_of(bf16_pair<j0, j0>(MN)), hd.ndm2[rh], hd.dm128[rh]);
            const __nv_bfloat162 mh = __hfma2(bf2_of(bf16_pair<j1, j1>(MN)), hd.ndm2[rh], hd.dm128[rh]);
            uint32_t lo[4], hi[4];
#pragma unroll
            for (int w = 0; w < 2; w++) {
                const uint32_t W = w ? q[rh].y : q[rh].x;
                const uint32_t L = W & 0x0f0f0f0fu, H = (W >> 4) & 0x0f0f0f0fu;
                lo[2 * w] = bf2_bits(__hfma2(__hadd2(bf2_of(bf16_pair<0, 1>(L)), m128), dl, ml));
                lo[2 * w + 1] = bf2_bits(__hfma2(__hadd2(bf2_of(bf16_pair<2, 3>(L)), m128), dl, ml));
                hi[2 * w] = bf2_bits(__hfma2(__hadd2(bf2_of(bf16_pair<0, 1>(H)), m128), dh, mh));
                hi[2 * w + 1] = bf2_bits(__hfma2(__hadd2(bf2_of(bf16_pair<2, 3>(H)), m128), dh, mh));
            }
            const uint32_t row = mi * 16 + g + 8 * rh;
            *reinterpret_cast<uint4*>(sa + sw128_off(row, t)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4*>(sa + sw128_off(row, 4 + t)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
    }
};

// Q6_K: slab c covers half n = c/2, runs kk = 2(c%2) and 2(c%2)+1; scale
// sc[8n + 2kk] (qw6's even-scale reading, qw6.c:1568-1571).  The two scales
// of slab c are bytes 8n + 2k0 and 8n + 2k0 + 2 of the row's 16 scales,
// i.e. bytes 0 and 2 of scale word c.  Scales are signed int8, converted
// exactly through fp32.
template <>
struct AHdr<QW6F_Q6_K> {
    uint4 sc[2];
    uint32_t dd[2];
    float d[2];
    __device__ __forceinline__ void load(const uint8_t* tb, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            sc[rh] = ldg128(tb + (g + 8 * rh) * 16);
            dd[rh] = ldg16(tb + 256 + (g + 8 * rh) * 2);
        }
    }
    __device__ __forceinline__ void unpack() {
#pragma unroll
        for (int rh = 0; rh < 2; rh++) d[rh] = f16f(dd[rh]);
    }
};
template <>
struct ASlab<QW6F_Q6_K> {
    static constexpr bool kPairShared = true;  // slabs 2m and 2m+1 read the same bytes (low/high nibbles)
    uint4 L[2];
    uint2 H[2];
    template <int C>
    __device__ __forceinline__ void load(const uint8_t* tb, int lane) {
        constexpr int n = C >> 1;
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            L[rh] = ldg128(tb + 288 + ((rh * 3 + n) * 32 + lane) * 16);
            H[rh] = ldg64(tb + 288 + ((rh * 3 + 2) * 32 + lane) * 16 + n * 8);
        }
    }
    template <int C>
    __device__ __forceinline__ void store(uint8_t* sa, const AHdr<QW6F_Q6_K>& hd, int mi, int lane) const {
        const int g = lane >> 2, t = lane & 3;
        constexpr int k0 = 2 * (C & 1);
        const __nv_bfloat162 m160 = __floats2bfloat162_rn(-160.f, -160.f);  // -(128 + 32)
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            const uint32_t scw = word_of(hd.sc[rh], C);
            // signed bytes 0 and 2 -> fp32 exactly: (2^23 + 128 + s) - (2^23 + 128)
            const float s0 = __uint_as_float(0x4b000000u | ((scw ^ 0x80u) & 0xffu)) - 8388736.f;
            const float s1 = __uint_as_float(0x4b000000u | (((scw >> 16) ^ 0x80u) & 0xffu)) - 8388736.f;
            const __nv_bfloat162 d0 = __float2bfloat162_rn(hd.d[rh] * s0);
            const __nv_bfloat162 d1 = __float2bfloat162_rn(hd.d[rh] * s1);
            uint32_t v0[4], v1[4];
#pragma unroll
            for (int hw = 0; hw < 2; hw++) {
                const uint32_t A = hw ? L[rh].y : L[rh].x, B = hw ? L[rh].w : L[rh].z, Hh = hw ? H[rh].y : H[rh].x;
                uint32_t q0, q1;
                if (k0 == 0) {
                    q0 = (A & 0x0f0f0f0fu) | ((Hh << 4) & 0x30303030u);
                    q1 = (B & 0x0f0f0f0fu) | ((Hh << 2) & 0x30303030u);
                } else {
                    q0 = ((A >> 4) & 0x0f0f0f0fu) | (Hh & 0x30303030u);
                    q1 = ((B >> 4) & 0x0f0f0f0fu) | ((Hh >> 2) & 0x30303030u);
                }
                v0[2 * hw] = bf2_bits(__hmul2(__hadd2(bf2_of(bf16_pair<0, 1>(q0)), m160), d0));
                v0[2 * hw + 1] = bf2_bits(__hmul2(__hadd2(bf2_of(bf16_pair<2, 3>(q0)), m160), d0));
                v1[2 * hw] = bf2_bits(__hmul2(__hadd2(bf2_of(bf16_pair<0, 1>(q1)), m160), d1));
                v1[2 * hw + 1] = bf2_bits(__hmul2(__hadd2(bf2_of(bf16_pair<2, 3>(q1)), m160), d1));
            }
            const uint32_t row = mi * 16 + g + 8 * rh;
            *reinterpret_cast<uint4*>(sa + sw128_off(row, t)) = make_uint4(v0[0], v0[1], v0[2], v0[3]);
            *reinterpret_cast<uint4*>(sa + sw128_off(row, 4 + t)) = make_uint4(v1[0], v1[1], v1[2], v1[3]);
        }
    }
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

// B rows: producer thread p always copies 16-byte chunk p % 8 of rows
// p / 8 + (NP / 8) k of each slab (NP producers); the source row pointers
// and swizzled destination offsets are computed once per tile.  Rows
// j >= cnt (up to npad) are zero-filled.
template <int NP>
struct BRows {
    static constexpr int R = kPfChunk * 8 / NP;  // rows per thread at npad = kPfChunk
    const __nv_bfloat16* src[R];
    uint32_t dst[R];
    uint32_t bytes[R];
    int n;
    __device__ __forceinline__ void init(const __nv_bfloat16* base, int ld, const int* rowidx, int cnt, int npad,
                                         int ptid) {
        const int cc = ptid & 7;
        n = 0;
#pragma unroll
        for (int k = 0; k < R; k++) {
            const int r = (ptid >> 3) + (NP / 8) * k;
            const bool live = r < cnt;
            // dead rows read nothing (src-size 0) from a valid address of row 0
            src[k] = base + (live ? (size_t)rowidx[r] * ld : 0) + cc * 8;
            dst[k] = sw128_off(r, cc);
            bytes[k] = live ? 16u : 0u;
            if (r < npad) n = k + 1;
        }
    }
    // slab C (0..3) of the current 256-wide K block
    template <int C>
    __device__ __forceinline__ void issue(uint8_t* sb) const {
#pragma unroll
        for (int k = 0; k < R; k++)
            if (k < n) cp_async16(sb + dst[k], src[k] + C * 64, bytes[k]);
    }
    __device__ __forceinline__ void issue_c(uint8_t* sb, int c) const {
        switch (c) {
        case 0: issue<0>(sb); break;
        case 1: issue<1>(sb); break;
        case 2: issue<2>(sb); break;
        default: issue<3>(sb); break;
        }
    }
    __device__ __forceinline__ void next_block() {
#pragma unroll
        for (int k = 0; k < R; k++) src[k] += 256;
    }
};

// arrive on *b once every cp.async this thread issued so far has landed
// (the barrier's expected count includes this arrival)
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// ------------------------------------------------------------- the GEMM --
// MODE 0 (gate/up): A0 = gate rows [128 ft, +128), A1 = up rows, K = hidden,
//   B = X rows of the item's tokens; epilogue H = bf16(silu(D0) * D1).
// MODE 1 (down): A0/A1 = down rows [256 ft, +128) / [256 ft + 128, +128),
//   K = inter, B = H rows of the item's assignments; epilogue writes the
//   per-assignment expert outputs (bf16) for the slot-order combine.
// Warp-specialized over a ring of shared-memory stages, one 64-wide K slab
// each (two 128 x 64 A tiles + npad x 64 B rows).  The ring fills a fixed
// shared-memory budget, so tiles with few tokens get more stages in flight
// (3 at npad 256 ... 5 at npad <= 64):
//   warps 0-15 (producers): wait stage empty; stream the slab's B rows with
//     cp.async (arriving on the stage's full barrier when they land);
//     dequantize A (warp w: 16-row m-tile w%8 of A(w/8)) from registers
//     loaded two slabs earlier into the swizzled stage; arrive on full; load
//     the A fragments of slab ks+2;
//   warp 16 (lane 0): wait full; 8 MMAs (two accumulators x 4 K-steps);
//     commit to the stage's empty barrier; at the end commit to `done`.
// Every wait is time-bounded; on a timeout the error word is set, in-flight
// copies and MMAs are drained and the CTA exits without an epilogue.
constexpr int kPfMaxStages = 6;
constexpr uint32_t kPfStageBudget = 200 * 1024;  // bytes of stages per CTA
constexpr int kPfProducers = 512;
constexpr int kPfThreads = kPfProducers + 32;
constexpr int kPfMmaWarp = kPfProducers / 32;

template <int F, int MODE>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(const PfArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t A_BYTES = 128 * 128;
    constexpr int TB = Fmt<F>::TB;
    __shared__ uint64_t full[kPfMaxStages], empty[kPfMaxStages], done;
    __shared__ uint32_t tmem_base;
    __shared__ int rows[kPfChunk];
    __shared__ __nv_bfloat16* drow[MODE == 1 ? kPfChunk : 1];  // push mode: output row pointers
    pdl_grid_wait();
    const int K = MODE == 0 ? a.hidden : a.inter;
    const int nft = MODE == 0 ? a.inter / 128 : a.hidden / 256;
    const int item = blockIdx.x / nft, ft = blockIdx.x % nft;
    if (item >= *a.nitems) return;
    const int4 it = a.items[item];
    const int e = it.x, off = it.y, cnt = it.z, npad = (cnt + 15) & ~15;
    const uint32_t STAGE = 2 * A_BYTES + (uint32_t)npad * 128;  // multiple of 2 KB: atoms stay 1 KB aligned
    const int S = min(kPfMaxStages, (int)(kPfStageBudget / STAGE));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t* ord = a.order;  // null: the rows are already grouped by expert (sorted mode)
    for (int j = tid; j < cnt; j += blockDim.x) {
        rows[j] = ord ? (MODE == 0 ? ord[off + j] / a.topk : ord[off + j])
                      : (MODE == 0 && a.slot_row ? a.slot_row[(size_t)(off + j) * a.slot_stride] : off + j);
        if (MODE == 1 && a.out_peers) {
            const int sd = a.slot_dst[(size_t)(off + j) * a.slot_stride], src = sd / a.out_rows;
            drow[MODE == 1 ? j : 0] = reinterpret_cast<__nv_bfloat16*>(a.out_peers[src] + a.out_off) +
                                      (size_t)(sd - src * a.out_rows) * a.hidden;
        }
    }
    if (warp == kPfMmaWarp) tmem_alloc(&tmem_base, 512);
    if (tid == 0) {
        for (int i = 0; i < kPfMaxStages; i++) {
            mbar_init(&full[i], 2 * kPfProducers);  // one plain + one cp.async arrival per producer
            mbar_init(&empty[i], 1);
        }
        mbar_init(&done, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    const int nbk = K / 256, nk = K / 64;
    bool ok = true;

    if (warp < kPfMmaWarp) {
        // ---------------------------------------------------- producers --
        const __nv_bfloat16* bsrc = MODE == 0 ? a.x : a.h;
        const int mtx = warp >> 3, mi = warp & 7;
        const uint8_t* wbase;
        int mt0;
        if (MODE == 0) {
            wbase = mtx ? a.up + (size_t)e * a.ustride : a.gate + (size_t)e * a.gstride;
            mt0 = ft * 8;
        } else {
            wbase = a.down + (size_t)e * a.dstride;
            mt0 = (2 * ft + mtx) * 8;
        }
        const uint8_t* tb = wbase + (size_t)(mt0 + mi) * nbk * TB;  // this warp's m-tile, K block 0
        BRows<kPfProducers> br;
        br.init(bsrc, K, rows, cnt, npad, tid);
        // The lane takes the packed data (and rows) of lane 4 g' + t with
        // g' = (g >> 1) | 4 (g & 1): the 8 lanes of each phase of a 16-byte
        // shared store then write rows r and r + 4, whose chunks t ^ (r & 7)
        // never coincide under the 128-byte swizzle (adjacent rows would
        // collide pairwise); the loads stay coalesced.
        const int plane = 4 * (((lane >> 3) & 3) | ((lane & 4) ? 4 : 0)) + (lane & 3);
        // A fragments and headers one K block (four slabs) ahead: buffer c
        // holds slab c of the block being stored, then slab c of the next one
        ASlab<F> rq[4];
        AHdr<F> hc, hn;
        hc.load(tb, plane);
        hc.unpack();
        hn = hc;
        rq[0].template load<0>(tb, plane);
        rq[2].template load<2>(tb, plane);
        if (!ASlab<F>::kPairShared) {
            rq[1].template load<1>(tb, plane);
            rq[3].template load<3>(tb, plane);
        }
        int s = 0;          // stage of slab ks
        uint32_t rnd = 0;   // how many times the ring has wrapped before slab ks
        for (int kb = 0; kb < nbk && ok; kb++) {
            const uint8_t* tbn = tb + TB;
            const bool more = kb + 1 < nbk;
            if (more) hn.load(tbn, plane);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                if (c > 0 && ++s == S) {
                    s = 0;
                    rnd++;
                }
                // stage reuse: wait for the MMAs of this stage's previous round
                if (rnd > 0 && !mbar_wait(&empty[s], (rnd - 1) & 1, a.err, 31 + MODE)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + s * STAGE;
                uint8_t* sa = st + mtx * A_BYTES;
                br.issue_c(st + 2 * A_BYTES, c);
                cp_async_arrive_noinc(&full[s]);
                constexpr bool share = ASlab<F>::kPairShared;
                // c is a compile-time constant after unrolling; with shared pairs
                // slab c reads buffer c & ~1, refilled after its second slab
                switch (c) {
                case 0:
                    rq[0].template store<0>(sa, hc, mi, plane);
                    if (!share && more) rq[0].template load<0>(tbn, plane);
                    break;
                case 1:
                    rq[share ? 0 : 1].template store<1>(sa, hc, mi, plane);
                    if (more) rq[share ? 0 : 1].template load<(share ? 0 : 1)>(tbn, plane);
                    break;
                case 2:
                    rq[2].template store<2>(sa, hc, mi, plane);
                    if (!share && more) rq[2].template load<2>(tbn, plane);
                    break;
                default:
                    rq[share ? 2 : 3].template store<3>(sa, hc, mi, plane);
                    if (more) rq[share ? 2 : 3].template load<(share ? 2 : 3)>(tbn, plane);
                    break;
                }
                fence_async_smem();
                mbar_arrive(&full[s]);
            }
            hc = hn;
            hc.unpack();
            tb = tbn;
            br.next_block();
            if (++s == S) {  // advance to the stage of the next block's slab 0
                s = 0;
                rnd++;
            }
        }
        cp_async_wait_all();
    } else if (lane == 0) {
        // ------------------------------------------------- MMA issuer ----
        const uint32_t idesc = umma_idesc_bf16(128, npad);
        int s = 0;
        uint32_t rnd = 0;
        for (int ks = 0; ks < nk; ks++, s = (s + 1 == S) ? 0 : s + 1, rnd += (s == 0)) {
            if (!mbar_wait(&full[s], rnd & 1, a.err, 35 + MODE)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(smem + s * STAGE), a1 = a0 + A_BYTES, bb = a0 + 2 * A_BYTES;
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) {
                const uint64_t bd = umma_desc_sw128(bb + 32 * k4);
                const uint32_t acc = (ks > 0 || k4 > 0) ? 1u : 0u;
                umma_bf16(tmem, umma_desc_sw128(a0 + 32 * k4), bd, idesc, acc);
                umma_bf16(tmem + 256, umma_desc_sw128(a1 + 32 * k4), bd, idesc, acc);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(&done);  // arrives once every MMA issued above has completed
    }
    // all MMAs drained before TMEM is read or released
    if (warp < kPfMmaWarp || lane == 0) ok = mbar_wait(&done, 0, a.err, 37 + MODE) && ok;
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok && warp < kPfMmaWarp) {
        // Warp w reads TMEM lanes 32 (w % 4) .. +31 (its 32 features of each
        // accumulator) for every (kPfMmaWarp/4)-th group of 16 token columns,
        // stages them token-major in its own 2 KB of the (now idle) stage
        // memory and writes 16-byte pieces of the output rows.
        constexpr int NG = kPfMmaWarp / 4;
        const int wq = warp & 3, wg = warp >> 2;
        const uint32_t lrow = (uint32_t)(wq * 32) << 16;
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(smem + warp * 2048);  // [16 tokens][64]
        for (int c0 = wg * 16; c0 < npad; c0 += 16 * NG) {
            float v0[16], v1[16];
            tmem_ld16(tmem + lrow + (uint32_t)c0, v0);
            tmem_ld16(tmem + lrow + 256u + (uint32_t)c0, v1);
            if (MODE == 0) {
#pragma unroll
                for (int j = 0; j < 16; j++) stg[j * 64 + lane] = __float2bfloat16_rn(silu_fast(v0[j]) * v1[j]);
                __syncwarp();
                // 16 tokens x 64 B: lane writes pieces (token idx/4, quarter idx%4) for idx = lane, lane + 32
#pragma unroll
                for (int it = 0; it < 2; it++) {
                    const int idx = it * 32 + lane, j = idx >> 2, q = idx & 3;
                    if (c0 + j < cnt) {
                        const uint4 v = *reinterpret_cast<const uint4*>(stg + j * 64 + q * 8);
                        __nv_bfloat16* o = a.h + (size_t)(ord ? ord[off + c0 + j] : off + c0 + j) * a.inter +
                                           ft * 128 + wq * 32 + q * 8;
                        *reinterpret_cast<uint4*>(o) = v;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    stg[j * 64 + lane] = __float2bfloat16_rn(v0[j]);
                    stg[j * 64 + 32 + lane] = __float2bfloat16_rn(v1[j]);
                }
                __syncwarp();
                // 16 tokens x 2 halves x 64 B: piece (token, half, quarter) per idx
#pragma unroll
                for (int it = 0; it < 4; it++) {
                    const int idx = it * 32 + lane, j = idx >> 3, h = (idx >> 2) & 1, q = idx & 3;
                    if (c0 + j < cnt) {
                        const uint4 v = *reinterpret_cast<const uint4*>(stg + j * 64 + h * 32 + q * 8);
                        __nv_bfloat16* o = (a.out_peers ? drow[MODE == 1 ? c0 + j : 0]
                                                        : a.dout + (size_t)rows[c0 + j] * a.hidden) +
                                           2 * ft * 128 + h * 128 + wq * 32 + q * 8;
                        *reinterpret_cast<uint4*>(o) = v;
                    }
                }
            }
            __syncwarp();
        }
    }
    // Pushed rows need no fence here: kernel completion flushes this grid's
    // writes at system scope, and the next kernel on the stream publishes the
    // layer's signal with a system-scope fence + release store.
    tc_fence_before();
    __syncthreads();
    if (warp == kPfMmaWarp) tmem_dealloc(tmem, 512);
}

// out[t][f] = sum_k w[t,k] * dout[t*topk + k][f], fp32 in slot order k
// (rows mode: out[r] = w[r] * dout[r]).  A thread takes 8 features of one
// token: one 16-byte load per slot, all slots' loads issued before the sums.
__device__ __forceinline__ void acc_bf16x8(float (&o)[8], float w, const uint4& v) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        o[2 * i] = fmaf(w, __uint_as_float(u[i] << 16), o[2 * i]);
        o[2 * i + 1] = fmaf(w, __uint_as_float(u[i] & 0xffff0000u), o[2 * i + 1]);
    }
}

__global__ void k_pf_combine(const PfArgs a) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int t = blockIdx.y, f = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (f >= a.hidden) return;
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const size_t s0 = (size_t)t * a.topk;
    if (a.topk == 8) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = *reinterpret_cast<const uint4*>(a.dout + (s0 + k) * a.hidden + f);
#pragma unroll
        for (int k = 0; k < 8; k++) acc_bf16x8(o, a.w[s0 + k], v[k]);
    } else {
        for (int k = 0; k < a.topk; k++)
            acc_bf16x8(o, a.w[s0 + k], *reinterpret_cast<const uint4*>(a.dout + (s0 + k) * a.hidden + f));
    }
    float4* op = reinterpret_cast<float4*>(a.out + (size_t)t * a.hidden + f);
    op[0] = make_float4(o[0], o[1], o[2], o[3]);
    op[1] = make_float4(o[4], o[5], o[6], o[7]);
}

}  // namespace qw6

using namespace qw6;

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static int pf_items_max(uint32_t tk, uint32_t ne) { return (int)((tk < ne ? tk : ne) + tk / kPfChunk + 1); }

extern "C" size_t qw6k_moe_prefill_ws_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t ne,
                                           uint32_t topk) {
    const size_t tk = (size_t)ntok * topk;
    return al256(tk * 4) * 4 + al256(256 * 4) * 2 + al256((size_t)pf_items_max((uint32_t)tk, ne) * 16) + 256 +
           al256(tk * inter * 2) + al256(tk * hidden * 2);
}

static int pf_args(const qw6k_moe_desc* d, int* err, PfArgs& a) {
    const bool rows_mode = d && !d->logits;
    const bool sorted = rows_mode && d->expert_counts;
    const bool push = sorted && d->out_peers;
    if (rows_mode && (d->topk != 1 || (!d->row_expert && !sorted) || (!d->dout && !push))) return QW6K_ERR_ARG;
    if (push && (!d->slot_dst || !d->out_rows)) return QW6K_ERR_ARG;
    if (!d || !d->gate || !d->up || !d->down || !d->x || (!d->out && !rows_mode) || !d->ws || !err || !d->ntok ||
        !d->ne || d->ne > 256 || !d->topk || d->topk > 32 || d->topk > d->ne || (size_t)d->ntok * d->topk > (1u << 22))
        return QW6K_ERR_ARG;
    if (d->hidden % 256 || d->inter % 128 || d->inter % 256 || !d->hidden || !d->inter || d->hidden > 16384 ||
        d->inter > 16384)
        return QW6K_ERR_ARG;
    if (d->gq != QW6F_Q4_K_M && d->gq != QW6F_Q4_K_S && d->gq != QW6F_Q6_K) return QW6K_ERR_QUANT;
    if (d->dq != QW6F_Q4_K_M && d->dq != QW6F_Q4_K_S && d->dq != QW6F_Q6_K) return QW6K_ERR_QUANT;
    if (d->ws_bytes < qw6k_moe_prefill_ws_bytes(d->ntok, d->hidden, d->inter, d->ne, d->topk)) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(d->x) | reinterpret_cast<uintptr_t>(d->out) |
         reinterpret_cast<uintptr_t>(d->gate) | reinterpret_cast<uintptr_t>(d->up) |
         reinterpret_cast<uintptr_t>(d->down) | d->gstride | d->ustride | d->dstride) & 15u)
        return QW6K_ERR_ALIGN;
    a.gate = (const uint8_t*)d->gate;
    a.up = (const uint8_t*)d->up;
    a.down = (const uint8_t*)d->down;
    a.gstride = d->gstride;
    a.ustride = d->ustride;
    a.dstride = d->dstride;
    a.logits = d->logits;
    a.x = (const __nv_bfloat16*)d->x;
    a.out = d->out;
    a.ntok = (int)d->ntok;
    a.hidden = (int)d->hidden;
    a.inter = (int)d->inter;
    a.ne = (int)d->ne;
    a.topk = (int)d->topk;
    a.err = err;
    const size_t tk = (size_t)d->ntok * d->topk;
    uint8_t* p = (uint8_t*)d->ws;
    a.idx = (int32_t*)p; p += al256(tk * 4);
    a.w = (float*)p; p += al256(tk * 4);
    a.pos = (int32_t*)p; p += al256(tk * 4);
    a.order = (int32_t*)p; p += al256(tk * 4);
    a.cnt = (int32_t*)p; p += al256(256 * 4);
    a.off = (int32_t*)p; p += al256(256 * 4);
    a.items = (int4*)p; p += al256((size_t)pf_items_max((uint32_t)tk, d->ne) * 16);
    a.nitems = (int*)p; p += 256;
    a.h = (__nv_bfloat16*)p; p += al256(tk * d->inter * 2);
    a.dout = (__nv_bfloat16*)p;
    a.slot_row = sorted ? d->slot_row : nullptr;
    a.slot_stride = d->slot_stride > 1 ? (int)d->slot_stride : 1;
    a.out_peers = nullptr;
    a.out_off = 0;
    a.slot_dst = nullptr;
    a.out_rows = 0;
    if (rows_mode) {  // caller-supplied routing; expert outputs into the caller's buffer
        if (reinterpret_cast<uintptr_t>(d->dout) & 15u) return QW6K_ERR_ALIGN;
        a.idx = const_cast<int32_t*>(d->row_expert);
        a.dout = (__nv_bfloat16*)d->dout;
    }
    if (push) {
        if (d->out_off & 15u) return QW6K_ERR_ALIGN;
        a.out_peers = d->out_peers;
        a.out_off = d->out_off;
        a.slot_dst = d->slot_dst;
        a.out_rows = (int)d->out_rows;
    }
    if (sorted) {  // rows grouped by expert in expert order, expert_counts[e] rows each
        a.cnt = const_cast<int32_t*>(d->expert_counts);
        a.order = nullptr;
    }
    return 0;
}

template <int F, int MODE>
static int launch_pf(const PfArgs& a, int mi, cudaStream_t st) {
    const size_t smem = (size_t)kPfStageBudget + 1024;
    static DevFlags cfg;
    if (smem_optin(cfg, k_pf_gemm<F, MODE>, (int)smem)) return QW6K_ERR_CUDA;
    const int nft = MODE == 0 ? a.inter / 128 : a.hidden / 256;
    return launch_pdl(k_pf_gemm<F, MODE>, dim3(mi * nft), dim3(kPfThreads), smem, st, a) == cudaSuccess ? 0
                                                                                             : QW6K_ERR_CUDA;
}

extern "C" int qw6k_moe_prefill_check(const qw6k_moe_desc* d, int* err) {
    PfArgs a;
    return pf_args(d, err, a);
}

/* phases: 0 route + count + offsets, 1 count + offsets (rows mode), 2 offsets
 * (sorted mode), 3 scatter,
 * 4 gate/up GEMM (+silu), 5 down GEMM (per-assignment outputs), 6 combine */
extern "C" int qw6k_moe_prefill_phase(const qw6k_moe_desc* d, int* err, int phase, cudaStream_t st) {
    PfArgs a;
    const int rc = pf_args(d, err, a);
    if (rc) return rc;
    const int tk = a.ntok * a.topk;
    const int mi = pf_items_max((uint32_t)tk, (uint32_t)a.ne);
    switch (phase) {
    case 0:  // route + count + offsets
        if (!d->logits) return 0;  // rows mode: routing supplied by the caller
        if (cudaMemsetAsync(a.cnt, 0, 256 * 4, st) != cudaSuccess ||
            cudaMemsetAsync(a.nitems + 1, 0, sizeof(int), st) != cudaSuccess)
            return QW6K_ERR_CUDA;
        if (launch_pdl(k_pf_route_count, dim3((a.ntok + 7) / 8), dim3(256), 0, st, a) != cudaSuccess)
            return QW6K_ERR_CUDA;
        break;
    case 1:  // rows mode: count + offsets
        if (d->logits || !a.order) return 0;  // counted in phase 0, or sorted mode: counts supplied
        if (cudaMemsetAsync(a.cnt, 0, 256 * 4, st) != cudaSuccess ||
            cudaMemsetAsync(a.nitems + 1, 0, sizeof(int), st) != cudaSuccess)
            return QW6K_ERR_CUDA;
        if (launch_pdl(k_pf_count, dim3((tk + 255) / 256), dim3(256), 0, st, a) != cudaSuccess) return QW6K_ERR_CUDA;
        break;
    case 2:  // sorted mode: offsets of the given counts
        if (a.order) return 0;  // done with the counting
        if (launch_pdl(k_pf_offsets, dim3(1), dim3(256), 0, st, a) != cudaSuccess) return QW6K_ERR_CUDA;
        break;
    case 3:
        if (!a.order) return 0;  // sorted mode: already in expert order
        if (launch_pdl(k_pf_scatter, dim3((tk + 255) / 256), dim3(256), 0, st, a) != cudaSuccess) return QW6K_ERR_CUDA;
        break;
    case 4:
        return (d->gq == QW6F_Q6_K) ? launch_pf<QW6F_Q6_K, 0>(a, mi, st) : launch_pf<QW6F_Q4_K_M, 0>(a, mi, st);
    case 5:
        return (d->dq == QW6F_Q6_K) ? launch_pf<QW6F_Q6_K, 1>(a, mi, st) : launch_pf<QW6F_Q4_K_M, 1>(a, mi, st);
    case 6: {
        if (!d->logits) return 0;  // rows mode: the caller combines
        dim3 g((a.hidden / 8 + 255) / 256, a.ntok);
        if (launch_pdl(k_pf_combine, g, dim3(256), 0, st, a) != cudaSuccess) return QW6K_ERR_CUDA;
        break;
    }
    default:
        return QW6K_ERR_ARG;
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
