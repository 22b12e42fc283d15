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
#include "qw6_launch.h"
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
    __nv_bfloat16* h;
    int* err;
};

// ------------------------------------------------------------------ plan --

__global__ void k_pf_route(const PfArgs a) {
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= a.ntok) return;
    route_token(a.logits + (size_t)t * a.ne, a.ne, a.topk, a.idx + (size_t)t * a.topk, a.w + (size_t)t * a.topk,
                threadIdx.x & 31);
}

__global__ void k_pf_count(const PfArgs a) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.ntok * a.topk) a.pos[i] = atomicAdd(&a.cnt[a.idx[i]], 1);
}

// exclusive scans of counts and of 256-token chunks; the work-item list
__global__ void __launch_bounds__(256) k_pf_offsets(const PfArgs a) {
    __shared__ int wsum[2][8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int own = tid < a.ne ? a.cnt[tid] : 0;
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

__global__ void k_pf_scatter(const PfArgs a) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.ntok * a.topk) a.order[a.off[a.idx[i]] + a.pos[i]] = i;
}

// ------------------------------------------------------ A-tile producers --
// Write rows (16*mi + g, 16*mi + g + 8) of a 128 x 64 bf16 A tile (K slab ks)
// from the packed tile-block `tb`; this lane covers K [8t, 8t+8) of both
// 32-halves of the slab, i.e. swizzle chunks t and 4 + t.

__device__ __forceinline__ uint4 pack8_bf16(const float (&v)[8]) {
    uint4 r;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]), p3 = __floats2bfloat162_rn(v[6], v[7]);
    r.x = *reinterpret_cast<uint32_t*>(&p0);
    r.y = *reinterpret_cast<uint32_t*>(&p1);
    r.z = *reinterpret_cast<uint32_t*>(&p2);
    r.w = *reinterpret_cast<uint32_t*>(&p3);
    return r;
}

// Q4_K: slab c = ks % 4 of block ks / 4 holds sub-blocks 2c (low nibbles of
// qs[32c..32c+32)) and 2c+1 (high nibbles).
__device__ __forceinline__ void produce_q4k(uint8_t* sa, const uint8_t* tb, int c, int mi, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int rh = 0; rh < 2; rh++) {
        const uint2 q = ldg64(tb + 256 + ((rh * 2 + (c >> 1)) * 32 + lane) * 16 + (c & 1) * 8);
        const uint4 h = ldg128(tb + (g + 8 * rh) * 16);
        const float d = f16f(h.x), dmin = f16f(h.x >> 16);
        const uint32_t S0 = h.y, S1 = h.z, S2 = h.w;
        const uint32_t SC0 = S0 & 0x3f3f3f3fu, MN0 = S1 & 0x3f3f3f3fu;
        const uint32_t SC1 = (S2 & 0x0f0f0f0fu) | ((S0 >> 2) & 0x30303030u);
        const uint32_t MN1 = ((S2 >> 4) & 0x0f0f0f0fu) | ((S1 >> 2) & 0x30303030u);
        const int j0 = 2 * c, j1 = 2 * c + 1;
        const float dl = d * (float)byte_of(j0 < 4 ? SC0 : SC1, j0 & 3);
        const float ml = dmin * (float)byte_of(j0 < 4 ? MN0 : MN1, j0 & 3);
        const float dh = d * (float)byte_of(j1 < 4 ? SC0 : SC1, j1 & 3);
        const float mh = dmin * (float)byte_of(j1 < 4 ? MN0 : MN1, j1 & 3);
        float lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t b = byte_of(i < 4 ? q.x : q.y, i & 3);
            lo[i] = fmaf(dl, (float)(b & 15u), -ml);
            hi[i] = fmaf(dh, (float)(b >> 4), -mh);
        }
        const uint32_t row = mi * 16 + g + 8 * rh;
        *reinterpret_cast<uint4*>(sa + sw128_off(row, t)) = pack8_bf16(lo);
        *reinterpret_cast<uint4*>(sa + sw128_off(row, 4 + t)) = pack8_bf16(hi);
    }
}

// Q6_K: slab c = ks % 4 covers half n = c/2, runs kk = 2(c%2) and 2(c%2)+1;
// scale sc[8n + 2kk] (qw6's even-scale reading, qw6.c:1568-1571).
__device__ __forceinline__ void produce_q6k(uint8_t* sa, const uint8_t* tb, int c, int mi, int lane) {
    const int g = lane >> 2, t = lane & 3, n = c >> 1, k0 = 2 * (c & 1);
#pragma unroll
    for (int rh = 0; rh < 2; rh++) {
        const uint4 L = ldg128(tb + 288 + ((rh * 3 + n) * 32 + lane) * 16);
        const uint2 H = ldg64(tb + 288 + ((rh * 3 + 2) * 32 + lane) * 16 + n * 8);
        const uint4 sc = ldg128(tb + (g + 8 * rh) * 16);
        const float d = f16f(ldg16(tb + 256 + (g + 8 * rh) * 2));
        const float d0 = d * (float)(int8_t)byte16(sc, 8 * n + 2 * k0);
        const float d1 = d * (float)(int8_t)byte16(sc, 8 * n + 2 * (k0 + 1));
        float v0[8], v1[8];
#pragma unroll
        for (int hw = 0; hw < 2; hw++) {
            const uint32_t A = hw ? L.y : L.x, B = hw ? L.w : L.z, Hh = hw ? H.y : H.x;
            uint32_t q0, q1;
            if (k0 == 0) {
                q0 = (A & 0x0f0f0f0fu) | ((Hh << 4) & 0x30303030u);
                q1 = (B & 0x0f0f0f0fu) | ((Hh << 2) & 0x30303030u);
            } else {
                q0 = ((A >> 4) & 0x0f0f0f0fu) | (Hh & 0x30303030u);
                q1 = ((B >> 4) & 0x0f0f0f0fu) | ((Hh >> 2) & 0x30303030u);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v0[4 * hw + i] = d0 * (float)((int)byte_of(q0, i) - 32);
                v1[4 * hw + i] = d1 * (float)((int)byte_of(q1, i) - 32);
            }
        }
        const uint32_t row = mi * 16 + g + 8 * rh;
        *reinterpret_cast<uint4*>(sa + sw128_off(row, t)) = pack8_bf16(v0);
        *reinterpret_cast<uint4*>(sa + sw128_off(row, 4 + t)) = pack8_bf16(v1);
    }
}

template <int F>
__device__ __forceinline__ void produce_a(uint8_t* sa, const uint8_t* tb, int c, int mi, int lane) {
    if constexpr (F == QW6F_Q6_K)
        produce_q6k(sa, tb, c, mi, lane);
    else
        produce_q4k(sa, tb, c, mi, lane);
}

// B rows: bf16 row j of the item from src + rowidx[j] * ld (K slab ks);
// rows >= cnt are zero (up to npad).
__device__ __forceinline__ void produce_b(uint8_t* sb, const __nv_bfloat16* src, int ld, const int* rowidx, int cnt,
                                          int npad, int ks) {
    for (int i = threadIdx.x; i < npad * 8; i += blockDim.x) {
        const int r = i >> 3, cc = i & 7;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < cnt) v = *reinterpret_cast<const uint4*>(src + (size_t)rowidx[r] * ld + ks * 64 + cc * 8);
        *reinterpret_cast<uint4*>(sb + sw128_off(r, cc)) = v;
    }
}

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// ----------------------------------------------------------------- gemm1 --
template <int GQ>
__global__ void __launch_bounds__(256, 1) k_pf_gemm1(const PfArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = kPfChunk * 128, STAGE = 2 * A_BYTES + B_BYTES;
    constexpr int TB = Fmt<GQ>::TB;
    __shared__ uint64_t mbar[2];
    __shared__ uint32_t tmem_base;
    __shared__ int ncommit[2];
    __shared__ int rowtok[kPfChunk];
    const int ftiles = a.inter / 128;
    const int item = blockIdx.x / ftiles, ft = blockIdx.x % ftiles;
    if (item >= *a.nitems) return;
    const int4 it = a.items[item];
    const int e = it.x, off = it.y, cnt = it.z, npad = (cnt + 15) & ~15;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int j = tid; j < cnt; j += blockDim.x) rowtok[j] = a.order[off + j] / a.topk;
    if (warp == 0) tmem_alloc(&tmem_base, 512);
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
    const uint32_t idesc = umma_idesc_bf16(128, npad);
    const int nbh = a.hidden / 256, nk = a.hidden / 64;
    // producer unit of this warp: matrix (gate/up) and two 16-row m-tiles
    const int mtx = warp >> 2, mi0 = 2 * (warp & 3);
    const uint8_t* wbase = (mtx ? a.up + (size_t)e * a.ustride : a.gate + (size_t)e * a.gstride);
    bool ok = true;
    for (int ks = 0; ks < nk && ok; ks++) {
        const int s = ks & 1;
        if (ks >= 2) ok = mbar_wait(&mbar[s], ((ks - 2) >> 1) & 1, a.err, 11);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        uint8_t* sa = smem + s * STAGE;
        const int b = ks >> 2, c = ks & 3;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int mi = mi0 + u;
            produce_a<GQ>(sa + mtx * A_BYTES, wbase + ((size_t)(ft * 8 + mi) * nbh + b) * TB, c, mi, lane);
        }
        produce_b(sa + 2 * A_BYTES, a.x, a.hidden, rowtok, cnt, npad, ks);
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t ag = smem_u32(sa), au = ag + A_BYTES, bb = ag + 2 * A_BYTES;
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++) {
                const uint64_t bd = umma_desc_sw128(bb + 32 * k4);
                const uint32_t acc = (ks > 0 || k4 > 0) ? 1u : 0u;
                umma_bf16(tmem, umma_desc_sw128(ag + 32 * k4), bd, idesc, acc);
                umma_bf16(tmem + 256, umma_desc_sw128(au + 32 * k4), bd, idesc, acc);
            }
            umma_commit(&mbar[s]);
            ncommit[s]++;
        }
    }
    if (ok) ok = mbar_wait(&mbar[(nk - 1) & 1], ((nk - 1) >> 1) & 1, a.err, 12);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        const int wq = warp & 3, wg = warp >> 2, f = ft * 128 + wq * 32 + lane;
        const uint32_t lrow = (uint32_t)(wq * 32) << 16;
        for (int c0 = wg * 16; c0 < npad; c0 += 32) {
            float gv[16], uv[16];
            tmem_ld16(tmem + lrow + (uint32_t)c0, gv);
            tmem_ld16(tmem + lrow + 256u + (uint32_t)c0, uv);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int r = c0 + j;
                if (r < cnt)
                    a.h[(size_t)a.order[off + r] * a.inter + f] = __float2bfloat16_rn(silu_fast(gv[j]) * uv[j]);
            }
        }
    } else {
        __syncthreads();
        for (int s = 0; s < 2; s++)
            if (ncommit[s] > 0) mbar_wait(&mbar[s], (ncommit[s] - 1) & 1, nullptr, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

// ----------------------------------------------------------------- gemm2 --
template <int DQ>
__global__ void __launch_bounds__(256, 2) k_pf_gemm2(const PfArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t A_BYTES = 128 * 128, B_BYTES = kPfChunk * 128, STAGE = A_BYTES + B_BYTES;
    constexpr int TB = Fmt<DQ>::TB;
    __shared__ uint64_t mbar[2];
    __shared__ uint32_t tmem_base;
    __shared__ int ncommit[2];
    __shared__ int rowa[kPfChunk];
    const int ftiles = a.hidden / 128;
    const int item = blockIdx.x / ftiles, ft = blockIdx.x % ftiles;
    if (item >= *a.nitems) return;
    const int4 it = a.items[item];
    const int e = it.x, off = it.y, cnt = it.z, npad = (cnt + 15) & ~15;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int j = tid; j < cnt; j += blockDim.x) rowa[j] = a.order[off + j];
    if (warp == 0) tmem_alloc(&tmem_base, 256);
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
    const uint32_t idesc = umma_idesc_bf16(128, npad);
    const int nbi = a.inter / 256, nk = a.inter / 64;
    const uint8_t* wbase = a.down + (size_t)e * a.dstride;
    bool ok = true;
    for (int ks = 0; ks < nk && ok; ks++) {
        const int s = ks & 1;
        if (ks >= 2) ok = mbar_wait(&mbar[s], ((ks - 2) >> 1) & 1, a.err, 21);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        uint8_t* sa = smem + s * STAGE;
        const int b = ks >> 2, c = ks & 3, mi = warp;
        produce_a<DQ>(sa, wbase + ((size_t)(ft * 8 + mi) * nbi + b) * TB, c, mi, lane);
        produce_b(sa + A_BYTES, a.h, a.inter, rowa, cnt, npad, ks);
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t aa = smem_u32(sa), bb = aa + A_BYTES;
#pragma unroll
            for (int k4 = 0; k4 < 4; k4++)
                umma_bf16(tmem, umma_desc_sw128(aa + 32 * k4), umma_desc_sw128(bb + 32 * k4), idesc,
                          (ks > 0 || k4 > 0) ? 1u : 0u);
            umma_commit(&mbar[s]);
            ncommit[s]++;
        }
    }
    if (ok) ok = mbar_wait(&mbar[(nk - 1) & 1], ((nk - 1) >> 1) & 1, a.err, 22);
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (ok) {
        const int wq = warp & 3, wg = warp >> 2, f = ft * 128 + wq * 32 + lane;
        const uint32_t lrow = (uint32_t)(wq * 32) << 16;
        for (int c0 = wg * 16; c0 < npad; c0 += 32) {
            float v[16];
            tmem_ld16(tmem + lrow + (uint32_t)c0, v);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int r = c0 + j;
                if (r < cnt) {
                    const int as = rowa[r];
                    atomicAdd(a.out + (size_t)(as / a.topk) * a.hidden + f, a.w[as] * v[j]);
                }
            }
        }
    } else {
        __syncthreads();
        for (int s = 0; s < 2; s++)
            if (ncommit[s] > 0) mbar_wait(&mbar[s], (ncommit[s] - 1) & 1, nullptr, 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace qw6

using namespace qw6;

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static int pf_items_max(uint32_t tk, uint32_t ne) { return (int)((tk < ne ? tk : ne) + tk / kPfChunk + 1); }

extern "C" size_t qw6k_moe_prefill_ws_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t ne,
                                           uint32_t topk) {
    (void)hidden;
    const size_t tk = (size_t)ntok * topk;
    return al256(tk * 4) * 4 + al256(256 * 4) * 2 + al256((size_t)pf_items_max((uint32_t)tk, ne) * 16) + 256 +
           al256(tk * inter * 2);
}

static int pf_args(const qw6k_moe_desc* d, int* err, PfArgs& a) {
    if (!d || !d->gate || !d->up || !d->down || !d->logits || !d->x || !d->out || !d->ws || !err || !d->ntok ||
        !d->ne || d->ne > 256 || !d->topk || d->topk > 32 || d->topk > d->ne || (size_t)d->ntok * d->topk > (1u << 22))
        return QW6K_ERR_ARG;
    if (d->hidden % 256 || d->inter % 256 || !d->hidden || !d->inter || d->hidden > 16384 || d->inter > 16384)
        return QW6K_ERR_ARG;
    if (d->gq != QW6F_Q4_K_M && d->gq != QW6F_Q4_K_S && d->gq != QW6F_Q6_K) return QW6K_ERR_QUANT;
    if (d->dq != QW6F_Q4_K_M && d->dq != QW6F_Q4_K_S && d->dq != QW6F_Q6_K) return QW6K_ERR_QUANT;
    if (d->ws_bytes < qw6k_moe_prefill_ws_bytes(d->ntok, d->hidden, d->inter, d->ne, d->topk)) return QW6K_ERR_ARG;
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
    a.h = (__nv_bfloat16*)p;
    return 0;
}

template <int GQ>
static int launch_g1(const PfArgs& a, int mi, cudaStream_t st) {
    const size_t smem = 2 * (2 * 128 * 128 + kPfChunk * 128) + 1024;
    static bool cfg = false;
    if (!cfg && cudaFuncSetAttribute(k_pf_gemm1<GQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                    cudaSuccess)
        return QW6K_ERR_CUDA;
    cfg = true;
    k_pf_gemm1<GQ><<<mi * (a.inter / 128), 256, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

template <int DQ>
static int launch_g2(const PfArgs& a, int mi, cudaStream_t st) {
    const size_t smem = 2 * (128 * 128 + kPfChunk * 128) + 1024;
    static bool cfg = false;
    if (!cfg && cudaFuncSetAttribute(k_pf_gemm2<DQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                    cudaSuccess)
        return QW6K_ERR_CUDA;
    cfg = true;
    k_pf_gemm2<DQ><<<mi * (a.hidden / 128), 256, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_moe_prefill_check(const qw6k_moe_desc* d, int* err) {
    PfArgs a;
    return pf_args(d, err, a);
}

/* phases: 0 route, 1 count (after zeroing counts), 2 offsets, 3 scatter,
 * 4 gate/up GEMM (+silu), 5 down GEMM with weighted scatter-add (after zeroing out) */
extern "C" int qw6k_moe_prefill_phase(const qw6k_moe_desc* d, int* err, int phase, cudaStream_t st) {
    PfArgs a;
    const int rc = pf_args(d, err, a);
    if (rc) return rc;
    const int tk = a.ntok * a.topk;
    const int mi = pf_items_max((uint32_t)tk, (uint32_t)a.ne);
    switch (phase) {
    case 0:
        k_pf_route<<<(a.ntok + 7) / 8, 256, 0, st>>>(a);
        break;
    case 1:
        if (cudaMemsetAsync(a.cnt, 0, 256 * 4, st) != cudaSuccess) return QW6K_ERR_CUDA;
        k_pf_count<<<(tk + 255) / 256, 256, 0, st>>>(a);
        break;
    case 2:
        k_pf_offsets<<<1, 256, 0, st>>>(a);
        break;
    case 3:
        k_pf_scatter<<<(tk + 255) / 256, 256, 0, st>>>(a);
        break;
    case 4:
        return (d->gq == QW6F_Q6_K) ? launch_g1<QW6F_Q6_K>(a, mi, st) : launch_g1<QW6F_Q4_K_M>(a, mi, st);
    case 5:
        if (cudaMemsetAsync(a.out, 0, (size_t)a.ntok * a.hidden * 4, st) != cudaSuccess) return QW6K_ERR_CUDA;
        return (d->dq == QW6F_Q6_K) ? launch_g2<QW6F_Q6_K>(a, mi, st) : launch_g2<QW6F_Q4_K_M>(a, mi, st);
    default:
        return QW6K_ERR_ARG;
    }
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
