// k_fwd.cu -- the token-mixing halves of qw6's decoder layers on the GPU, for
// the decode-step executor (qw6_decoder.c).  One token per step; the step's
// token id and position are read from device memory (qw6k_step), so a whole
// step is position-independent and is captured once in a CUDA graph.
//
// Gated DeltaNet layer (qw6_apply_linear_attn, qw6.c:2292-2360), after the
// projections [qkv 8192 | z 4096 | beta 32 | alpha 32] of the normalised row,
// in one kernel (k_dn_token): the 4-tap causal conv with silu, the l2 norm
// of the 16 query and 16 key heads (qw6.c:2055-2063), beta = sigmoid(beta),
// g = softplus(alpha + dt) * a, then per value head vh (key head vh % 16,
// qw6.c:2084) for every state row j: row *= exp(g); pred = row . k;
// row += (v[j] - pred) * beta * k; o[j] = (row . q) / sqrt(128)
// (qw6_gated_delta_net_single, qw6.c:2079-2108), and rmsnorm(o) * silu(z)
// (qw6.c:2349-2355).
// Gated attention layer (qw6_apply_full_attn, qw6.c:2368-2424), after the
// projections [q|gate per head: 16 x 512 | k 512 | v 512]:
//   k_fa_prep     rmsnorm per head with q_norm / k_norm, RoPE on the first 64
//                 dimensions of each head (adjacent pairs, qw6_cpu_mrope,
//                 qw6.c:2711-2745), k and v into the caches at pos;
//   k_fa_attn     split-sequence attention of each query head over the pos+1
//                 cached positions of its key/value head (8 query heads per
//                 kv head): per chunk the max score, the sum of exp and the
//                 exp-weighted sum of values;
//   k_fa_combine  merge the chunks (qw6_cpu_attention_gqa's softmax,
//                 qw6.c:2750-2793) and gate with sigmoid(gate) (qw6.c:2419).
// Element-wise steps use qw6's operations in its order with IEEE rounding
// (__fmul_rn, __fadd_rn, ...: no contraction); dot products and sums are
// reductions in another order than qw6's sequential loops.  Every kernel is
// launched with programmatic dependent launch: it lets its successor start,
// may load weights (written once, at upload) and its own recurrent state
// (written only by the same kernel of the previous step), and waits for its
// predecessor before it reads what that one writes.  Data an earlier kernel
// writes comes through plain pointers, never `const __restrict__` (see
// qw6_pdl.cuh).
#include <cuda_runtime.h>

#include "qw6_launch.h"
#include "qw6_norm.cuh"
#include "qw6_pdl.cuh"

namespace qw6 {

constexpr int kQH = 16, kKVH = 2, kHD = 256;     // attention heads (qw6.h:29-31)
constexpr int kKH = 16, kKD = 128;               // DeltaNet key heads (qw6.h:34-35)
constexpr int kVH = 32, kVD = 128;               // DeltaNet value heads (qw6.h:36-37)
constexpr int kQKV = kKH * kKD * 2 + kVH * kVD;  // 8192
constexpr int kVDim = kVH * kVD;                 // 4096
constexpr int kRot = 64;                         // (int)(256 * 0.25f) rotary dims
constexpr int kFaSplit = QW6K_FA_SPLIT;          // sequence chunks per kv head

__device__ __forceinline__ float silu_f(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float sigmoid_f(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float softplus_f(float v) {  // qw6_softplus, qw6.h:298-302
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return log1pf(expf(v));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// out = rmsnorm(x) * w as qw6_cpu_rmsnorm evaluates it; one CTA of 256
// threads, dim <= 4096 (each thread keeps its values in registers).
__global__ void __launch_bounds__(256) k_rmsnorm(const float* x, const float* __restrict__ w, float* out,
                                                 int dim) {
    __shared__ float red[8];
    pdl_trigger_dependents();
    float wv[16], xv[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        wv[u] = i < dim ? w[i] : 0.f;
    }
    pdl_grid_wait();
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        xv[u] = i < dim ? x[i] : 0.f;
        ss = fmaf(xv[u], xv[u], ss);
    }
    const float t = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)dim), kRmsEps)));
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        if (i < dim) out[i] = __fmul_rn(__fmul_rn(xv[u], inv), wv[u]);
    }
}

// One token step of a Gated DeltaNet layer, one CTA per value head vh (key
// head kh = vh % 16, qw6.c:2084), 512 threads.  Threads 0-127 take query
// channel kh*128 + i of the causal conv, 128-255 key channel 2048 + kh*128 + i,
// 256-383 value channel 4096 + vh*128 + i: conv over the 4 latest qkv rows,
// silu, and the l2 norm of the query and key heads (qw6.c:2324-2343).  The
// conv window is a ring of 4 rows, row p % 4 holding position p's qkv, so a
// step reads the three older rows and the new projection and writes only row
// pos % 4 (qw6 shifts its window instead, qw6.c:2327-2331; the taps meet the
// same positions): the two value heads that share a key head can both
// compute its query and key without ordering.  Then the state rows, as
// qw6_gated_delta_net_single (qw6.c:2079-2108), and rmsnorm(o) * silu(z)
// (qw6.c:2349-2355).
__global__ void __launch_bounds__(512) k_dn_token(const float* proj, const qw6k_step* step, float* ring, const float* __restrict__ cw,
                                                  const float* __restrict__ dt, const float* __restrict__ a,
                                                  const float* __restrict__ nw, float* state, float* gated) {
    __shared__ __align__(16) float qk[2][kKD];
    __shared__ float vs[kVD], o[kVD], gbs[2];
    __shared__ float red[16];
    pdl_trigger_dependents();
    const int vh = blockIdx.x, kh = vh % kKH, tid = threadIdx.x, part = tid >> 7, i = tid & 127;
    const int warp = tid >> 5, lane = tid & 31;
    // this warp's 8 state rows, written only by this kernel in the previous
    // step: loaded while the projections finish
    float4* s = reinterpret_cast<float4*>(state + (size_t)vh * kVD * kVD);
    float4 row[8];
#pragma unroll
    for (int r = 0; r < 8; r++) row[r] = s[(warp * 8 + r) * (kVD / 4) + lane];
    pdl_grid_wait();
    const uint32_t pos = step->pos;
    float v = 0.f;
    if (part < 3) {
        const int c = part == 0 ? kh * kKD + i : part == 1 ? kKH * kKD + kh * kKD + i : 2 * kKH * kKD + vh * kVD + i;
        const float4 w = reinterpret_cast<const float4*>(cw)[c];
        const float s3 = proj[c];
        const float s0 = ring[(size_t)((pos + 1) & 3) * kQKV + c];  // position pos - 3
        const float s1 = ring[(size_t)((pos + 2) & 3) * kQKV + c];  // pos - 2
        const float s2 = ring[(size_t)((pos + 3) & 3) * kQKV + c];  // pos - 1
        float sum = __fmul_rn(s0, w.x);
        sum = __fadd_rn(sum, __fmul_rn(s1, w.y));
        sum = __fadd_rn(sum, __fmul_rn(s2, w.z));
        sum = __fadd_rn(sum, __fmul_rn(s3, w.w));
        v = silu_f(sum);
        if (part == 2 || vh < kKH) ring[(size_t)(pos & 3) * kQKV + c] = s3;  // one writer per channel
    }
    // l2 norms of the query (part 0) and key (part 1) heads: warps 0-3 and 4-7
    float sq = part < 2 ? v * v : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (lane == 0) red[warp] = sq;
    if (tid == 0) {
        gbs[0] = sigmoid_f(proj[kQKV + kVDim + vh]);
        gbs[1] = __fmul_rn(softplus_f(__fadd_rn(proj[kQKV + kVDim + kVH + vh], dt[vh])), a[vh]);
    }
    __syncthreads();
    if (part < 2) {
        const float ss = red[4 * part] + red[4 * part + 1] + red[4 * part + 2] + red[4 * part + 3];
        qk[part][i] = __fmul_rn(v, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, kRmsEps))));
    } else if (part == 2) {
        vs[i] = v;
    }
    __syncthreads();
    const float4 q4 = reinterpret_cast<const float4*>(qk[0])[lane];
    const float4 k4 = reinterpret_cast<const float4*>(qk[1])[lane];
    const float b = gbs[0], decay = expf(gbs[1]);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kVD));
#pragma unroll
    for (int r = 0; r < 8; r++) {
        const int j = warp * 8 + r;
        float4 x = row[r];
        x.x = __fmul_rn(x.x, decay);
        x.y = __fmul_rn(x.y, decay);
        x.z = __fmul_rn(x.z, decay);
        x.w = __fmul_rn(x.w, decay);
        const float pred = warp_sum(fmaf(x.w, k4.w, fmaf(x.z, k4.z, fmaf(x.y, k4.y, x.x * k4.x))));
        const float delta = __fmul_rn(__fsub_rn(vs[j], pred), b);
        x.x = __fadd_rn(x.x, __fmul_rn(delta, k4.x));
        x.y = __fadd_rn(x.y, __fmul_rn(delta, k4.y));
        x.z = __fadd_rn(x.z, __fmul_rn(delta, k4.z));
        x.w = __fadd_rn(x.w, __fmul_rn(delta, k4.w));
        s[j * (kVD / 4) + lane] = x;
        const float sum = warp_sum(fmaf(x.w, q4.w, fmaf(x.z, q4.z, fmaf(x.y, q4.y, x.x * q4.x))));
        if (lane == 0) o[j] = __fmul_rn(sum, scale);
    }
    __syncthreads();
    const float oi = tid < kVD ? o[tid] : 0.f;
    const float ss = block_sum(oi * oi, red);
    if (tid < kVD) {
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kVD), kRmsEps)));
        const float y = __fmul_rn(__fmul_rn(oi, inv), nw[tid]);
        gated[vh * kVD + tid] = __fmul_rn(y, silu_f(proj[kQKV + vh * kVD + tid]));
    }
}

// grid 18 x 256: CTAs 0-15 the query heads, 16-17 the key/value heads.
// freq[i/2] = powf(1e7, i / 64) for even i < 64, computed by the host's libm
// as qw6 computes it, so that theta = pos / freq is qw6's value.
__global__ void __launch_bounds__(256) k_fa_prep(const float* proj, const float* __restrict__ qn,
                                                 const float* __restrict__ kn, const float* __restrict__ freq,
                                                 const qw6k_step* step, float* kc, float* vc, float* qr) {
    __shared__ float y[kHD];
    __shared__ float red[8];
    pdl_trigger_dependents();
    pdl_grid_wait();
    const int h = blockIdx.x, d = threadIdx.x;
    const uint32_t pos = step->pos;
    const bool isq = h < kQH;
    const int kvh = h - kQH;
    const float x = isq ? proj[h * 2 * kHD + d] : proj[kQH * 2 * kHD + kvh * kHD + d];
    const float ss = block_sum(x * x, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), kRmsEps)));
    float val = __fmul_rn(__fmul_rn(x, inv), isq ? qn[d] : kn[d]);
    y[d] = val;
    __syncthreads();
    if (d < kRot) {
        const int i = d & ~1;
        const float theta = __fdiv_rn((float)pos, freq[i >> 1]);
        const float c = cosf(theta), sn = sinf(theta), av = y[i], bv = y[i + 1];
        val = (d & 1) ? __fadd_rn(__fmul_rn(av, sn), __fmul_rn(bv, c)) : __fsub_rn(__fmul_rn(av, c), __fmul_rn(bv, sn));
    }
    if (isq) {
        qr[h * kHD + d] = val;
    } else {
        const size_t slot = ((size_t)pos * kKVH + kvh) * kHD + d;
        kc[slot] = val;
        vc[slot] = proj[kQH * 2 * kHD + kKVH * kHD + kvh * kHD + d];
    }
}

// positions [c0, c1) of chunk blockIdx.x for the current sequence length
__device__ __forceinline__ void fa_chunk(uint32_t seq, int c, uint32_t& c0, uint32_t& c1) {
    const uint32_t per = 32u * ((seq + 32u * kFaSplit - 1) / (32u * kFaSplit));
    c0 = (uint32_t)c * per;
    c1 = c0 + per < seq ? c0 + per : seq;
}

// grid (kFaSplit, 2 kv heads) x 256: warp w is query head 8 g + w; lane owns
// dimensions [8 lane, 8 lane + 8).  part: m, l per (head, chunk), then the
// [head][chunk][256] value sums.
__global__ void __launch_bounds__(256) k_fa_attn(const float* qr, const float* kc, const float* vc,
                                                 const qw6k_step* step, float* part) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const uint32_t seq = step->pos + 1;
    uint32_t c0, c1;
    fa_chunk(seq, blockIdx.x, c0, c1);
    if (c0 >= seq) return;
    const int g = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, h = g * (kQH / kKVH) + warp;
    const float4* q = reinterpret_cast<const float4*>(qr + h * kHD) + 2 * lane;
    const float4 qa = q[0], qb = q[1];
    float m = -INFINITY, l = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (uint32_t t0 = c0; t0 < c1; t0 += 32) {
        const int n = (int)(c1 - t0 < 32 ? c1 - t0 : 32);
        float mine = -INFINITY;
        for (int t = 0; t < n; t += 4) {
            float p[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                p[u] = 0.f;
                if (t + u < n) {
                    const float4* kr = reinterpret_cast<const float4*>(kc + ((size_t)(t0 + t + u) * kKVH + g) * kHD) +
                                       2 * lane;
                    const float4 ka = kr[0], kb = kr[1];
                    p[u] = fmaf(qa.x, ka.x, fmaf(qa.y, ka.y, fmaf(qa.z, ka.z, fmaf(qa.w, ka.w,
                           fmaf(qb.x, kb.x, fmaf(qb.y, kb.y, fmaf(qb.z, kb.z, qb.w * kb.w)))))));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float sc = __fmul_rn(warp_sum(p[u]), 0.0625f);  // dot / sqrtf(256), exact
                if (lane == t + u) mine = sc;
            }
        }
        const float mn = fmaxf(m, warp_max(mine));
        const float alpha = expf(m - mn);  // 0 for the first sub-chunk
        const float e = lane < n ? expf(mine - mn) : 0.f;
        l = fmaf(l, alpha, warp_sum(e));
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] *= alpha;
        for (int t = 0; t < n; t++) {
            const float et = __shfl_sync(0xffffffffu, e, t);
            const float4* vr = reinterpret_cast<const float4*>(vc + ((size_t)(t0 + t) * kKVH + g) * kHD) + 2 * lane;
            const float4 va = vr[0], vb = vr[1];
            acc[0] = fmaf(et, va.x, acc[0]);
            acc[1] = fmaf(et, va.y, acc[1]);
            acc[2] = fmaf(et, va.z, acc[2]);
            acc[3] = fmaf(et, va.w, acc[3]);
            acc[4] = fmaf(et, vb.x, acc[4]);
            acc[5] = fmaf(et, vb.y, acc[5]);
            acc[6] = fmaf(et, vb.z, acc[6]);
            acc[7] = fmaf(et, vb.w, acc[7]);
        }
        m = mn;
    }
    const int slot = h * kFaSplit + blockIdx.x;
    if (lane == 0) {
        part[2 * slot] = m;
        part[2 * slot + 1] = l;
    }
    float4* o = reinterpret_cast<float4*>(part + 2 * kQH * kFaSplit + (size_t)slot * kHD) + 2 * lane;
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// grid 16 (query heads) x 256 (dimensions)
__global__ void __launch_bounds__(256) k_fa_combine(const float* part, const float* proj, const qw6k_step* step,
                                                    float* attn) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    const uint32_t seq = step->pos + 1;
    const int h = blockIdx.x, d = threadIdx.x;
    int nc = 0;
    for (; nc < kFaSplit; nc++) {
        uint32_t c0, c1;
        fa_chunk(seq, nc, c0, c1);
        if (c0 >= seq) break;
    }
    float mx = -INFINITY;
    for (int c = 0; c < nc; c++) mx = fmaxf(mx, part[2 * (h * kFaSplit + c)]);
    float l = 0.f, o = 0.f;
    for (int c = 0; c < nc; c++) {
        const int slot = h * kFaSplit + c;
        const float f = expf(part[2 * slot] - mx);
        l = fmaf(part[2 * slot + 1], f, l);
        o = fmaf(part[2 * kQH * kFaSplit + (size_t)slot * kHD + d], f, o);
    }
    const float gate = proj[h * 2 * kHD + kHD + d];
    attn[h * kHD + d] = __fmul_rn(__fdiv_rn(o, l), sigmoid_f(gate));
}

__global__ void k_check_finite(const float* x, uint32_t n, int* bad) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    bool finite = true;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        finite = finite && isfinite(x[i]);
    if (!finite) atomicOr(bad, 1);
}

// the step's greedy token (largest packed argmax key: largest logit, lowest
// index on ties) becomes the next step's input at the next position
__global__ void k_step_next(qw6k_step* step, const unsigned long long* key) {
    pdl_grid_wait();
    step->token = ~(uint32_t)(*key & 0xffffffffull);
    step->pos += 1;
}

}  // namespace qw6

using namespace qw6;

extern "C" size_t qw6k_fa_part_floats(void) { return (size_t)kQH * kFaSplit * (2 + kHD); }

extern "C" int qw6k_rmsnorm(const float* x, const float* w, float* out, uint32_t dim, cudaStream_t st) {
    if (!x || !w || !out || !dim) return QW6K_ERR_ARG;
    if (dim > 4096) return QW6K_ERR_ARG;
    return launch_pdl(k_rmsnorm, dim3(1), dim3(256), 0, st, x, w, out, (int)dim) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_dn_token(const float* proj, const qw6k_step* step, float* ring, const float* conv_w,
                             const float* dt, const float* a, const float* dn_norm, float* state, float* gated,
                             cudaStream_t st) {
    if (!proj || !step || !ring || !conv_w || !dt || !a || !dn_norm || !state || !gated) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(conv_w) | reinterpret_cast<uintptr_t>(state)) & 15u) return QW6K_ERR_ALIGN;
    return launch_pdl(k_dn_token, dim3(kVH), dim3(512), 0, st, proj, step, ring, conv_w, dt, a, dn_norm, state,
                      gated) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_fa_prep(const float* proj, const float* q_norm, const float* k_norm, const float* freq,
                            const qw6k_step* step, float* k_cache, float* v_cache, float* q_rot, cudaStream_t st) {
    if (!proj || !q_norm || !k_norm || !freq || !step || !k_cache || !v_cache || !q_rot) return QW6K_ERR_ARG;
    return launch_pdl(k_fa_prep, dim3(kQH + kKVH), dim3(kHD), 0, st, proj, q_norm, k_norm, freq, step, k_cache,
                      v_cache, q_rot) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_fa_attn(const float* q_rot, const float* k_cache, const float* v_cache, const qw6k_step* step,
                            float* part, const float* proj, float* attn, cudaStream_t st) {
    if (!q_rot || !k_cache || !v_cache || !step || !part || !proj || !attn) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(q_rot) | reinterpret_cast<uintptr_t>(k_cache) |
         reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(part)) & 15u)
        return QW6K_ERR_ALIGN;
    if (launch_pdl(k_fa_attn, dim3(kFaSplit, kKVH), dim3(256), 0, st, q_rot, k_cache, v_cache, step, part) !=
        cudaSuccess)
        return QW6K_ERR_CUDA;
    return launch_pdl(k_fa_combine, dim3(kQH), dim3(kHD), 0, st, part, proj, step, attn) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_check_finite(const float* x, uint32_t n, int* bad, cudaStream_t st) {
    if (!x || !n || !bad) return QW6K_ERR_ARG;
    const uint32_t grid = (n + 1023) / 1024 < 148 ? (n + 1023) / 1024 : 148;
    return launch_pdl(k_check_finite, dim3(grid), dim3(256), 0, st, x, n, bad) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_step_next(qw6k_step* step, const unsigned long long* key, cudaStream_t st) {
    if (!step || !key) return QW6K_ERR_ARG;
    return launch_pdl(k_step_next, dim3(1), dim3(1), 0, st, step, key) == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
