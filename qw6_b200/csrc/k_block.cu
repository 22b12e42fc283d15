// k_block.cu -- the MoE FFN block around the routed experts, as qw6's
// forward pass applies it to every layer (qw6.c:2474-2484 around
// qw6_apply_layer_moe, qw6.c:2226-2290):
//   normed = rmsnorm(x) * norm_w                   (qw6_cpu_rmsnorm, qw6.c:2502-2512)
//   logits = router . normed                       (fp32 router, qw6.c:2247)
//   ffn    = routed experts (k_moe.cu)             (qw6.c:2249-2264)
//   s      = sigmoid(shared_router . normed) or 1  (qw6.c:2268-2273)
//   ffn   += s * shared_down(silu(shared_gate normed) * shared_up normed)
//   out    = x + ffn                               (qw6.c:2482-2483)
// This file holds the prologue (RMSNorm + router logits + shared gate, one
// pass over x per token) and the epilogue (shared-expert weighting and the
// residual); the routed experts and the shared expert's matvecs are the
// library's existing kernels, so the whole block is device-resident.
#include <cuda_runtime.h>

#include "qw6_dev.cuh"
#include "qw6_devcfg.cuh"
#include "qw6_launch.h"
#include "qw6_norm.cuh"
#include "qw6_pdl.cuh"

namespace qw6 {

constexpr int kBlkThreads = 256;  // 8 router rows per CTA
constexpr int kRowRegs = 16;  // float4 of a router row a lane holds in registers (hidden <= 2048)
constexpr int kRowVals = 16;  // values of the token row a thread holds in registers (hidden <= 4096)

// grid (ceil((ne + 1) / 8), ntok): CTA (b, t) computes rows [8b, 8b+8) of
// token t (warp per row): rows < ne are the router's, row ne is the shared
// router (gate sigmoid(shared_router . normed), or 1 without one); CTA (0, t)
// also writes normed[t].
// normed[i] = (x[i] * inv) * w[i] as qw6 evaluates it.  With `add` the block
// input is x + add (the residual add before the FFN, qw6.c:2469-2470), which
// CTA (0, t) stores to xsum and checks for NaN/Inf (sets *bad, qw6.c:2472).
__global__ void __launch_bounds__(kBlkThreads) k_block_pre(const float* x, const float* add, float* xsum, int* bad,
                                                           const float* __restrict__ norm_w,
                                                           const float* __restrict__ router,
                                                           const float* __restrict__ srouter, float* normed, float* logits,
                                                           float* sgate,
                                                           int hidden, int ne) {
    extern __shared__ __align__(16) float nrm[];  // [hidden]
    __shared__ float red[kBlkThreads / 32];
    const int t = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // launched with programmatic dependent launch: the warp's router row
    // (no kernel before this one writes it) is loaded while the previous
    // kernel finishes, then the wait for x / add
    pdl_trigger_dependents();
    const int r = blockIdx.x * (kBlkThreads / 32) + warp;
    // this warp's row: a router row, or the shared router as row ne
    const float* wr = r < ne ? router + (size_t)r * hidden : (r == ne ? srouter : nullptr);
    const bool held = wr && hidden <= 128 * kRowRegs;
    float4 wv[kRowRegs];
#pragma unroll
    for (int u = 0; u < kRowRegs; u++) {
        const int c = 4 * lane + 128 * u;
        wv[u] = held && c < hidden ? __ldg(reinterpret_cast<const float4*>(wr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float* xt = x + (size_t)t * hidden;
    if (hidden <= kBlkThreads * kRowVals) {
        // the row in registers: every load of a phase is issued before the
        // first use (a load loop that also stores is issued one load at a time)
        float nw[kRowVals], xv[kRowVals], av[kRowVals];
#pragma unroll
        for (int u = 0; u < kRowVals; u++) {
            const int i = threadIdx.x + kBlkThreads * u;
            nw[u] = i < hidden ? norm_w[i] : 0.f;
        }
        pdl_grid_wait();
#pragma unroll
        for (int u = 0; u < kRowVals; u++) {
            const int i = threadIdx.x + kBlkThreads * u;
            xv[u] = i < hidden ? xt[i] : 0.f;
            av[u] = add && i < hidden ? add[(size_t)t * hidden + i] : 0.f;
        }
        float ss = 0.f;
        bool finite = true;
#pragma unroll
        for (int u = 0; u < kRowVals; u++) {
            if (add) xv[u] = __fadd_rn(xv[u], av[u]);  // the residual add (qw6.c:2469-2470)
            finite = finite && isfinite(xv[u]);
            ss = fmaf(xv[u], xv[u], ss);
        }
        if (add && blockIdx.x == 0) {
#pragma unroll
            for (int u = 0; u < kRowVals; u++) {
                const int i = threadIdx.x + kBlkThreads * u;
                if (i < hidden) xsum[(size_t)t * hidden + i] = xv[u];
            }
            if (!finite && bad) atomicOr(bad, 1);
        }
        const float tot = block_sum(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)hidden), kRmsEps)));
#pragma unroll
        for (int u = 0; u < kRowVals; u++) {
            const int i = threadIdx.x + kBlkThreads * u;
            if (i < hidden) {
                const float v = __fmul_rn(__fmul_rn(xv[u], inv), nw[u]);
                nrm[i] = v;
                if (blockIdx.x == 0) normed[(size_t)t * hidden + i] = v;
            }
        }
    } else {  // hidden > 4096: strided loops
        pdl_grid_wait();
        if (add) {  // x + add into shared memory first, then the norm of the sum
            const float* at = add + (size_t)t * hidden;
            bool finite = true;
#pragma unroll 8
            for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
                const float v = __fadd_rn(xt[i], at[i]);
                nrm[i] = v;
                finite = finite && isfinite(v);
                if (blockIdx.x == 0) xsum[(size_t)t * hidden + i] = v;
            }
            if (!finite && blockIdx.x == 0 && bad) atomicOr(bad, 1);
            __syncthreads();
            xt = nrm;
        }
        const float inv = rms_inv(xt, hidden, red);
#pragma unroll 8
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
            const float v = __fmul_rn(__fmul_rn(xt[i], inv), norm_w[i]);
            nrm[i] = v;  // each thread rewrites only the entries it read
            if (blockIdx.x == 0) normed[(size_t)t * hidden + i] = v;
        }
    }
    __syncthreads();
    if (wr) {
        float acc = 0.f;
        if (held) {
#pragma unroll
            for (int u = 0; u < kRowRegs; u++) {
                const int c = 4 * lane + 128 * u;
                if (c < hidden) {
                    acc = fmaf(wv[u].x, nrm[c], acc);
                    acc = fmaf(wv[u].y, nrm[c + 1], acc);
                    acc = fmaf(wv[u].z, nrm[c + 2], acc);
                    acc = fmaf(wv[u].w, nrm[c + 3], acc);
                }
            }
        } else {
            for (int c = 4 * lane; c < hidden; c += 128) {
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(wr + c));
                acc = fmaf(w4.x, nrm[c], acc);
                acc = fmaf(w4.y, nrm[c + 1], acc);
                acc = fmaf(w4.z, nrm[c + 2], acc);
                acc = fmaf(w4.w, nrm[c + 3], acc);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            if (r < ne) logits[(size_t)t * ne + r] = acc;
            else sgate[t] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-acc)));  // qw6_sigmoid (qw6.h:295-297)
        }
    }
    if (!srouter && r == ne && lane == 0) sgate[t] = 1.0f;  // no shared router: weight 1 (qw6.c:2268)
}

// out[t][i] = x[t][i] + (ffn[t][i] + s[t] * sh[t][i])  (sh may be null: no
// shared expert), each operation rounded once as qw6's loops do; a NaN/Inf
// in out sets *bad (qw6.c:2485-2487).
__global__ void k_block_post(const float* x, const float* ffn, const float* sh, const float* sgate, float* out, int* bad,
                             int hidden, long long n) {
    pdl_trigger_dependents();
    pdl_grid_wait();
    bool finite = true;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        float f = ffn[i];
        if (sh) f = __fadd_rn(f, __fmul_rn(sgate[i / hidden], sh[i]));
        const float o = __fadd_rn(x[i], f);
        out[i] = o;
        finite = finite && isfinite(o);
    }
    if (!finite && bad) atomicOr(bad, 1);
}

// One token row per CTA (hidden <= 4096): out = x + (ffn + s * sh) as
// k_block_post, then normed = rmsnorm(out) * w as qw6_cpu_rmsnorm (the next
// layer's input norm, or the final norm before the LM head, qw6.c:2462,
// 2493): the residual add and the norm that follows it in one pass.
__global__ void __launch_bounds__(256) k_post_norm(const float* x, const float* ffn, const float* sh,
                                                   const float* sgate, float* out, int* bad,
                                                   const float* __restrict__ w, float* normed,
                                                   int hidden) {
    __shared__ float red[8];
    pdl_trigger_dependents();
    float wv[16], ov[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        wv[u] = i < hidden ? w[i] : 0.f;
    }
    pdl_grid_wait();
    const size_t base = (size_t)blockIdx.x * hidden;
    const float s = sh ? sgate[blockIdx.x] : 0.f;
    float fv[16], hv[16];
#pragma unroll
    for (int u = 0; u < 16; u++) {  // every load before the first store
        const int i = threadIdx.x + 256 * u;
        ov[u] = i < hidden ? x[base + i] : 0.f;
        fv[u] = i < hidden ? ffn[base + i] : 0.f;
        hv[u] = sh && i < hidden ? sh[base + i] : 0.f;
    }
    bool finite = true;
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        if (i < hidden) {
            float f = fv[u];
            if (sh) f = __fadd_rn(f, __fmul_rn(s, hv[u]));
            const float o = __fadd_rn(ov[u], f);
            ov[u] = o;
            finite = finite && isfinite(o);
            ss = fmaf(o, o, ss);
        }
    }
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        if (i < hidden) out[base + i] = ov[u];
    }
    if (!finite && bad) atomicOr(bad, 1);
    const float t = block_sum(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hidden), kRmsEps)));
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int i = threadIdx.x + 256 * u;
        if (i < hidden) normed[base + i] = __fmul_rn(__fmul_rn(ov[u], inv), wv[u]);
    }
}

}  // namespace qw6

using namespace qw6;

extern "C" int qw6k_block_pre(const float* x, const float* add, float* xsum, int* bad, const float* norm_w,
                              const float* router, const float* srouter, float* normed, float* logits, float* sgate,
                              uint32_t ntok, uint32_t hidden, uint32_t ne, cudaStream_t st) {
    if (!x || !norm_w || !router || !normed || !logits || !sgate || !ntok || ntok > 65535 || !hidden ||
        hidden % 4 || hidden > 16384 || !ne || ne > 256 || (add && !xsum))
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(router) | reinterpret_cast<uintptr_t>(srouter) | reinterpret_cast<uintptr_t>(x)) &
        15u)
        return QW6K_ERR_ALIGN;
    static DevFlags cfg;
    if (hidden * 4 > 48 * 1024 && smem_optin(cfg, k_block_pre, (int)hidden * 4)) return QW6K_ERR_CUDA;
    const dim3 grid((ne + 1 + kBlkThreads / 32 - 1) / (kBlkThreads / 32), ntok);
    return launch_pdl(k_block_pre, grid, dim3(kBlkThreads), (size_t)hidden * 4, st, x, add, xsum, bad, norm_w, router,
                      srouter, normed, logits, sgate, (int)hidden, (int)ne) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_block_post(const float* x, const float* ffn, const float* shared, const float* sgate, float* out,
                               int* bad, uint32_t ntok, uint32_t hidden, cudaStream_t st) {
    if (!x || !ffn || !out || !ntok || !hidden || (shared && !sgate)) return QW6K_ERR_ARG;
    const long long n = (long long)ntok * hidden;
    const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    return launch_pdl(k_block_post, dim3(grid), dim3(256), 0, st, x, ffn, shared, sgate, out, bad, (int)hidden, n) ==
                   cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

extern "C" int qw6k_post_norm(const float* x, const float* ffn, const float* shared, const float* sgate, float* out,
                              int* bad, const float* norm_w, float* normed, uint32_t ntok, uint32_t hidden,
                              cudaStream_t st) {
    if (!x || !ffn || !out || !norm_w || !normed || !ntok || ntok > 65535 || !hidden || hidden > 4096 ||
        (shared && !sgate))
        return QW6K_ERR_ARG;
    return launch_pdl(k_post_norm, dim3(ntok), dim3(256), 0, st, x, ffn, shared, sgate, out, bad, norm_w, normed,
                      (int)hidden) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}
