// k_matvec.cu -- GGUF super-block kernels: exact dequantization, repacking
// into the tile layout, and the streaming int8 tensor-core matvec.
//
// Reference behaviour: qw6_tensor_dequantize_row (qw6.c:1674-1724) and
// qw6_tensor_matvec (qw6.c:1769-1791); the Vulkan dispatch this replaces is
// qw6_vk_pipe_matvec (qw6_vk.c:2386-2430) with the matmul_*.comp shaders.
#include <cuda_runtime.h>

#include "qw6_argmax.cuh"
#include "qw6_dev.cuh"
#include "qw6_devcfg.cuh"
#include "qw6_grids.cuh"
#include "qw6_launch.h"
#include "qw6_pdl.cuh"

namespace qw6 {

// ======================================================= exact dequant ====
// One thread per (row, super-block, 32-weight group).  Every product and
// difference is rounded separately (no FMA) in qw6's evaluation order, so the
// output is bit-identical to qw6_tensor_dequantize_row.

__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int j, uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
        mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ uint32_t rd16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

__device__ __forceinline__ float sgnmul(float v, uint32_t bit) { return bit ? -v : v; }

template <int F>
__device__ void dequant_group(const uint8_t* blk, int j, float* o) {
    if constexpr (F == QW6F_Q4_K_M || F == QW6F_Q5_K) {
        const float d = f16_bits_exact(rd16(blk)), dm = f16_bits_exact(rd16(blk + 2));
        uint32_t sc, mn;
        k4_scale_min(blk + 4, j, sc, mn);
        const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dm, (float)mn);
        const int c = j >> 1, hh = j & 1;
        const uint8_t* q = blk + (F == QW6F_Q5_K ? 48 : 16) + 32 * c;
        for (int l = 0; l < 32; l++) {
            uint32_t v = hh ? (q[l] >> 4) : (q[l] & 15u);
            if constexpr (F == QW6F_Q5_K) v += (blk[16 + l] >> j) & 1u ? 16u : 0u;
            o[l] = __fsub_rn(__fmul_rn(dl, (float)v), ml);
        }
    } else if constexpr (F == QW6F_Q6_K) {
        const float d = f16_bits_exact(rd16(blk + 208));
        const int n = j >> 2, kk = j & 3;
        const uint8_t* ql = blk + 64 * n + ((kk & 1) ? 32 : 0);
        const uint8_t* qh = blk + 128 + 32 * n;
        const float ds = __fmul_rn(d, (float)(int8_t)blk[192 + 8 * n + 2 * kk]);
        for (int l = 0; l < 32; l++) {
            const int lo = (kk & 2) ? (ql[l] >> 4) : (ql[l] & 15);
            const int q = (lo | (((qh[l] >> (2 * kk)) & 3) << 4)) - 32;
            o[l] = __fmul_rn(ds, (float)q);
        }
    } else if constexpr (F == QW6F_IQ2_XXS) {
        const float d = f16_bits_exact(rd16(blk));
        const uint8_t* grp = blk + 2 + 8 * j;
        const uint32_t aux = (uint32_t)grp[4] | ((uint32_t)grp[5] << 8) | ((uint32_t)grp[6] << 16) |
                             ((uint32_t)grp[7] << 24);
        const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.25f);
        for (int l = 0; l < 4; l++) {
            const uint8_t* gr = d_grid_iq2xxs + 8u * grp[l];
            const uint32_t s = qw6_ksigns((aux >> (7 * l)) & 127u);
            for (int jj = 0; jj < 8; jj++) o[8 * l + jj] = sgnmul(__fmul_rn(db, (float)gr[jj]), (s >> jj) & 1u);
        }
    } else if constexpr (F == QW6F_IQ2_S) {
        const float d = f16_bits_exact(rd16(blk));
        const uint8_t *qs = blk + 2, *sg = blk + 34, *qh = blk + 66, *sc = blk + 74;
        const float d0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc[j] & 15u))), 0.25f);
        const float d1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc[j] >> 4))), 0.25f);
        for (int l = 0; l < 4; l++) {
            const uint32_t gi = qs[4 * j + l] | (((uint32_t)qh[j] << (8 - 2 * l)) & 0x300u);
            const uint8_t* gr = d_grid_iq2s + 8u * gi;
            const float dl = l < 2 ? d0 : d1;
            const uint32_t s = sg[4 * j + l];
            for (int jj = 0; jj < 8; jj++) o[8 * l + jj] = sgnmul(__fmul_rn(dl, (float)gr[jj]), (s >> jj) & 1u);
        }
    } else if constexpr (F == QW6F_IQ3_S) {
        const float d = f16_bits_exact(rd16(blk));
        const uint8_t *qs = blk + 2 + 8 * j, *s = blk + 74 + 4 * j;
        const uint32_t h = blk[66 + j], scb = blk[106 + (j >> 1)];
        const uint32_t nib = (j & 1) ? (scb >> 4) : (scb & 15u);
        const float db = __fmul_rn(d, (float)(int)(1 + 2 * nib));
        for (int l = 0; l < 4; l++) {
            const uint32_t i1 = qs[2 * l] | ((h << (8 - 2 * l)) & 256u);
            const uint32_t i2 = qs[2 * l + 1] | ((h << (7 - 2 * l)) & 256u);
            const uint8_t *g1 = d_grid_iq3s + 4u * i1, *g2 = d_grid_iq3s + 4u * i2;
            for (int jj = 0; jj < 4; jj++) {
                o[8 * l + jj] = sgnmul(__fmul_rn(db, (float)g1[jj]), (s[l] >> jj) & 1u);
                o[8 * l + jj + 4] = sgnmul(__fmul_rn(db, (float)g2[jj]), (s[l] >> (jj + 4)) & 1u);
            }
        }
    }
}

template <int F>
__global__ void k_dequant(const uint8_t* __restrict__ w, float* __restrict__ out, int rows, int cols) {
    const int nb = cols / 256;
    const long long item = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)rows * nb * 8;
    if (item >= total) return;
    const int j = (int)(item & 7), b = (int)((item >> 3) % nb);
    const long long r = (item >> 3) / nb;
    const uint8_t* blk = w + ((size_t)r * nb + b) * (size_t)Fmt<F>::BB;
    dequant_group<F>(blk, j, out + (size_t)r * cols + 256 * b + 32 * j);
}

// =============================================================== repack ====
// raw GGUF rows -> tile layout; one CTA per (tile-block, matrix).  Rows past
// `rows` in the last m-tile are zero-filled (d = 0 makes them inert).

template <int F>
__global__ void k_pack(const uint8_t* __restrict__ raw, uint8_t* __restrict__ packed, int rows, int cols,
                       size_t raw_stride, size_t pk_stride) {
    constexpr int BB = Fmt<F>::BB, TB = Fmt<F>::TB;
    __shared__ __align__(16) uint8_t s[TB];
    const int nb = cols / 256;
    const int tb = blockIdx.x, mt = tb / nb, b = tb % nb;
    const uint8_t* src = raw + (size_t)blockIdx.y * raw_stride;
    uint8_t* dst = packed + (size_t)blockIdx.y * pk_stride + (size_t)tb * TB;
    const size_t rb = (size_t)nb * BB;
    for (int i = threadIdx.x; i < TB; i += blockDim.x) {
        const int r = i / BB, p = i % BB, row = mt * 16 + r;
        s[Fmt<F>::dst(r, p)] = row < rows ? src[(size_t)row * rb + (size_t)b * BB + p] : 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < TB / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(s)[i];
}

// ============================================================== matvec ====
// y[tok][r] = sum_c W[r][c] x[tok][c] for tok < ntok (<= 4*NQ).
// Work item = (m-tile of 16 rows, k-split).  A CTA of 8 warps covers
// 8/ks m-tiles x ks splits; the ks partial sums of an m-tile are combined in
// shared memory in split order (deterministic).  Each warp double-buffers its
// tile-block fragments in registers; the first block of the next item is
// prefetched while the current one is consumed.

struct MvArgs {
    const uint8_t* w;
    const float* x;
    float* y;  // may be null when KEYS (argmax only)
    int rows, cols, ntok, ldx, ldy, ks, nb, mtiles;
    unsigned long long* keys;  // KEYS: per-token packed (value, row_offset + row) max
    uint32_t row_offset;
};

// Batch-1 kernels run 2 CTAs per SM; those of the smaller tile formats keep
// two tile-blocks in flight per warp (three register buffers), the rest
// double-buffer.
template <int F, int NQ>
struct MvTriple {
    static constexpr bool value = NQ == 1 && F != QW6F_Q6_K;
};

template <int F, int NQ, bool KEYS>
__global__ void __launch_bounds__(kThreads, NQ == 1 ? 2 : 1) k_matvec(const MvArgs a) {
    constexpr bool kTriple = MvTriple<F, NQ>::value;
    extern __shared__ __align__(16) uint8_t smem[];
    using T = Tile<F, NQ>;
    constexpr int TB = T::TB;
    constexpr size_t tbl_bytes = IQLut<F>::bytes;
    uint32_t* tbl = reinterpret_cast<uint32_t*>(smem);
    XStage xs = xstage_carve(smem + tbl_bytes, 4 * NQ, a.cols);
    float* red = reinterpret_cast<float*>(smem + tbl_bytes + xstage_bytes(4 * NQ, a.cols));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = a.ks, wpm = kWarps / ks, ms = warp / ks, split = warp % ks, nbk = a.nb / ks;
    const int ngrp = (a.mtiles + wpm - 1) / wpm;
    // token chunk of this CTA (grid y): tokens [tok0, tok0 + 4 NQ)
    const int tok0 = (int)blockIdx.y * 4 * NQ;
    const int ntok = min(a.ntok - tok0, 4 * NQ);
    const float* xin = a.x + (size_t)tok0 * a.ldx;
    float* yout = a.y ? a.y + (size_t)tok0 * a.ldy : nullptr;
    unsigned long long* kout = KEYS ? a.keys + tok0 : nullptr;
    const int n_iter = blockIdx.x < ngrp ? (ngrp - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nsteps = n_iter * nbk;

    auto item_mt = [&](int it) { return ((int)blockIdx.x + it * (int)gridDim.x) * wpm + ms; };
    auto tile_ptr = [&](int step) {
        const int it = step / nbk, i = step % nbk;
        return a.w + ((size_t)item_mt(it) * a.nb + (size_t)split * nbk + i) * TB;
    };
    auto step_ok = [&](int step) { return step < nsteps && item_mt(step / nbk) < a.mtiles; };

    pdl_trigger();
    typename T::Frag fa, fb, fc;
    if (step_ok(0)) T::load(fa, tile_ptr(0), lane);  // weights: nothing earlier in the stream writes them
    if constexpr (IsIQ<F>::value) IQLut<F>::init(tbl, grid_ptr<F>());
    pdl_wait();  // x comes from the previous kernel
    xstage_fill(xs, xin, a.ldx, ntok, 4 * NQ, a.cols);
    __syncthreads();
    const XView xv = xs.view();

    float acc[2][NQ];
    unsigned long long best[NQ];
#pragma unroll
    for (int qt = 0; qt < NQ; qt++) {
        acc[0][qt] = acc[1][qt] = 0.f;
        best[qt] = 0ull;
    }

    auto epilogue = [&](int step) {
        const int mt = item_mt(step / nbk);
        const int g = lane >> 2, t = lane & 3;
        if (ks > 1) {
#pragma unroll
            for (int qt = 0; qt < NQ; qt++) {
                red[(warp * 32 + lane) * 2 * NQ + 2 * qt] = acc[0][qt];
                red[(warp * 32 + lane) * 2 * NQ + 2 * qt + 1] = acc[1][qt];
            }
            __syncthreads();
            if (split == 0) {
#pragma unroll
                for (int qt = 0; qt < NQ; qt++) {
                    float s0 = 0.f, s1 = 0.f;
                    for (int s = 0; s < ks; s++) {
                        s0 += red[((warp + s) * 32 + lane) * 2 * NQ + 2 * qt];
                        s1 += red[((warp + s) * 32 + lane) * 2 * NQ + 2 * qt + 1];
                    }
                    acc[0][qt] = s0;
                    acc[1][qt] = s1;
                }
            }
            __syncthreads();
        }
        if (split == 0 && mt < a.mtiles) {
#pragma unroll
            for (int qt = 0; qt < NQ; qt++) {
                const int tok = 4 * qt + t;
                if (tok < ntok) {
                    const int r0 = mt * 16 + g;
                    if (!KEYS || yout) {
                        if (r0 < a.rows) yout[(size_t)tok * a.ldy + r0] = acc[0][qt];
                        if (r0 + 8 < a.rows) yout[(size_t)tok * a.ldy + r0 + 8] = acc[1][qt];
                    }
                    if (KEYS) {
                        if (r0 < a.rows) {
                            const unsigned long long k0 = argmax_key(acc[0][qt], a.row_offset + (uint32_t)r0);
                            best[qt] = k0 > best[qt] ? k0 : best[qt];
                        }
                        if (r0 + 8 < a.rows) {
                            const unsigned long long k1 = argmax_key(acc[1][qt], a.row_offset + (uint32_t)r0 + 8);
                            best[qt] = k1 > best[qt] ? k1 : best[qt];
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) acc[0][qt] = acc[1][qt] = 0.f;
    };

    if constexpr (!kTriple) {
        for (int s = 0; s < nsteps; s += 2) {
            if (step_ok(s + 1)) T::load(fb, tile_ptr(s + 1), lane);
            if (step_ok(s)) tile_dot<F, NQ>(fa, xv, split * nbk + s % nbk, acc, lane, tbl);
            if (s % nbk == nbk - 1) epilogue(s);
            if (s + 1 < nsteps) {
                if (step_ok(s + 2)) T::load(fa, tile_ptr(s + 2), lane);
                if (step_ok(s + 1)) tile_dot<F, NQ>(fb, xv, split * nbk + (s + 1) % nbk, acc, lane, tbl);
                if ((s + 1) % nbk == nbk - 1) epilogue(s + 1);
            }
        }
    } else {
    // three fragment buffers: the loads of steps s+1 and s+2 are in flight
    // while step s is consumed
    if (step_ok(1)) T::load(fb, tile_ptr(1), lane);
    for (int s = 0; s < nsteps; s += 3) {
        if (step_ok(s + 2)) T::load(fc, tile_ptr(s + 2), lane);
        if (step_ok(s)) tile_dot<F, NQ>(fa, xv, split * nbk + s % nbk, acc, lane, tbl);
        if (s % nbk == nbk - 1) epilogue(s);
        if (s + 1 >= nsteps) break;
        if (step_ok(s + 3)) T::load(fa, tile_ptr(s + 3), lane);
        if (step_ok(s + 1)) tile_dot<F, NQ>(fb, xv, split * nbk + (s + 1) % nbk, acc, lane, tbl);
        if ((s + 1) % nbk == nbk - 1) epilogue(s + 1);
        if (s + 2 >= nsteps) break;
        if (step_ok(s + 4)) T::load(fb, tile_ptr(s + 4), lane);
        if (step_ok(s + 2)) tile_dot<F, NQ>(fc, xv, split * nbk + (s + 2) % nbk, acc, lane, tbl);
        if ((s + 2) % nbk == nbk - 1) epilogue(s + 2);
    }
    }
    if (KEYS) {
        // lanes 4g+t share token t: fold over g (lane bits 2..4), one atomic per warp and token
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) {
            unsigned long long k = best[qt];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const unsigned long long v = __shfl_xor_sync(0xffffffffu, k, o);
                k = v > k ? v : k;
            }
            const int tok = 4 * qt + (lane & 3);
            if (lane < 4 && tok < ntok && k) atomicMax(kout + tok, k);
        }
    }
}

// ===================================================== 16-bit weights ====
// FP16 / BF16 weight rows (qw6_tensor_dequantize_row, qw6.c:1686-1692): no
// blocks and no repacking -- the matrix stays row-major.  Dequantization is
// the exact widening (qw6_fp16_to_f32 with subnormals, Inf, NaN; bf16 << 16).
// The matvec is one warp per row: 16-byte loads of 8 weights, fp32 fma with
// each token's x (read through L1, shared by all rows of the CTA), a warp
// reduction; HBM-bound (weight bytes + x + y per launch).

template <bool BF>
__device__ __forceinline__ float w16(uint32_t h) {
    if constexpr (BF) return __uint_as_float(h << 16);
    else return f16_bits_exact(h);
}

template <bool BF>
__global__ void k_dequant16(const uint16_t* __restrict__ w, float* __restrict__ out, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = w16<BF>(w[i]);
}

template <bool BF, int NT>
__global__ void __launch_bounds__(256) k_matvec16(const uint16_t* __restrict__ w, const float* __restrict__ x,
                                                  float* __restrict__ y, int rows, int cols, int ntok, int ldx,
                                                  int ldy) {
    const int lane = threadIdx.x & 31;
    const int nw = gridDim.x * (blockDim.x >> 5);
    for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
        const uint16_t* wr = w + (size_t)r * cols;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = 0.f;
        for (int c = 8 * lane; c < cols; c += 256) {
            const uint4 v = ldg128(wr + c);
            float wv[8];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                wv[2 * i] = w16<BF>(u[i] & 0xffffu);
                wv[2 * i + 1] = w16<BF>(u[i] >> 16);
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < ntok) {
                    const float4 x0 = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * ldx + c));
                    const float4 x1 = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * ldx + c + 4));
                    float a = acc[t];
                    a = fmaf(wv[0], x0.x, a);
                    a = fmaf(wv[1], x0.y, a);
                    a = fmaf(wv[2], x0.z, a);
                    a = fmaf(wv[3], x0.w, a);
                    a = fmaf(wv[4], x1.x, a);
                    a = fmaf(wv[5], x1.y, a);
                    a = fmaf(wv[6], x1.z, a);
                    a = fmaf(wv[7], x1.w, a);
                    acc[t] = a;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            float a = acc[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0 && t < ntok) y[(size_t)t * ldy + r] = a;
        }
    }
}

template <bool BF>
static int launch_matvec16(const void* w, const float* x, float* y, int rows, int cols, int ntok, int ldx, int ldy,
                           cudaStream_t st) {
    const long long want = ((long long)rows + 7) / 8;
    const int grid = (int)(want < (long long)device_sms() * 8 ? want : (long long)device_sms() * 8);
    const uint16_t* wp = static_cast<const uint16_t*>(w);
    if (ntok == 1) k_matvec16<BF, 1><<<grid, 256, 0, st>>>(wp, x, y, rows, cols, ntok, ldx, ldy);
    else if (ntok <= 4) k_matvec16<BF, 4><<<grid, 256, 0, st>>>(wp, x, y, rows, cols, ntok, ldx, ldy);
    else if (ntok <= 8) k_matvec16<BF, 8><<<grid, 256, 0, st>>>(wp, x, y, rows, cols, ntok, ldx, ldy);
    else k_matvec16<BF, 32><<<grid, 256, 0, st>>>(wp, x, y, rows, cols, ntok, ldx, ldy);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

static bool is16(uint32_t q) { return q == QW6F_FP16 || q == QW6F_BF16; }

// ---------------------------------------------------------- launchers ----

static int num_sms() { return device_sms(); }

constexpr size_t kMvSmemMax = 200 * 1024;  // dynamic shared memory a matvec launch may use

template <int F, int NQ>
static size_t mv_smem(int cols) {
    return IQLut<F>::bytes + xstage_bytes(4 * NQ, cols) + (size_t)kThreads * 2 * NQ * 4;
}

template <int F, int NQ, bool KEYS>
static int launch_mv(const uint8_t* w, const float* x, float* y, int rows, int cols, int ntok, int ldx,
                     int ldy, cudaStream_t st, unsigned long long* keys = nullptr, uint32_t row_offset = 0,
                     int chunks = 1) {
    const size_t smem = mv_smem<F, NQ>(cols);
    if (smem > kMvSmemMax) return QW6K_ERR_ARG;
    static DevFlags configured;
    int occ = 1;
    if (smem_optin(configured, k_matvec<F, NQ, KEYS>, 200 * 1024)) return QW6K_ERR_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_matvec<F, NQ, KEYS>, kThreads, smem) != cudaSuccess ||
        occ < 1)
        return QW6K_ERR_CUDA;
    MvArgs a;
    a.keys = keys;
    a.row_offset = row_offset;
    a.w = w;
    a.x = x;
    a.y = y;
    a.rows = rows;
    a.cols = cols;
    a.ntok = ntok;
    a.ldx = ldx;
    a.ldy = ldy;
    a.nb = cols / 256;
    a.mtiles = (rows + 15) / 16;
    const int slots = num_sms() * occ * kWarps;  // resident warps
    int ks = 1;
    while (ks < 8 && a.nb % (ks * 2) == 0 && (long long)a.mtiles * ks < slots) ks *= 2;
    // The fused argmax keeps ks = 1: each row's logit is then summed block by
    // block in one warp, whatever the row count, so row shards of one
    // vocabulary give the same bits as the whole and combine exactly.
    if (KEYS) ks = 1;
    a.ks = ks;
    const int wpm = kWarps / ks;
    const long long ngrp = (a.mtiles + wpm - 1) / wpm;
    const int grid = (int)(ngrp < (long long)num_sms() * occ ? ngrp : (long long)num_sms() * occ);
    return launch_pdl(k_matvec<F, NQ, KEYS>, dim3(grid, chunks), dim3(kThreads), smem, st, a) == cudaSuccess
               ? 0
               : QW6K_ERR_CUDA;
}

// Token batches: 1-4 tokens in one launch.  A small matrix (<= 1024 tile-
// blocks, IQ formats <= 2048) with more tokens runs as chunks of 4 tokens side
// by side (grid y), up to 2048 tile-blocks the K formats as chunks of 16: the
// chunks read the same weights (from L2 after the first), and a CTA stages and
// multiplies only its chunk's tokens, so a small matrix at batch 32 fills the
// GPU instead of a few CTAs each staging all 32 tokens (measured on config 0 /
// 4's projections at batch 32: Q4_K 512x2048 28.6 -> 5.5 us, IQ3_S 2048^2 28.2
// -> 24.0, IQ2_S 2048x4096 58.1 -> 47.0, Q5_K 4096x2048 34.0 -> 32.0 with
// 16-token chunks).  Otherwise 5-8 tokens in one launch, 9-32 in one pass when
// the activation stage of 32 tokens fits in shared memory, else in passes of 16
// tokens (each pass streams the weights again; only very wide matrices, e.g.
// 4096 columns, need that).
template <int F, bool KEYS>
static int launch_mv_batch(const uint8_t* w, const float* x, float* y, int rows, int cols, int ntok, int ldx,
                           int ldy, cudaStream_t st, unsigned long long* keys, uint32_t row_offset) {
    if (ntok <= 4) return launch_mv<F, 1, KEYS>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset);
    const long long tbs = (long long)((rows + 15) / 16) * (cols / 256);  // tile-blocks
    if (ntok <= 32 && (tbs <= 1024 || (IsIQ<F>::value && tbs <= 2048)))
        return launch_mv<F, 1, KEYS>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset, (ntok + 3) / 4);
    if (ntok <= 32 && ntok > 8 && tbs <= 2048 && mv_smem<F, 4>(cols) <= kMvSmemMax)
        return launch_mv<F, 4, KEYS>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset, (ntok + 15) / 16);
    if (ntok <= 8) return launch_mv<F, 2, KEYS>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset);
    if (ntok > 32) return QW6K_ERR_ARG;
    if (mv_smem<F, 8>(cols) <= kMvSmemMax)
        return launch_mv<F, 8, KEYS>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset);
    for (int t0 = 0; t0 < ntok; t0 += 16) {
        const int n = ntok - t0 < 16 ? ntok - t0 : 16;
        const int rc = launch_mv<F, 4, KEYS>(w, x + (size_t)t0 * ldx, y ? y + (size_t)t0 * ldy : nullptr, rows, cols,
                                             n, ldx, ldy, st, keys ? keys + t0 : nullptr, row_offset);
        if (rc) return rc;
    }
    return 0;
}

template <int F>
static int launch_mv_nq(const uint8_t* w, const float* x, float* y, int rows, int cols, int ntok, int ldx,
                        int ldy, cudaStream_t st) {
    return launch_mv_batch<F, false>(w, x, y, rows, cols, ntok, ldx, ldy, st, nullptr, 0);
}

template <int F>
static int launch_mv_keys(const uint8_t* w, const float* x, float* y, int rows, int cols, int ntok, int ldx,
                          int ldy, unsigned long long* keys, uint32_t row_offset, cudaStream_t st) {
    return launch_mv_batch<F, true>(w, x, y, rows, cols, ntok, ldx, ldy, st, keys, row_offset);
}

template <int F>
static int launch_pack(const void* raw, void* packed, int rows, int cols, int nmat, size_t raw_stride,
                       size_t pk_stride, cudaStream_t st) {
    const int nb = cols / 256, mtiles = (rows + 15) / 16;
    dim3 grid((unsigned)(mtiles * nb), (unsigned)nmat);
    k_pack<F><<<grid, 256, 0, st>>>((const uint8_t*)raw, (uint8_t*)packed, rows, cols, raw_stride, pk_stride);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

template <int F>
static int launch_dequant(const void* raw, float* out, int rows, int cols, cudaStream_t st) {
    const long long total = (long long)rows * (cols / 256) * 8;
    const int threads = 128;
    const long long blocks = (total + threads - 1) / threads;
    if (blocks > 0x7fffffffLL) return QW6K_ERR_ARG;
    k_dequant<F><<<(unsigned)blocks, threads, 0, st>>>((const uint8_t*)raw, out, rows, cols);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

}  // namespace qw6

using namespace qw6;

#define QW6_DISPATCH_BLOCK(quant, CALL)             \
    switch (quant) {                                \
    case QW6F_Q4_K_M:                               \
    case QW6F_Q4_K_S: return CALL(QW6F_Q4_K_M);     \
    case QW6F_Q5_K: return CALL(QW6F_Q5_K);         \
    case QW6F_Q6_K: return CALL(QW6F_Q6_K);         \
    case QW6F_IQ2_XXS: return CALL(QW6F_IQ2_XXS);   \
    case QW6F_IQ2_S: return CALL(QW6F_IQ2_S);       \
    case QW6F_IQ3_S: return CALL(QW6F_IQ3_S);       \
    default: return QW6K_ERR_QUANT;                 \
    }

extern "C" size_t qw6k_tile_bytes(uint32_t quant) { return (size_t)16 * qw6_block_bytes(quant); }

extern "C" size_t qw6k_packed_bytes(uint32_t quant, uint32_t rows, uint32_t cols) {
    if (is16(quant)) return (rows && cols && cols % 8 == 0) ? (size_t)rows * cols * 2 : 0;  // row-major as stored
    if (!qw6_block_bytes(quant) || cols == 0 || cols % 256 || rows == 0) return 0;
    return (size_t)((rows + 15) / 16) * (cols / 256) * qw6k_tile_bytes(quant);
}

extern "C" int qw6k_pack(uint32_t quant, const void* raw, void* packed, uint32_t rows, uint32_t cols,
                         uint32_t nmat, size_t raw_stride, size_t packed_stride, cudaStream_t st) {
    if (is16(quant)) {  // no repacking: copy the rows of each matrix
        if (!raw || !packed || !rows || !cols || cols % 8 || !nmat) return QW6K_ERR_ARG;
        const size_t bytes = (size_t)rows * cols * 2;
        return cudaMemcpy2DAsync(packed, nmat > 1 ? packed_stride : bytes, raw, nmat > 1 ? raw_stride : bytes, bytes,
                                 nmat, cudaMemcpyDeviceToDevice, st) == cudaSuccess
                   ? 0
                   : QW6K_ERR_CUDA;
    }
    if (!raw || !packed || !rows || !cols || cols % 256 || !nmat || nmat > 65535) return QW6K_ERR_ARG;
#define CALL(F) launch_pack<F>(raw, packed, (int)rows, (int)cols, (int)nmat, raw_stride, packed_stride, st)
    QW6_DISPATCH_BLOCK(quant, CALL)
#undef CALL
}

extern "C" int qw6k_dequant(uint32_t quant, const void* raw, float* out, uint32_t rows, uint32_t cols,
                            cudaStream_t st) {
    if (is16(quant)) {
        if (!raw || !out || !rows || !cols) return QW6K_ERR_ARG;
        const long long n = (long long)rows * cols;
        const int grid = (int)((n + 255) / 256 < 65535 ? (n + 255) / 256 : 65535);
        if (quant == QW6F_FP16) k_dequant16<false><<<grid, 256, 0, st>>>((const uint16_t*)raw, out, n);
        else k_dequant16<true><<<grid, 256, 0, st>>>((const uint16_t*)raw, out, n);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
    }
    if (!raw || !out || !rows || !cols || cols % 256) return QW6K_ERR_ARG;
#define CALL(F) launch_dequant<F>(raw, out, (int)rows, (int)cols, st)
    QW6_DISPATCH_BLOCK(quant, CALL)
#undef CALL
}

// One row of a raw matrix, the row index read from device memory (the token
// id of an embedding lookup, qw6.c:2456): out[cols] = the exact dequantized
// row (qw6_tensor_dequantize_row, qw6.c:1674-1724).  An index past the
// matrix, or a NaN/Inf in the row (qw6.c:2457), sets *bad; the row is then
// zero-filled or written as is.
template <int F>
__global__ void k_dequant_row(const uint8_t* __restrict__ w, const uint32_t* __restrict__ row, float* __restrict__ out,
                              int* __restrict__ bad, uint32_t rows, int cols) {
    const uint32_t r = *row;
    const int nb = cols / 256;
    bool finite = true;
    for (int item = threadIdx.x; item < nb * 8; item += blockDim.x) {
        float* o = out + 32 * item;
        if (r >= rows) {
            for (int i = 0; i < 32; i++) o[i] = 0.f;
            continue;
        }
        dequant_group<F>(w + ((size_t)r * nb + (item >> 3)) * (size_t)Fmt<F>::BB, item & 7, o);
        for (int i = 0; i < 32; i++) finite = finite && isfinite(o[i]);
    }
    if ((r >= rows || !finite) && bad) atomicOr(bad, 1);
}

template <int BYTES>  // 4: fp32, 2: fp16 (BF = false) / bf16 (BF = true)
__global__ void k_dequant_row_plain(const uint8_t* __restrict__ w, const uint32_t* __restrict__ row,
                                    float* __restrict__ out, int* __restrict__ bad, uint32_t rows, int cols, bool bf) {
    const uint32_t r = *row;
    bool finite = true;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        float v = 0.f;
        if (r < rows) {
            if constexpr (BYTES == 4) v = reinterpret_cast<const float*>(w)[(size_t)r * cols + i];
            else {
                const uint32_t h = reinterpret_cast<const uint16_t*>(w)[(size_t)r * cols + i];
                v = bf ? w16<true>(h) : w16<false>(h);
            }
        }
        out[i] = v;
        finite = finite && isfinite(v);
    }
    if ((r >= rows || !finite) && bad) atomicOr(bad, 1);
}

template <int F>
static int launch_dequant_row(const void* raw, uint32_t rows, uint32_t cols, const uint32_t* row, float* out, int* bad,
                              cudaStream_t st) {
    k_dequant_row<F><<<1, 256, 0, st>>>((const uint8_t*)raw, row, out, bad, rows, (int)cols);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_dequant_row(uint32_t quant, const void* raw, uint32_t rows, uint32_t cols, const uint32_t* row,
                                float* out, int* bad, cudaStream_t st) {
    if (!raw || !row || !out || !rows || !cols) return QW6K_ERR_ARG;
    if (quant == QW6F_FP32 || is16(quant)) {
        if (quant == QW6F_FP32)
            k_dequant_row_plain<4><<<1, 256, 0, st>>>((const uint8_t*)raw, row, out, bad, rows, (int)cols, false);
        else
            k_dequant_row_plain<2><<<1, 256, 0, st>>>((const uint8_t*)raw, row, out, bad, rows, (int)cols,
                                                      quant == QW6F_BF16);
        return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
    }
    if (cols % 256) return QW6K_ERR_ARG;
#define CALL(F) launch_dequant_row<F>(raw, rows, cols, row, out, bad, st)
    QW6_DISPATCH_BLOCK(quant, CALL)
#undef CALL
}

extern "C" int qw6k_matvec(uint32_t quant, const void* packed, const float* x, float* y, uint32_t rows,
                           uint32_t cols, uint32_t ntok, uint32_t ldx, uint32_t ldy, cudaStream_t st) {
    if (is16(quant)) {
        if (!packed || !x || !y || !rows || !cols || cols % 8 || !ntok || ntok > 32 || ldx < cols || ldy < rows ||
            rows > (1u << 30))
            return QW6K_ERR_ARG;
        if ((reinterpret_cast<uintptr_t>(packed) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (ldx & 3u))
            return QW6K_ERR_ALIGN;
        return quant == QW6F_FP16 ? launch_matvec16<false>(packed, x, y, (int)rows, (int)cols, (int)ntok, (int)ldx,
                                                           (int)ldy, st)
                                  : launch_matvec16<true>(packed, x, y, (int)rows, (int)cols, (int)ntok, (int)ldx,
                                                          (int)ldy, st);
    }
    if (!packed || !x || !y || !rows || !cols || cols % 256 || !ntok || ntok > 32 || ldx < cols || ldy < rows ||
        rows > (1u << 30) || cols > 65536)
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(packed) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (ldx & 3u))
        return QW6K_ERR_ALIGN;
#define CALL(F) launch_mv_nq<F>((const uint8_t*)packed, x, y, (int)rows, (int)cols, (int)ntok, (int)ldx, (int)ldy, st)
    QW6_DISPATCH_BLOCK(quant, CALL)
#undef CALL
}

extern "C" int qw6k_matvec_argmax(uint32_t quant, const void* packed, const float* x, float* y,
                                  unsigned long long* keys, uint32_t rows, uint32_t cols, uint32_t ntok,
                                  uint32_t ldx, uint32_t ldy, uint32_t row_offset, cudaStream_t st) {
    if (!packed || !x || !keys || !rows || !cols || cols % 256 || !ntok || ntok > 32 || ldx < cols ||
        (y && ldy < rows) || rows > (1u << 30) || cols > 65536 || (uint64_t)row_offset + rows > 0xffffffffull)
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(packed) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (ldx & 3u))
        return QW6K_ERR_ALIGN;
    if (cudaMemsetAsync(keys, 0, (size_t)ntok * sizeof(unsigned long long), st) != cudaSuccess) return QW6K_ERR_CUDA;
#define CALL(F) launch_mv_keys<F>((const uint8_t*)packed, x, y, (int)rows, (int)cols, (int)ntok, (int)ldx, (int)ldy, keys, row_offset, st)
    QW6_DISPATCH_BLOCK(quant, CALL)
#undef CALL
}
