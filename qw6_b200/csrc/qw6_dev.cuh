// qw6_dev.cuh -- device-side core of libqw6cuda (sm_100a).
//
// Contents
//   * fp16 decoding (bit-exact with qw6_fp16_to_f32, qw6.c:1448-1471)
//   * IQ codebooks and sign-mask tables
//   * the PACKED TILE layout: a same-size byte permutation of the GGUF
//     super-blocks of 16 consecutive rows ("tile-block" = 16 rows x 256
//     columns) arranged so that every lane of a warp fetches exactly the
//     bytes of its mma.sync A-fragments with coalesced 16-byte loads
//   * per-format fragment decoders feeding int8 tensor-core MMAs
//     (mma.sync m16n8k32 / m16n8k16 .s8), with activations split into two
//     int8 limbs (hi*256 + lo, 15-bit fixed point per 256-block).
//
// Why this shape: a decode matvec moves each weight byte once, so HBM
// bandwidth is the roofline.  The blocks are 144/176/210/66/82/110 bytes --
// most not even 4-byte aligned -- so the raw layout cannot be read with
// wide coalesced loads.  Repacking once at upload (qw6's own pipeline also
// uploads weights once, qw6_vk.c:2920-2958) turns every weight load into an
// LDG.128 of contiguous lanes.  The GGUF weights are small integers (Q4_K
// 0..15, Q5_K 0..31, Q6_K -32..31, IQ grids +-8..43 / +-1..15) times per
// 16/32-weight integer scales, so they are exact in int8 and an int8 MMA
// with int32 accumulation is exact; the per-sub-block integer scales are
// applied with integer multiply-adds and the fp16 super-block scale once
// per block.  Rounding enters only through the 15-bit activation limbs
// (relative 1.5e-5 of the block maximum), far inside the 1e-3 budget.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "qw6_formats.h"
#include "qw6_iq_grids.h"

namespace qw6 {

constexpr int kWarps = 8;            // warps per CTA of the streaming kernels
constexpr int kThreads = kWarps * 32;

// ---------------------------------------------------------------- fp16 ----

// Exact IEEE half -> float including subnormals, Inf and NaN payloads; the
// same bit construction as qw6_fp16_to_f32 (qw6.c:1448-1471).
__device__ __forceinline__ float f16_bits_exact(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t out;
    if (e == 31u) {
        out = sign | 0x7f800000u | (m << 13);
    } else if (e == 0u) {
        if (m == 0u) {
            out = sign;
        } else {
            const int shift = __clz(m) - 21;  // bring the leading 1 to bit 10
            out = sign | ((uint32_t)(1 - shift + 112) << 23) | (((m << shift) & 1023u) << 13);
        }
    } else {
        out = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(out);
}

// Fast conversion for the matvec scales (value-exact for finite inputs).
__device__ __forceinline__ float f16f(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// ----------------------------------------------------------- loads -------

__device__ __forceinline__ uint4 ldg128(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg64(const void* p) {
    uint2 r;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg32(const void* p) {
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg16(const void* p) {
    unsigned short r;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t byte16(const uint4& v, int i) { return byte_of(word_of(v, i >> 2), i & 3); }

// ---------------------------------------------------------------- MMA ----

// D = A(16x32 s8, row) * B(32x8 s8, col) + C, int32.
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1, int c0, int c1,
                                        int c2, int c3) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}
// D = A(16x16 s8) * B(16x8 s8), int32.
__device__ __forceinline__ void mma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%7,%7,%7,%7};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// ------------------------------------------------------------ tables ----
//
// Codebooks are staged in shared memory as byte-SELECTOR tables for prmt:
// every IQ2 grid byte is one of {8, 25, 43} and every IQ3_S grid byte one of
// {1, 3, ..., 15}, so an entry is stored as one 4-bit selector per weight
// (IQ2: 8 weights -> 32 bits; IQ3_S: 4 weights -> 16 bits) and expanded by
// prmt against constant registers holding the value set.  Half the bytes of
// the raw codebook per lookup means fewer shared-memory bank conflicts.
//
// Signs.  IQ2 selectors use values 0..2 per nibble; with the second prmt
// source holding the negated values, bit 2 of a nibble selects the negative
// byte, so a sign pattern becomes an OR of a mask with bit 4j+2 set for every
// negative weight j: sgn[] maps the 7 stored sign bits of IQ2_XXS (the 8th is
// their parity) or the 8 sign bits of IQ2_S to that mask.  IQ3_S's eight
// values fill both prmt sources; its sgn[] maps 4 sign bits to the pair
// (xor mask 0xff, increment 0x01 per negative byte) of two's-complement
// negation.
constexpr uint32_t kIQ2Vals = 0x002b1908u;               // bytes {8, 25, 43}
constexpr uint32_t kIQ2Neg = 0x00d5e7f8u;                // bytes {-8, -25, -43}
constexpr uint32_t kIQ3Lo = 0x07050301u, kIQ3Hi = 0x0f0d0b09u;  // bytes {1..15 odd}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t nibble_bit2_mask(uint32_t s8) {
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) m |= ((s8 >> j) & 1u) << (4 * j + 2);
    return m;
}

template <int F>
struct IsIQ {
    static constexpr bool value = F == QW6F_IQ2_XXS || F == QW6F_IQ2_S || F == QW6F_IQ3_S;
};

// Layout in shared memory (32-bit words): the selector table, then the sign
// table.
//   IQ2_XXS: sel 256 entries; sgn 128 masks, indexed by the 7 stored sign bits
//   IQ2_S:   sel 1024 entries; sgn 256 masks
//   IQ3_S:   sel 512 16-bit selectors, one per word; sgn 16 (xor, inc) pairs
// (Per-lane copies of the tables, which make a warp's 32 random lookups one
// shared-memory wavefront, measured no faster on B200: the IQ kernels wait
// on instruction latency, not on bank conflicts.)
template <int F>
struct IQLut {
    static constexpr int kSel = F == QW6F_IQ2_S ? 1024 : F == QW6F_IQ3_S ? 512 : 256;
    static constexpr int kSgn = F == QW6F_IQ2_S ? 256 : F == QW6F_IQ3_S ? 32 : 128;  // words
    static constexpr size_t bytes = IsIQ<F>::value ? 4 * ((size_t)kSel + kSgn) : 0;

    __device__ __forceinline__ static uint32_t sel(const uint32_t* t, uint32_t e) { return t[e]; }
    __device__ __forceinline__ static uint32_t sgn(const uint32_t* t, uint32_t e) { return t[kSel + e]; }
    __device__ __forceinline__ static uint2 sgn2(const uint32_t* t, uint32_t p) {
        return reinterpret_cast<const uint2*>(t + kSel)[p];
    }

    // Build the tables from the raw grid bytes (all threads take part; the
    // caller synchronizes).
    __device__ static void init(uint32_t* t, const uint8_t* grid_g) {
        for (int e = threadIdx.x; e < kSel; e += blockDim.x) {
            uint32_t v = 0;
            if constexpr (F == QW6F_IQ3_S) {
#pragma unroll
                for (int j = 0; j < 4; j++) v |= ((uint32_t)(grid_g[4 * e + j] >> 1)) << (4 * j);
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const uint32_t b = grid_g[8 * e + j];
                    v |= (b == 8u ? 0u : b == 25u ? 1u : 2u) << (4 * j);
                }
            }
            t[e] = v;
        }
        if constexpr (F == QW6F_IQ3_S) {
            for (int n = threadIdx.x; n < 16; n += blockDim.x) {
                uint32_t m = 0, inc = 0;
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if ((n >> j) & 1) {
                        m |= 0xffu << (8 * j);
                        inc |= 1u << (8 * j);
                    }
                reinterpret_cast<uint2*>(t + kSel)[n] = make_uint2(m, inc);
            }
        } else {
            for (int i = threadIdx.x; i < kSgn; i += blockDim.x)
                t[kSel + i] = nibble_bit2_mask(F == QW6F_IQ2_XXS ? i | ((__popc(i) & 1u) << 7) : i);
        }
    }
};

// --------------------------------------------------- packed tile layout ---
//
// Tile-block = rows [16i, 16i+16) x super-block column b; TB = 16*block bytes.
// Tile-blocks are stored m-tile-major: offset ((i*nb + b) * TB).  Within a
// tile-block, lane = 4*g + t of a warp handles rows g and g+8 ("rh" = 0/1)
// and, inside every 32-weight sub-block, the 8 weights [8t, 8t+8) (IQ2_S:
// 4 weights of each 16-half).  pack_dst(F, r, p) is the destination of raw
// byte p of row r's block; it is a bijection onto [0, TB).

template <int F>
struct Fmt;

template <>
struct Fmt<QW6F_Q4_K_M> {
    static constexpr int BB = 144, TB = 16 * BB;
    // [0,256)   row headers {d, dmin, scales[12]}, 16 B per row
    // [256,...) 4 chunks x 32 lanes x 16 B: chunk rh*2+c/2 holds, for row
    //           g+8rh, qs[32c+8t .. +8] (c even: bytes 0-7, c odd: 8-15)
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        if (p < 16) return r * 16 + p;
        const uint32_t q = p - 16, c = q / 32, l = q % 32, t = l / 8, o = l % 8;
        const uint32_t lane = (r % 8) * 4 + t, k = (r / 8) * 2 + c / 2;
        return 256 + (k * 32 + lane) * 16 + (c % 2) * 8 + o;
    }
};
template <>
struct Fmt<QW6F_Q4_K_S> : Fmt<QW6F_Q4_K_M> {};

template <>
struct Fmt<QW6F_Q5_K> {
    static constexpr int BB = 176, TB = 16 * BB;
    // headers as Q4_K; chunks 0-3 = qs as Q4_K; chunk 4 = qh[8t..+8] of
    // rows g (bytes 0-7) and g+8 (bytes 8-15)
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        if (p < 16) return r * 16 + p;
        const uint32_t lanebase = (r % 8) * 4;
        if (p < 48) {
            const uint32_t l = p - 16, t = l / 8, o = l % 8;
            return 256 + (4 * 32 + lanebase + t) * 16 + (r / 8) * 8 + o;
        }
        const uint32_t q = p - 48, c = q / 32, l = q % 32, t = l / 8, o = l % 8;
        const uint32_t k = (r / 8) * 2 + c / 2;
        return 256 + (k * 32 + lanebase + t) * 16 + (c % 2) * 8 + o;
    }
};

template <>
struct Fmt<QW6F_Q6_K> {
    static constexpr int BB = 210, TB = 16 * BB;
    // [0,256) int8 scales[16] per row; [256,288) d per row;
    // [288,...) 6 chunks: chunk rh*3+n = {ql[64n+8t..+8], ql[64n+32+8t..+8]},
    //                     chunk rh*3+2 = {qh[8t..+8], qh[32+8t..+8]}
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        const uint32_t lanebase = (r % 8) * 4, rh = r / 8;
        if (p >= 208) return 256 + r * 2 + (p - 208);
        if (p >= 192) return r * 16 + (p - 192);
        if (p < 128) {
            const uint32_t n = p / 64, q = p % 64, which = q / 32, l = q % 32, t = l / 8, o = l % 8;
            return 288 + ((rh * 3 + n) * 32 + lanebase + t) * 16 + which * 8 + o;
        }
        const uint32_t q = p - 128, n = q / 32, l = q % 32, t = l / 8, o = l % 8;
        return 288 + ((rh * 3 + 2) * 32 + lanebase + t) * 16 + n * 8 + o;
    }
};

template <>
struct Fmt<QW6F_IQ2_XXS> {
    static constexpr int BB = 66, TB = 16 * BB;
    // [0,32) d per row; [32,544) the 8 aux words per row (32 B per row);
    // [544,1056) per lane 16 B: grid index of entry t for groups 0..7 of
    //            row g (bytes 0-7) and row g+8 (bytes 8-15)
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        if (p < 2) return r * 2 + p;
        const uint32_t q = p - 2, grp = q / 8, w = q % 8;
        if (w >= 4) return 32 + r * 32 + grp * 4 + (w - 4);
        return 544 + ((r % 8) * 4 + w) * 16 + (r / 8) * 8 + grp;
    }
};

template <>
struct Fmt<QW6F_IQ2_S> {
    static constexpr int BB = 82, TB = 16 * BB;
    // [0,32) d per row; [32,288) {qh[8], scales[8]} per row;
    // [288,1312) per row and lane pair p = t/2 (32 B): grid-index low bytes
    //            of entries l = p and l = 2+p of groups 0..7 ([grp][hi]),
    //            then their sign bytes in the same order
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        if (p < 2) return r * 2 + p;
        if (p >= 66) return 32 + r * 16 + (p - 66);
        const uint32_t sgn = p >= 34, q = p - (sgn ? 34 : 2), grp = q / 4, l = q % 4;
        const uint32_t pair = l % 2, hi = l / 2;
        return 288 + (r * 2 + pair) * 32 + sgn * 16 + grp * 2 + hi;
    }
};

template <>
struct Fmt<QW6F_IQ3_S> {
    static constexpr int BB = 110, TB = 16 * BB;
    // [0,32) d; [32,160) qh[8] per row; [160,224) scales[4] per row;
    // [224,...) chunk rh: per lane qs[8grp+2t], qs[8grp+2t+1] for grp 0..7 of
    //           row g+8rh; chunk 2: signs[4grp+t] of row g (0-7), g+8 (8-15)
    __host__ __device__ static uint32_t dst(uint32_t r, uint32_t p) {
        const uint32_t lane_r = (r % 8) * 4, rh = r / 8;
        if (p < 2) return r * 2 + p;
        if (p >= 106) return 160 + r * 4 + (p - 106);
        if (p >= 66 && p < 74) return 32 + r * 8 + (p - 66);
        if (p < 66) {
            const uint32_t q = p - 2, grp = q / 8, w = q % 8, t = w / 2, which = w % 2;
            return 224 + (rh * 32 + lane_r + t) * 16 + grp * 2 + which;
        }
        const uint32_t q = p - 74, grp = q / 4, t = q % 4;
        return 224 + (2 * 32 + lane_r + t) * 16 + rh * 8 + grp;
    }
};

// ------------------------------------------------- staged activations ---
//
// Activations are staged per CTA in shared memory as two int8 limbs:
// for token tok and 256-block b, s = amax/32639, X = rint(x/s),
// H = (X+128) >> 8, L = X - 256 H (both in [-128, 127]), x ~= s*(256H+L).
// MMA column n of n-tile q is token 4q + n/2, limb n%2, so C columns
// (2t, 2t+1) of lane t carry the two limbs of token 4q+t.
// The per-token rows of sx, xsum and nx32 are padded (xs_sx_ld etc.): the
// four lanes t of a quad read four tokens' entries of the same block at
// once, and unpadded rows of 2^k bytes would put them in one bank.
__host__ __device__ constexpr int xs_sx_ld(int nb) { return nb + 1; }   // floats
__host__ __device__ constexpr int xs_sum_ld(int ns) { return ns + 4; }  // floats (float4 reads)
__host__ __device__ constexpr int xs_nx_ld(int ns) { return ns + 1; }   // int2
struct XView {
    const int8_t* q;    // [ntp][2][stride]
    const float* sx;    // [ntp][xs_sx_ld(nb)]
    const float* xsum;  // [ntp][xs_sum_ld(ns)]  fp32 sum of each 32-sub-block (K formats)
    const int2* nx32;   // [ntp][xs_nx_ld(ns)]   (-32*sum H, -32*sum L) per sub-block (Q6_K)
    int stride, nb, ns;

    __device__ __forceinline__ uint2 b64(int qt, int j, int lane) const {
        const int g = lane >> 2, t = lane & 3;
        return *reinterpret_cast<const uint2*>(q + ((qt * 4 + (g >> 1)) * 2 + (g & 1)) * stride + 32 * j + 8 * t);
    }
    __device__ __forceinline__ uint32_t b32(int qt, int col, int lane) const {
        const int g = lane >> 2, t = lane & 3;
        return *reinterpret_cast<const uint32_t*>(q + ((qt * 4 + (g >> 1)) * 2 + (g & 1)) * stride + col + 4 * t);
    }
};

// Shared-memory bytes for staging ntp tokens of `cols` columns.
__host__ __device__ inline int xstage_stride(int cols) { return cols + 32; }
__host__ __device__ inline size_t xstage_bytes(int ntp, int cols) {
    const int nb = cols / 256, ns = cols / 32;
    return (size_t)ntp * 2 * xstage_stride(cols) + (size_t)ntp * xs_sx_ld(nb) * 4 +
           (size_t)ntp * xs_sum_ld(ns) * 4 + (size_t)ntp * xs_nx_ld(ns) * 8;
}

struct XStage {
    int8_t* q;
    float* sx;
    float* xsum;
    int2* nx32;
    int stride, nb, ns;
    __device__ XView view() const { return XView{q, sx, xsum, nx32, stride, nb, ns}; }
};

__device__ __forceinline__ XStage xstage_carve(uint8_t* base, int ntp, int cols) {
    XStage s;
    s.stride = xstage_stride(cols);
    s.nb = cols / 256;
    s.ns = cols / 32;
    s.q = reinterpret_cast<int8_t*>(base);
    uint8_t* p = base + (size_t)ntp * 2 * s.stride;
    s.nx32 = reinterpret_cast<int2*>(p);
    p += (size_t)ntp * xs_nx_ld(s.ns) * 8;
    s.xsum = reinterpret_cast<float*>(p);  // 16-byte aligned for its float4 reads (ntp is a multiple of 4)
    p += (size_t)ntp * xs_sum_ld(s.ns) * 4;
    s.sx = reinterpret_cast<float*>(p);
    return s;
}

__device__ __forceinline__ void xstage_fill_warps(const XStage& s, const float* x, int ldx, int ntok, int ntp,
                                                  int cols, const int32_t* rowsel, int rowdiv, int first_warp,
                                                  int nwarps);

// Quantize ntok token rows of x (row stride ldx floats) into the stage;
// tokens [ntok, ntp) are zero.  Stage row j reads x row j, or row
// rowsel[j] / rowdiv when rowsel is given (gather through an index list; a
// negative entry stages a zero row).
// One warp per (token, 256-block); all threads of the CTA must call it
// (caller synchronizes afterwards).
__device__ __forceinline__ void xstage_fill(const XStage& s, const float* x, int ldx,
                                            int ntok, int ntp, int cols, const int32_t* rowsel = nullptr,
                                            int rowdiv = 1) {
    xstage_fill_warps(s, x, ldx, ntok, ntp, cols, rowsel, rowdiv, threadIdx.x >> 5, blockDim.x >> 5);
}

// Same, executed by warps first_warp, first_warp + nwarps, ... only (no
// block-wide synchronization inside; a single warp may stage on its own).
__device__ __forceinline__ void xstage_fill_warps(const XStage& s, const float* x, int ldx, int ntok, int ntp,
                                                  int cols, const int32_t* rowsel, int rowdiv, int first_warp,
                                                  int nwarps) {
    const int warp = first_warp, lane = threadIdx.x & 31, nw = nwarps;
    const int nb = cols / 256;
    for (int item = warp; item < ntp * nb; item += nw) {
        const int tok = item / nb, b = item % nb;
        float v[8];
        const int sel = (tok < ntok) ? (rowsel ? rowsel[tok] : tok) : -1;
        if (sel < 0) {  // zero row: warp-uniform fast path
            *reinterpret_cast<uint2*>(s.q + (tok * 2 + 0) * s.stride + 256 * b + 8 * lane) = make_uint2(0u, 0u);
            *reinterpret_cast<uint2*>(s.q + (tok * 2 + 1) * s.stride + 256 * b + 8 * lane) = make_uint2(0u, 0u);
            if ((lane & 3) == 0) {
                const int j = 8 * b + (lane >> 2);
                s.xsum[tok * xs_sum_ld(s.ns) + j] = 0.f;
                s.nx32[tok * xs_nx_ld(s.ns) + j] = make_int2(0, 0);
            }
            if (lane == 0) s.sx[tok * xs_sx_ld(nb) + b] = 0.f;
            continue;
        }
        if (sel >= 0) {
            const int srow = rowsel ? sel / rowdiv : sel;
            const float4* src = reinterpret_cast<const float4*>(x + (size_t)srow * ldx + 256 * b + 8 * lane);
            const float4 u0 = src[0], u1 = src[1];
            v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
            v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = 0.f;
        }
        float amax = 0.f, sum = 0.f;
        bool finite = true;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            amax = fmaxf(amax, fabsf(v[i]));
            sum += v[i];
            finite = finite && isfinite(v[i]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        // a NaN or Inf in the block makes the block's scale NaN, so that it
        // reaches the outputs as in qw6's fp32 dot products
        if (!__all_sync(0xffffffffu, finite)) amax = __int_as_float(0x7fc00000);
        const float inv = amax > 0.f ? 32639.f / amax : 0.f;  // 0 for a NaN scale
        uint32_t hw[2] = {0, 0}, lw[2] = {0, 0};
        int sh = 0, sl = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int X = __float2int_rn(v[i] * inv);
            X = max(-32639, min(32639, X));
            const int H = (X + 128) >> 8, L = X - (H << 8);
            sh += H;
            sl += L;
            hw[i >> 2] |= (uint32_t)(H & 0xff) << (8 * (i & 3));
            lw[i >> 2] |= (uint32_t)(L & 0xff) << (8 * (i & 3));
        }
        *reinterpret_cast<uint2*>(s.q + (tok * 2 + 0) * s.stride + 256 * b + 8 * lane) = make_uint2(hw[0], hw[1]);
        *reinterpret_cast<uint2*>(s.q + (tok * 2 + 1) * s.stride + 256 * b + 8 * lane) = make_uint2(lw[0], lw[1]);
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            sh += __shfl_xor_sync(0xffffffffu, sh, o);
            sl += __shfl_xor_sync(0xffffffffu, sl, o);
        }
        if ((lane & 3) == 0) {
            const int j = 8 * b + (lane >> 2);
            s.xsum[tok * xs_sum_ld(s.ns) + j] = sum;
            s.nx32[tok * xs_nx_ld(s.ns) + j] = make_int2(-32 * sh, -32 * sl);
        }
        if (lane == 0) s.sx[tok * xs_sx_ld(nb) + b] = (amax > 0.f || amax != amax) ? amax / 32639.f : 0.f;
    }
}

// ------------------------------------------- programmatic dependent launch -
// A kernel launched with the programmatic-serialization attribute may start
// while its predecessor in the stream still runs; pdl_wait() blocks until
// the predecessor grid has completed and its writes are visible (a no-op when
// launched normally).  pdl_trigger() lets the successor start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------ per-format decoders ---
//
// Frag<F> holds one lane's share of one tile-block; load() issues its
// global loads, dot() consumes it and adds the block's contribution to
// acc[rh][q] (row g+8rh, token 4q+t).

template <int F, int NQ>
struct Tile;

template <int NQ>
__device__ __forceinline__ void finish_block(float (&acc)[2][NQ], const int (&iH)[2][NQ],
                                             const int (&iL)[2][NQ], const float (&dfac)[2],
                                             const XView& xv, int b, int lane) {
    const int t = lane & 3;
#pragma unroll
    for (int qt = 0; qt < NQ; qt++) {
        const float s = xv.sx[(4 * qt + t) * xs_sx_ld(xv.nb) + b];
#pragma unroll
        for (int rh = 0; rh < 2; rh++)
            acc[rh][qt] += dfac[rh] * s * fmaf(256.f, (float)iH[rh][qt], (float)iL[rh][qt]);
    }
}

// ---- Q4_K / Q5_K (shared scale handling) ----
template <int NQ, bool Q5>
struct TileK45 {
    static constexpr int NCH = Q5 ? 5 : 4;
    static constexpr int TB = Q5 ? Fmt<QW6F_Q5_K>::TB : Fmt<QW6F_Q4_K_M>::TB;
    struct Frag {
        uint4 q[NCH];
        uint4 h[2];
    };
    __device__ __forceinline__ static void load(Frag& f, const uint8_t* tb, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int k = 0; k < NCH; k++) f.q[k] = ldg128(tb + 256 + (k * 32 + lane) * 16);
        f.h[0] = ldg128(tb + g * 16);
        f.h[1] = ldg128(tb + (g + 8) * 16);
    }
    __device__ __forceinline__ static void dot(const Frag& f, const XView& xv, int b, float (&acc)[2][NQ],
                                               int lane) {
        const int t = lane & 3;
        uint32_t SC[2][2], MN[2][2];
        float dfac[2], dmin[2];
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            dfac[rh] = f16f(f.h[rh].x);
            dmin[rh] = f16f(f.h[rh].x >> 16);
            const uint32_t S0 = f.h[rh].y, S1 = f.h[rh].z, S2 = f.h[rh].w;
            SC[rh][0] = S0 & 0x3f3f3f3fu;
            MN[rh][0] = S1 & 0x3f3f3f3fu;
            SC[rh][1] = (S2 & 0x0f0f0f0fu) | ((S0 >> 2) & 0x30303030u);
            MN[rh][1] = ((S2 >> 4) & 0x0f0f0f0fu) | ((S1 >> 2) & 0x30303030u);
        }
        int iH[2][NQ], iL[2][NQ];
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) iH[0][qt] = iH[1][qt] = iL[0][qt] = iL[1][qt] = 0;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint32_t w0 = (c & 1) ? f.q[c >> 1].z : f.q[c >> 1].x;
            const uint32_t w1 = (c & 1) ? f.q[c >> 1].w : f.q[c >> 1].y;
            const uint32_t v0 = (c & 1) ? f.q[2 + (c >> 1)].z : f.q[2 + (c >> 1)].x;
            const uint32_t v1 = (c & 1) ? f.q[2 + (c >> 1)].w : f.q[2 + (c >> 1)].y;
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int j = 2 * c + hh;
                uint32_t a0 = (w0 >> (4 * hh)) & 0x0f0f0f0fu, a2 = (w1 >> (4 * hh)) & 0x0f0f0f0fu;
                uint32_t a1 = (v0 >> (4 * hh)) & 0x0f0f0f0fu, a3 = (v1 >> (4 * hh)) & 0x0f0f0f0fu;
                if (Q5) {
                    const uint4 qh = f.q[4];
                    a0 |= ((qh.x >> j) << 4) & 0x10101010u;
                    a2 |= ((qh.y >> j) << 4) & 0x10101010u;
                    a1 |= ((qh.z >> j) << 4) & 0x10101010u;
                    a3 |= ((qh.w >> j) << 4) & 0x10101010u;
                }
                const int s0 = (int)byte_of(SC[0][j >> 2], j & 3), s1 = (int)byte_of(SC[1][j >> 2], j & 3);
#pragma unroll
                for (int qt = 0; qt < NQ; qt++) {
                    const uint2 bb = xv.b64(qt, 8 * b + j, lane);
                    int d[4];
                    mma_k32(d, a0, a1, a2, a3, bb.x, bb.y, 0, 0, 0, 0);
                    iH[0][qt] += s0 * d[0];
                    iL[0][qt] += s0 * d[1];
                    iH[1][qt] += s1 * d[2];
                    iL[1][qt] += s1 * d[3];
                }
            }
        }
        finish_block<NQ>(acc, iH, iL, dfac, xv, b, lane);
        // minimum term: - dmin * sum_j m_j * xsum_j
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) {
            const float* xs = xv.xsum + (4 * qt + t) * xs_sum_ld(xv.ns) + 8 * b;
            const float4 x0 = *reinterpret_cast<const float4*>(xs);
            const float4 x1 = *reinterpret_cast<const float4*>(xs + 4);
#pragma unroll
            for (int rh = 0; rh < 2; rh++) {
                const uint32_t m0 = MN[rh][0], m1 = MN[rh][1];
                float mt = (float)byte_of(m0, 0) * x0.x;
                mt = fmaf((float)byte_of(m0, 1), x0.y, mt);
                mt = fmaf((float)byte_of(m0, 2), x0.z, mt);
                mt = fmaf((float)byte_of(m0, 3), x0.w, mt);
                mt = fmaf((float)byte_of(m1, 0), x1.x, mt);
                mt = fmaf((float)byte_of(m1, 1), x1.y, mt);
                mt = fmaf((float)byte_of(m1, 2), x1.z, mt);
                mt = fmaf((float)byte_of(m1, 3), x1.w, mt);
                acc[rh][qt] -= dmin[rh] * mt;
            }
        }
    }
};

template <int NQ>
struct Tile<QW6F_Q4_K_M, NQ> : TileK45<NQ, false> {};
template <int NQ>
struct Tile<QW6F_Q4_K_S, NQ> : TileK45<NQ, false> {};
template <int NQ>
struct Tile<QW6F_Q5_K, NQ> : TileK45<NQ, true> {};

// ---- Q6_K ----
template <int NQ>
struct Tile<QW6F_Q6_K, NQ> {
    static constexpr int TB = Fmt<QW6F_Q6_K>::TB;
    struct Frag {
        uint4 q[6];
        uint4 sc[2];
        uint32_t d[2];
    };
    __device__ __forceinline__ static void load(Frag& f, const uint8_t* tb, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int k = 0; k < 6; k++) f.q[k] = ldg128(tb + 288 + (k * 32 + lane) * 16);
        f.sc[0] = ldg128(tb + g * 16);
        f.sc[1] = ldg128(tb + (g + 8) * 16);
        f.d[0] = ldg16(tb + 256 + g * 2);
        f.d[1] = ldg16(tb + 256 + (g + 8) * 2);
    }
    __device__ __forceinline__ static void dot(const Frag& f, const XView& xv, int b, float (&acc)[2][NQ],
                                               int lane) {
        const int t = lane & 3;
        float dfac[2] = {f16f(f.d[0]), f16f(f.d[1])};
        int iH[2][NQ], iL[2][NQ];
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) iH[0][qt] = iH[1][qt] = iL[0][qt] = iL[1][qt] = 0;
#pragma unroll
        for (int n = 0; n < 2; n++) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const int j = 4 * n + kk;
                uint32_t a[2][2];
#pragma unroll
                for (int rh = 0; rh < 2; rh++) {
                    const uint4 L = f.q[rh * 3 + n], Hq = f.q[rh * 3 + 2];
                    const uint32_t h0 = n ? Hq.z : Hq.x, h1 = n ? Hq.w : Hq.y;
#pragma unroll
                    for (int hw = 0; hw < 2; hw++) {
                        const uint32_t A = hw ? L.y : L.x, B = hw ? L.w : L.z, H = hw ? h1 : h0;
                        uint32_t lo, hi;
                        if (kk == 0) { lo = A & 0x0f0f0f0fu; hi = (H << 4) & 0x30303030u; }
                        else if (kk == 1) { lo = B & 0x0f0f0f0fu; hi = (H << 2) & 0x30303030u; }
                        else if (kk == 2) { lo = (A >> 4) & 0x0f0f0f0fu; hi = H & 0x30303030u; }
                        else { lo = (B >> 4) & 0x0f0f0f0fu; hi = (H >> 2) & 0x30303030u; }
                        a[rh][hw] = lo | hi;
                    }
                }
                // qw6 reads only the even scales: sc[8n + 2kk] (qw6.c:1568-1571)
                const int si = 8 * n + 2 * kk;
                const int s0 = (int)(int8_t)byte16(f.sc[0], si), s1 = (int)(int8_t)byte16(f.sc[1], si);
#pragma unroll
                for (int qt = 0; qt < NQ; qt++) {
                    const uint2 bb = xv.b64(qt, 8 * b + j, lane);
                    const int2 nx = xv.nx32[(4 * qt + t) * xs_nx_ld(xv.ns) + 8 * b + j];
                    int d[4];
                    mma_k32(d, a[0][0], a[1][0], a[0][1], a[1][1], bb.x, bb.y, nx.x, nx.y, nx.x, nx.y);
                    iH[0][qt] += s0 * d[0];
                    iL[0][qt] += s0 * d[1];
                    iH[1][qt] += s1 * d[2];
                    iL[1][qt] += s1 * d[3];
                }
            }
        }
        finish_block<NQ>(acc, iH, iL, dfac, xv, b, lane);
    }
};

// ---- IQ2_XXS ----
template <int NQ>
struct Tile<QW6F_IQ2_XXS, NQ> {
    static constexpr int TB = Fmt<QW6F_IQ2_XXS>::TB;
    struct Frag {
        uint4 idx;
        uint4 aux[2][2];
        uint32_t d[2];
    };
    __device__ __forceinline__ static void load(Frag& f, const uint8_t* tb, int lane) {
        const int g = lane >> 2;
        f.idx = ldg128(tb + 544 + lane * 16);
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            f.aux[rh][0] = ldg128(tb + 32 + (g + 8 * rh) * 32);
            f.aux[rh][1] = ldg128(tb + 32 + (g + 8 * rh) * 32 + 16);
            f.d[rh] = ldg16(tb + (g + 8 * rh) * 2);
        }
    }
    __device__ __forceinline__ static void dot(const Frag& f, const XView& xv, int b, float (&acc)[2][NQ],
                                               int lane, const uint32_t* tbl) {
        const int t = lane & 3;
        float dfac[2] = {f16f(f.d[0]) * 0.125f, f16f(f.d[1]) * 0.125f};
        int iH[2][NQ], iL[2][NQ];
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) iH[0][qt] = iH[1][qt] = iL[0][qt] = iL[1][qt] = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t lo[2], hi[2];
            int scl[2];
#pragma unroll
            for (int rh = 0; rh < 2; rh++) {
                const uint32_t iw = rh ? (j < 4 ? f.idx.z : f.idx.w) : (j < 4 ? f.idx.x : f.idx.y);
                const uint32_t gi = byte_of(iw, j & 3);
                const uint32_t aw = word_of(f.aux[rh][j >> 2], j & 3);
                const uint32_t sf = (aw >> (7 * t)) & 127u;  // signs of qw6_ksigns(sf) via sgn[]
                scl[rh] = 2 * (int)(aw >> 28) + 1;
                const uint32_t ss = IQLut<QW6F_IQ2_XXS>::sel(tbl, gi) | IQLut<QW6F_IQ2_XXS>::sgn(tbl, sf);
                lo[rh] = prmt(kIQ2Vals, kIQ2Neg, ss);
                hi[rh] = prmt(kIQ2Vals, kIQ2Neg, ss >> 16);
            }
#pragma unroll
            for (int qt = 0; qt < NQ; qt++) {
                const uint2 bb = xv.b64(qt, 8 * b + j, lane);
                int d[4];
                mma_k32(d, lo[0], lo[1], hi[0], hi[1], bb.x, bb.y, 0, 0, 0, 0);
                iH[0][qt] += scl[0] * d[0];
                iL[0][qt] += scl[0] * d[1];
                iH[1][qt] += scl[1] * d[2];
                iL[1][qt] += scl[1] * d[3];
            }
        }
        finish_block<NQ>(acc, iH, iL, dfac, xv, b, lane);
    }
};

// ---- IQ2_S (16-weight scales -> k16 MMAs) ----
template <int NQ>
struct Tile<QW6F_IQ2_S, NQ> {
    static constexpr int TB = Fmt<QW6F_IQ2_S>::TB;
    struct Frag {
        uint4 P[2][2];  // [rh][idx|signs]
        uint4 sh[2];    // [rh] {qh 8 B, scales 8 B}
        uint32_t d[2];
    };
    __device__ __forceinline__ static void load(Frag& f, const uint8_t* tb, int lane) {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            const uint8_t* pp = tb + 288 + ((g + 8 * rh) * 2 + (t >> 1)) * 32;
            f.P[rh][0] = ldg128(pp);
            f.P[rh][1] = ldg128(pp + 16);
            f.sh[rh] = ldg128(tb + 32 + (g + 8 * rh) * 16);
            f.d[rh] = ldg16(tb + (g + 8 * rh) * 2);
        }
    }
    __device__ __forceinline__ static void dot(const Frag& f, const XView& xv, int b, float (&acc)[2][NQ],
                                               int lane, const uint32_t* tbl) {
        const int t = lane & 3, pr = t >> 1, half4 = 4 * (t & 1);
        float dfac[2] = {f16f(f.d[0]) * 0.125f, f16f(f.d[1]) * 0.125f};
        int iH[2][NQ], iL[2][NQ];
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) iH[0][qt] = iH[1][qt] = iL[0][qt] = iL[1][qt] = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int l = 2 * hh + pr;
                uint32_t a[2];
                int scl[2];
#pragma unroll
                for (int rh = 0; rh < 2; rh++) {
                    const uint32_t ib = byte16(f.P[rh][0], 2 * j + hh);
                    const uint32_t qhb = byte_of(j < 4 ? f.sh[rh].x : f.sh[rh].y, j & 3);
                    const uint32_t gi = ib | (((qhb >> (2 * l)) & 3u) << 8);
                    const uint32_t sb = byte16(f.P[rh][1], 2 * j + hh);
                    a[rh] = prmt(kIQ2Vals, kIQ2Neg,
                                 (IQLut<QW6F_IQ2_S>::sel(tbl, gi) | IQLut<QW6F_IQ2_S>::sgn(tbl, sb)) >>
                                     (4 * half4));
                    const uint32_t scb = byte_of(j < 4 ? f.sh[rh].z : f.sh[rh].w, j & 3);
                    scl[rh] = 2 * (int)((scb >> (4 * hh)) & 15u) + 1;
                }
#pragma unroll
                for (int qt = 0; qt < NQ; qt++) {
                    const uint32_t bb = xv.b32(qt, 256 * b + 32 * j + 16 * hh, lane);
                    int d[4];
                    mma_k16(d, a[0], a[1], bb);
                    iH[0][qt] += scl[0] * d[0];
                    iL[0][qt] += scl[0] * d[1];
                    iH[1][qt] += scl[1] * d[2];
                    iL[1][qt] += scl[1] * d[3];
                }
            }
        }
        finish_block<NQ>(acc, iH, iL, dfac, xv, b, lane);
    }
};

// ---- IQ3_S ----
template <int NQ>
struct Tile<QW6F_IQ3_S, NQ> {
    static constexpr int TB = Fmt<QW6F_IQ3_S>::TB;
    struct Frag {
        uint4 c[3];
        uint2 qh[2];
        uint32_t sc[2];
        uint32_t d[2];
    };
    __device__ __forceinline__ static void load(Frag& f, const uint8_t* tb, int lane) {
        const int g = lane >> 2;
#pragma unroll
        for (int k = 0; k < 3; k++) f.c[k] = ldg128(tb + 224 + (k * 32 + lane) * 16);
#pragma unroll
        for (int rh = 0; rh < 2; rh++) {
            f.qh[rh] = ldg64(tb + 32 + (g + 8 * rh) * 8);
            f.sc[rh] = ldg32(tb + 160 + (g + 8 * rh) * 4);
            f.d[rh] = ldg16(tb + (g + 8 * rh) * 2);
        }
    }
    __device__ __forceinline__ static void dot(const Frag& f, const XView& xv, int b, float (&acc)[2][NQ],
                                               int lane, const uint32_t* tbl) {
        const int t = lane & 3;
        float dfac[2] = {f16f(f.d[0]), f16f(f.d[1])};
        int iH[2][NQ], iL[2][NQ];
#pragma unroll
        for (int qt = 0; qt < NQ; qt++) iH[0][qt] = iH[1][qt] = iL[0][qt] = iL[1][qt] = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t lo[2], hi[2];
            int scl[2];
#pragma unroll
            for (int rh = 0; rh < 2; rh++) {
                const uint32_t i1 = byte16(f.c[rh], 2 * j), i2 = byte16(f.c[rh], 2 * j + 1);
                const uint32_t qhb = byte_of(j < 4 ? f.qh[rh].x : f.qh[rh].y, j & 3);
                const uint32_t g1 = i1 | (((qhb >> (2 * t)) & 1u) << 8);
                const uint32_t g2 = i2 | (((qhb >> (2 * t + 1)) & 1u) << 8);
                using Lut = IQLut<QW6F_IQ3_S>;
                const uint32_t gw1 = prmt(kIQ3Lo, kIQ3Hi, Lut::sel(tbl, g1));
                const uint32_t gw2 = prmt(kIQ3Lo, kIQ3Hi, Lut::sel(tbl, g2));
                const uint32_t sb = byte_of(rh ? (j < 4 ? f.c[2].z : f.c[2].w) : (j < 4 ? f.c[2].x : f.c[2].y), j & 3);
                const uint2 ml = Lut::sgn2(tbl, sb & 15u);
                const uint2 mh = Lut::sgn2(tbl, sb >> 4);
                lo[rh] = (gw1 ^ ml.x) + ml.y;
                hi[rh] = (gw2 ^ mh.x) + mh.y;
                const uint32_t scb = byte_of(f.sc[rh], j >> 1);
                scl[rh] = 1 + 2 * (int)((j & 1) ? (scb >> 4) : (scb & 15u));
            }
#pragma unroll
            for (int qt = 0; qt < NQ; qt++) {
                const uint2 bb = xv.b64(qt, 8 * b + j, lane);
                int d[4];
                mma_k32(d, lo[0], lo[1], hi[0], hi[1], bb.x, bb.y, 0, 0, 0, 0);
                iH[0][qt] += scl[0] * d[0];
                iL[0][qt] += scl[0] * d[1];
                iH[1][qt] += scl[1] * d[2];
                iL[1][qt] += scl[1] * d[3];
            }
        }
        finish_block<NQ>(acc, iH, iL, dfac, xv, b, lane);
    }
};

// Uniform call shape for the kernels (K formats ignore the tables).

template <int F, int NQ>
__device__ __forceinline__ void tile_dot(const typename Tile<F, NQ>::Frag& f, const XView& xv, int b,
                                         float (&acc)[2][NQ], int lane, const uint32_t* tbl) {
    if constexpr (IsIQ<F>::value)
        Tile<F, NQ>::dot(f, xv, b, acc, lane, tbl);
    else
        Tile<F, NQ>::dot(f, xv, b, acc, lane);
}

}  // namespace qw6
