// k_sample.cu -- temperature / top-k / top-p sampling over rows of logits on
// the GPU, with qw6_sample's semantics (qw6.c:2904-2982) and its uniform
// draw u given per row:
//   temp <= 0                -> argmax (qw6_cpu_argmax);
//   score_i = logit_i / temp (fp32); items in descending score order, lower
//   index first on ties;
//   limit   = top_k if 0 < top_k < n, else n;
//   sum     = sum over the first `limit` items of exp(score - max) (double);
//   sum <= 0                 -> the first item;
//   nucleus = top_p < 1 ? the shortest prefix whose probabilities reach top_p
//             : limit;
//   pick    = the first item whose running exp(score - max) sum reaches
//             u * (the nucleus's sum), else the nucleus's last item.
// No sort of the row.  key = order-preserving(score) << 32 | ~index orders
// the items exactly as qw6's comparator (larger key first).  Three launches:
//   k_smp_max     the largest key of every row (the top item, the max score);
//   k_smp_hist    a per-row histogram over the top 16 bits of the ordered
//                 score: item count and exp(score - max) sum (double) per
//                 bucket (65536 buckets, higher bucket = higher scores);
//   k_smp_pick    one CTA per row walks the buckets from the top to each
//                 boundary (the top_k-th item, the end of the nucleus, the
//                 pick), gathers the boundary bucket's items into shared
//                 memory, sorts them by key and walks them in qw6's order.
// A boundary bucket with more items than fit in shared memory (e.g. many
// equal logits) is resolved by a radix selection over the row instead.  The
// double sums over whole buckets run in another order than qw6's sequential
// loop, which can change a pick only when u * sum falls within rounding of a
// cumulative boundary.  Logits must not contain NaN.
#include <cuda_runtime.h>

#include "qw6_argmax.cuh"
#include "qw6_devcfg.cuh"
#include "qw6_launch.h"

namespace qw6 {

constexpr int kSmpBuckets = 65536;
constexpr int kSmpThreads = 1024;
constexpr int kSmpCap = 8192;  // items of one boundary bucket sorted in shared memory

__device__ __forceinline__ uint32_t ord32(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unord32(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
__device__ __forceinline__ unsigned long long smp_key(float s, uint32_t i) {
    return ((unsigned long long)ord32(s) << 32) | (unsigned long long)(~i);
}
__device__ __forceinline__ uint32_t key_index(unsigned long long k) { return ~(uint32_t)(k & 0xffffffffull); }
__device__ __forceinline__ float key_score(unsigned long long k) { return unord32((uint32_t)(k >> 32)); }

struct SmpArgs {
    const float* logits;
    int n, ld;
    float temp, top_p;
    int top_k;
    const float* u;
    uint32_t* out;
    unsigned long long* top;  // [rows] largest key (zeroed)
    unsigned int* cnt;        // [rows][65536] (zeroed)
    double* mass;             // [rows][65536] (zeroed)
};

__global__ void k_smp_max(const SmpArgs a) {
    const float* lg = a.logits + (size_t)blockIdx.y * a.ld;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const unsigned long long k =
            a.temp > 0.f ? smp_key(__fdiv_rn(lg[i], a.temp), (uint32_t)i) : argmax_key(lg[i], (uint32_t)i);
        best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0 && best) atomicMax(a.top + blockIdx.y, best);
}

__global__ void k_smp_hist(const SmpArgs a) {
    if (a.temp <= 0.f) return;
    const float* lg = a.logits + (size_t)blockIdx.y * a.ld;
    const double smax = (double)key_score(a.top[blockIdx.y]);
    unsigned int* cnt = a.cnt + (size_t)blockIdx.y * kSmpBuckets;
    double* mass = a.mass + (size_t)blockIdx.y * kSmpBuckets;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const float s = __fdiv_rn(lg[i], a.temp);
        const uint32_t b = ord32(s) >> 16;
        atomicAdd(&cnt[b], 1u);
        atomicAdd(&mass[b], exp((double)s - smax));
    }
}

struct SmpShared {
    unsigned long long keys[kSmpCap];
    unsigned long long wk[kSmpThreads / 32];
    double csum[kSmpThreads];  // per-thread chunk totals, then their exclusive scan
    unsigned int ccnt[kSmpThreads];
    unsigned int ngath;
    int bsel;
    double above_m;
    unsigned int above_c;
    unsigned long long kres;
    double vres;
    int ok;
};

// Walk the buckets from the top: the bucket where the running count (MASS
// false) or mass first reaches `target` (bucket order; within a bucket the
// exact order is resolved later).  The current set is every bucket above
// `bmin` plus the part of bucket `bmin` given by `part_c` / `part_m` (the
// items of the cut bucket whose key is >= the set's floor); buckets below
// bmin are outside it.  Sets S.bsel (-1: never reached) and S.above_c /
// S.above_m (totals of the set's buckets above the selected one, or of the
// whole set when never reached).
template <bool MASS>
__device__ void bucket_walk(const unsigned int* cnt, const double* mass, int bmin, unsigned part_c, double part_m,
                            double target, SmpShared& S) {
    constexpr int per = kSmpBuckets / kSmpThreads;  // 64 buckets per thread, thread 0 at the top
    const int hi = kSmpBuckets - 1 - threadIdx.x * per;
    double m = 0.0;
    unsigned c = 0;
    for (int j = 0; j < per; j++) {
        const int b = hi - j;
        if (b < bmin) continue;
        const unsigned bc = b == bmin ? part_c : cnt[b];
        const double bm = b == bmin ? part_m : mass[b];
        c += bc;
        m += bm;
    }
    S.csum[threadIdx.x] = m;
    S.ccnt[threadIdx.x] = c;
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the chunk totals (1024 entries, from the top)
        double am = 0.0;
        unsigned ac = 0;
        int tsel = -1;
        for (int t = 0; t < kSmpThreads; t++) {
            const double nm = am + S.csum[t];
            const unsigned nc = ac + S.ccnt[t];
            if (tsel < 0 && (MASS ? (S.ccnt[t] && nm >= target) : ((double)nc >= target && S.ccnt[t]))) {
                tsel = t;
                break;
            }
            am = nm;
            ac = nc;
        }
        S.bsel = -1;
        if (tsel >= 0) {  // walk that thread's buckets
            const int h = kSmpBuckets - 1 - tsel * per;
            for (int j = 0; j < per; j++) {
                const int b = h - j;
                if (b < bmin) continue;
                const unsigned bc = b == bmin ? part_c : cnt[b];
                const double bm = b == bmin ? part_m : mass[b];
                if (bc && (MASS ? am + bm >= target : (double)(ac + bc) >= target)) {
                    S.bsel = b;
                    break;
                }
                am += bm;
                ac += bc;
            }
        }
        S.above_m = am;
        S.above_c = ac;
    }
    __syncthreads();
}

// Gather the keys of bucket b with key >= floor into shared memory and sort
// them in descending order (bitonic); false if they do not fit.
__device__ bool gather_sorted(const SmpArgs& a, const float* lg, int b, unsigned long long floor, SmpShared& S) {
    if (threadIdx.x == 0) S.ngath = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
        const float s = __fdiv_rn(lg[i], a.temp);
        if ((int)(ord32(s) >> 16) != b) continue;
        const unsigned long long k = smp_key(s, (uint32_t)i);
        if (k < floor) continue;
        const unsigned p = atomicAdd(&S.ngath, 1u);
        if (p < (unsigned)kSmpCap) S.keys[p] = k;
    }
    __syncthreads();
    const unsigned n = S.ngath;
    if (n > (unsigned)kSmpCap) return false;
    unsigned np = 1;
    while (np < n) np <<= 1;
    for (unsigned i = n + threadIdx.x; i < np; i += blockDim.x) S.keys[i] = 0ull;  // pad with the smallest key
    __syncthreads();
    for (unsigned k = 2; k <= np; k <<= 1)
        for (unsigned j = k >> 1; j > 0; j >>= 1) {
            for (unsigned i = threadIdx.x; i < np; i += blockDim.x) {
                const unsigned l = i ^ j;
                if (l > i) {
                    const unsigned long long x = S.keys[i], y = S.keys[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? x < y : x > y) {
                        S.keys[i] = y;
                        S.keys[l] = x;
                    }
                }
            }
            __syncthreads();
        }
    return true;
}

// Radix selection over the whole row (slow path for an oversized bucket):
// the key where the running count / mass of the items with key >= floor, in
// descending key order, first reaches target; S.vres = count / mass above it.
template <bool MASS>
__device__ bool radix_select(const SmpArgs& a, const float* lg, double smax, unsigned long long floor, double target,
                             SmpShared& S) {
    __shared__ unsigned int hc[256];
    __shared__ double hm[256];
    unsigned long long prefix = 0ull, mask = 0ull;
    double above = 0.0;
    for (int pass = 0; pass < 8; pass++) {
        const int shift = 56 - 8 * pass;
        for (int b = threadIdx.x; b < 256; b += blockDim.x) {
            hc[b] = 0u;
            hm[b] = 0.0;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
            const float s = __fdiv_rn(lg[i], a.temp);
            const unsigned long long k = smp_key(s, (uint32_t)i);
            if (k >= floor && (k & mask) == prefix) {
                const int d = (int)((k >> shift) & 255u);
                atomicAdd(&hc[d], 1u);
                if (MASS) atomicAdd(&hm[d], exp((double)s - smax));
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double acc = above;
            int dsel = -1;
            for (int d = 255; d >= 0; d--) {
                const double c = MASS ? hm[d] : (double)hc[d];
                if (hc[d] && acc + c >= target) {
                    dsel = d;
                    break;
                }
                acc += c;
            }
            S.ok = dsel >= 0;
            S.vres = acc;
            S.kres = prefix | ((unsigned long long)(dsel < 0 ? 0 : dsel) << shift);
        }
        __syncthreads();
        if (!S.ok) return false;
        above = S.vres;
        prefix = S.kres;
        mask |= 255ull << shift;
        __syncthreads();
    }
    return true;
}

// The boundary item of the set {key >= floor} (bucket_walk's bmin / part
// describe its cut bucket) where the running count / mass, in descending key
// order, first reaches target.  kout: its key, vout: the running count /
// mass including it.  false: never reached.
template <bool MASS>
__device__ bool find_boundary(const SmpArgs& a, const float* lg, double smax, const unsigned* cnt, const double* mass,
                              int bmin, unsigned part_c, double part_m, unsigned long long floor, double target,
                              SmpShared& S, unsigned long long* kout, double* vout) {
    bucket_walk<MASS>(cnt, mass, bmin, part_c, part_m, target, S);
    const int b = S.bsel;
    if (b < 0) return false;
    const double above = MASS ? S.above_m : (double)S.above_c;
    if (gather_sorted(a, lg, b, floor, S)) {
        if (threadIdx.x == 0) {
            double acc = above;
            unsigned long long kk = S.keys[0];
            for (unsigned i = 0; i < S.ngath; i++) {
                kk = S.keys[i];
                acc += MASS ? exp((double)key_score(kk) - smax) : 1.0;
                if (acc >= target) break;
            }
            S.kres = kk;
            S.vres = acc;
        }
        __syncthreads();
        *kout = S.kres;
        *vout = S.vres;
        return true;
    }
    if (!radix_select<MASS>(a, lg, smax, floor, target, S)) return false;
    *kout = S.kres;
    *vout = S.vres + (MASS ? exp((double)key_score(S.kres) - smax) : 1.0);
    return true;
}

// Count and mass of the items of bucket b with key >= floor (the cut bucket
// of a set).
__device__ void bucket_part(const SmpArgs& a, const float* lg, double smax, int b, unsigned long long floor,
                            SmpShared& S, unsigned* pc, double* pm) {
    double m = 0.0;
    unsigned c = 0;
    for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
        const float s = __fdiv_rn(lg[i], a.temp);
        if ((int)(ord32(s) >> 16) != b || smp_key(s, (uint32_t)i) < floor) continue;
        c++;
        m += exp((double)s - smax);
    }
    S.csum[threadIdx.x] = m;
    S.ccnt[threadIdx.x] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tm = 0.0;
        unsigned tc = 0;
        for (int t = 0; t < kSmpThreads; t++) {
            tm += S.csum[t];
            tc += S.ccnt[t];
        }
        S.vres = tm;
        S.ngath = tc;
    }
    __syncthreads();
    *pm = S.vres;
    *pc = S.ngath;
    __syncthreads();
}

__global__ void __launch_bounds__(kSmpThreads) k_smp_pick(const SmpArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    SmpShared& S = *reinterpret_cast<SmpShared*>(smem);
    const int row = blockIdx.x;
    const float* lg = a.logits + (size_t)row * a.ld;
    const unsigned long long top = a.top[row];
    if (a.temp <= 0.f) {  // qw6_cpu_argmax
        if (threadIdx.x == 0) a.out[row] = argmax_key_index(top);
        return;
    }
    const double smax = (double)key_score(top);
    const unsigned* cnt = a.cnt + (size_t)row * kSmpBuckets;
    const double* mass = a.mass + (size_t)row * kSmpBuckets;
    const float top_p = (a.top_p <= 0.f || a.top_p > 1.f) ? 1.f : a.top_p;
    // limit: the first top_k items (the set {key >= floor}; bmin is the bucket
    // of its floor item, pc / pm the count and mass of the set in bmin)
    unsigned long long floor = 0ull;
    int bmin = 0;
    unsigned pc = cnt[0];
    double pm = mass[0];
    if (a.top_k > 0 && a.top_k < a.n) {
        unsigned long long k;
        double v;
        if (find_boundary<false>(a, lg, smax, cnt, mass, 0, pc, pm, 0ull, (double)a.top_k, S, &k, &v)) {
            floor = k;
            bmin = (int)(ord32(key_score(k)) >> 16);
            bucket_part(a, lg, smax, bmin, floor, S, &pc, &pm);
        }
    }
    bucket_walk<true>(cnt, mass, bmin, pc, pm, 1e300, S);  // target never reached: the set's total
    const double sum = S.above_m;
    if (!(sum > 0.0)) {
        if (threadIdx.x == 0) a.out[row] = key_index(top);
        return;
    }
    // nucleus
    unsigned long long nfloor = floor;
    double keep = sum;
    if (top_p < 1.f) {
        unsigned long long k;
        double v;
        if (find_boundary<true>(a, lg, smax, cnt, mass, bmin, pc, pm, floor, (double)top_p * sum, S, &k, &v)) {
            nfloor = k;
            keep = v;
            bmin = (int)(ord32(key_score(k)) >> 16);
            bucket_part(a, lg, smax, bmin, nfloor, S, &pc, &pm);
        }
    }
    // the pick
    const double target = (double)a.u[row] * keep;
    unsigned long long k;
    double v;
    uint32_t tok;
    if (find_boundary<true>(a, lg, smax, cnt, mass, bmin, pc, pm, nfloor, target, S, &k, &v)) {
        tok = key_index(k);
    } else if (nfloor) {
        tok = key_index(nfloor);  // the nucleus's last item
    } else {  // the last item of the whole order: the smallest key
        unsigned long long lo = ~0ull;
        for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
            const unsigned long long kk = smp_key(__fdiv_rn(lg[i], a.temp), (uint32_t)i);
            lo = kk < lo ? kk : lo;
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, lo, o);
            lo = x < lo ? x : lo;
        }
        if ((threadIdx.x & 31) == 0) S.wk[threadIdx.x >> 5] = lo;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long m = ~0ull;
            for (int w = 0; w < kSmpThreads / 32; w++) m = S.wk[w] < m ? S.wk[w] : m;
            S.kres = m;
        }
        __syncthreads();
        tok = key_index(S.kres);
    }
    if (threadIdx.x == 0) a.out[row] = tok;
}

}  // namespace qw6

using namespace qw6;

extern "C" size_t qw6k_sample_ws_bytes(uint32_t nrows) {
    return (size_t)nrows * (8 + (size_t)kSmpBuckets * (4 + 8)) + 256;
}

extern "C" int qw6k_sample(const float* logits, uint32_t n, uint32_t ld, uint32_t nrows, float temp, float top_p,
                           int top_k, const float* u, uint32_t* out, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (!logits || !u || !out || !ws || !n || n > 0x7fffffffu || ld < n || !nrows || nrows > 65535 ||
        ws_bytes < qw6k_sample_ws_bytes(nrows))
        return QW6K_ERR_ARG;
    SmpArgs a;
    a.logits = logits;
    a.n = (int)n;
    a.ld = (int)ld;
    a.temp = temp;
    a.top_p = top_p;
    a.top_k = top_k;
    a.u = u;
    a.out = out;
    uint8_t* p = static_cast<uint8_t*>(ws);
    a.mass = reinterpret_cast<double*>(p);
    p += (size_t)nrows * kSmpBuckets * 8;
    a.top = reinterpret_cast<unsigned long long*>(p);
    p += (size_t)nrows * 8;
    a.cnt = reinterpret_cast<unsigned int*>(p);
    if (cudaMemsetAsync(ws, 0, qw6k_sample_ws_bytes(nrows), st) != cudaSuccess) return QW6K_ERR_CUDA;
    const size_t smem = sizeof(SmpShared);
    static DevFlags cfg;
    if (smem_optin(cfg, k_smp_pick, (int)smem)) return QW6K_ERR_CUDA;
    const int gx = (int)(((long long)n + 256 * 16 - 1) / (256 * 16));
    k_smp_max<<<dim3(gx, nrows), 256, 0, st>>>(a);
    k_smp_hist<<<dim3(gx, nrows), 256, 0, st>>>(a);
    k_smp_pick<<<nrows, kSmpThreads, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
