// k_ep.cu -- expert-parallel dispatch/combine kernels for the prefill MoE.
//
// Experts are sharded contiguously: rank r owns experts [r*epr, (r+1)*epr).
// For the assignments a = t*topk + k of this rank's tokens:
//   count    per-GLOBAL-expert assignment counts and each assignment's
//            position among those of its expert (atomic order -- it decides
//            only which send row an assignment occupies, never a value);
//   pack     send row p = (exclusive prefix of the counts over experts)[e]
//            + pos[a] gets the token's bf16 row; send_pos[a] = p.  Send rows
//            are therefore sorted by global expert, which also groups them
//            by destination rank, and inside each destination's block by
//            the destination's local expert -- the receiver recovers every
//            row's expert from the exchanged per-expert counts alone;
//   expand   on the owner: row_expert of every received row from the
//            [source][local expert] count matrix;
//   combine  out[t] = sum_k w[a] * ret[send_pos[a]] (fp32 fma, slot order),
//            where ret holds the owners' unweighted bf16 expert outputs
//            returned in send-row order -- the same arithmetic, in the same
//            order, as the single-GPU prefill combine.
// The all-to-all exchanges in between go through NCCL (qw6_b200/ep.py).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qw6_launch.h"
#include "qw6_pdl.cuh"

namespace qw6 {

__global__ void k_ep_count(const int32_t* __restrict__ idx, int n, int32_t* __restrict__ cnt,
                           int32_t* __restrict__ pos) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a < n) pos[a] = atomicAdd(&cnt[idx[a]], 1);
}

// exclusive prefix of cnt[0..ne) into off[] (ne <= 256, blockDim 256)
__device__ __forceinline__ void block_prefix256(const int32_t* __restrict__ cnt, int ne, int* off) {
    __shared__ int wsum[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int v = tid < ne ? cnt[tid] : 0;
    int s = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, s, d);
        if (lane >= d) s += u;
    }
    if (lane == 31) wsum[warp] = s;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; w++) base += wsum[w];
    off[tid] = base + s - v;
    __syncthreads();
}

// one warp per assignment: 16-byte copies of the token row
__global__ void __launch_bounds__(256) k_ep_pack(const int32_t* __restrict__ idx, const int32_t* __restrict__ pos,
                                                 const int32_t* __restrict__ cnt, int n, int topk, int ne,
                                                 const __nv_bfloat16* __restrict__ x, int hidden,
                                                 __nv_bfloat16* __restrict__ send_x, int32_t* __restrict__ send_pos) {
    __shared__ int off[256];
    block_prefix256(cnt, ne, off);
    const int a = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (a >= n) return;
    const int p = off[idx[a]] + pos[a];
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(a / topk) * hidden);
    uint4* dstp = reinterpret_cast<uint4*>(send_x + (size_t)p * hidden);
    for (int i = lane; i < hidden / 8; i += 32) dstp[i] = src[i];
    if (lane == 0) send_pos[a] = p;
}

// recv_cnt[s*epr + e] rows from source s for local expert e arrive in
// (s, e) order; row_expert[r] = e of received row r.
__global__ void __launch_bounds__(256) k_ep_expand(const int32_t* __restrict__ recv_cnt, int nblk, int epr,
                                                   int32_t* __restrict__ row_expert) {
    __shared__ int off[256];
    block_prefix256(recv_cnt, nblk, off);
    const int b = blockIdx.x;  // one CTA per (source, local expert) block
    const int o = off[b], c = recv_cnt[b], e = b % epr;
    for (int i = threadIdx.x; i < c; i += blockDim.x) row_expert[o + i] = e;
}

__global__ void k_ep_combine(const __nv_bfloat16* __restrict__ ret, const float* __restrict__ w,
                             const int32_t* __restrict__ send_pos, int topk, int hidden, float* __restrict__ out) {
    const int t = blockIdx.y, f = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (f >= hidden) return;
    float o0 = 0.f, o1 = 0.f;
    for (int k = 0; k < topk; k++) {
        const size_t a = (size_t)t * topk + k;
        const float wk = w[a];
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(ret + (size_t)send_pos[a] * hidden + f);
        o0 = fmaf(wk, __bfloat162float(v.x), o0);
        o1 = fmaf(wk, __bfloat162float(v.y), o1);
    }
    *reinterpret_cast<float2*>(out + (size_t)t * hidden + f) = make_float2(o0, o1);
}

// ------------------------------------------------ peer-memory EP layer --
// One layer of expert parallelism without host round trips: the count
// exchange, the dispatch of token rows into the owners' receive buffers and
// the owners' down GEMM writing each output row back into its source's
// memory all go through peer memory (NVLink), ordered by epoch-stamped
// signal words; the combine then reads only local memory.  Receive rows are
// laid out by (local expert, source rank), so each owner's rows for an
// expert are contiguous and the grouped GEMM runs in sorted mode.  Buffers
// are reused across steps without extra barriers: a source writes step i+1
// data into an owner only after its own step-i combine, which waited for
// that owner's step-i outputs, so the owner is done with them.

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ep_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr uint64_t kEpWaitLimitNs = 2000000000ull;  // 2 s unless the endpoint sets another limit

__device__ __forceinline__ uint64_t ep_limit(const qw6k_ep_desc& d) { return d.wait_ns ? d.wait_ns : kEpWaitLimitNs; }

// wait until *f has reached epoch ep (wrap-safe); false after the time limit
__device__ bool ep_wait_flag(const uint32_t* f, uint32_t ep, uint64_t limit) {
    if ((int)(ld_acquire_sys(f) - ep) >= 0) return true;
    const uint64_t t0 = ep_now_ns();
    while ((int)(ld_acquire_sys(f) - ep) < 0)
        if (ep_now_ns() - t0 > limit) return false;
    return true;
}

__device__ __forceinline__ uint32_t* ep_sig(const qw6k_ep_desc& d, uint32_t p, int kind, uint32_t src) {
    return reinterpret_cast<uint32_t*>(d.peers[p] + d.o_sig) + kind * QW6K_EP_MAX_WORLD + src;
}

// wait (threads 0..world-1) for signal `kind` from every source; sets abort
__device__ bool ep_wait_all(const qw6k_ep_desc& d, int kind, uint32_t ep) {
    bool ok = true;
    if (threadIdx.x < d.world) {
        ok = ep_wait_flag(ep_sig(d, d.rank, kind, threadIdx.x), ep, ep_limit(d));
        if (!ok) {
            atomicExch(d.err, 41 + kind);
            atomicExch(d.abort, 1);
        }
    }
    return __syncthreads_and(ok);
}

// phase 6 (runs first; counters zeroed by the launcher), thread per token:
// per placed expert counts and positions, and per owner the unique token
// rows -- a token whose experts share an owner sends its row there once
// (upos >= 0 on its first such slot, -1 - position on the later ones).
__global__ void k_ep_count_u(const qw6k_ep_desc d) {
    pdl_grid_wait();
    const int topk = (int)d.topk, epr = (int)(d.ne / d.world);
    if (topk <= 8) {  // 8 lanes per token, one slot each
        const int lane = threadIdx.x & 31, sub = lane & 7;
        const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;
        const bool act = t < (int)d.ntok && sub < topk;
        const int a = t * topk + sub;
        const int g = act ? d.eslot[d.idx[a]] : -1, own = act ? g / epr : -1;
        // first slot of this token with the same owner (lanes of one token share an 8-lane group)
        int first = sub;
        for (int j = 0; j < 8; j++) {
            const int oj = __shfl_sync(0xffffffffu, own, (lane & ~7) | j);
            if (j < sub && oj == own && first == sub) first = j;
        }
        int up = 0;
        if (act) {
            d.pos[a] = atomicAdd(&d.cnt_self[g], 1);
            if (first == sub) up = atomicAdd(&d.ucnt[own], 1);
        }
        const int upf = __shfl_sync(0xffffffffu, up, (lane & ~7) | first);
        if (act) d.upos[a] = first == sub ? up : -1 - upf;
        return;
    }
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int)d.ntok) return;
    const int32_t* ix = d.idx + (size_t)t * topk;
    for (int k = 0; k < topk; k++) {
        const int a = t * topk + k, g = d.eslot[ix[k]], own = g / epr;
        d.pos[a] = atomicAdd(&d.cnt_self[g], 1);
        int first = k;
        for (int j = 0; j < k; j++)
            if (d.eslot[ix[j]] / epr == own) {
                first = j;
                break;
            }
        d.upos[a] = first == k ? atomicAdd(&d.ucnt[own], 1) : -1 - d.upos[t * topk + first];
    }
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// phase 0 (1 CTA x 256): stamp the step, publish this rank's per-expert and
// per-owner unique-row counts into every rank's matrix, wait for all
// sources, then plan (placed expert ids):
//   colsum[g]  = slots of expert g over all sources,
//   base[g]    = exclusive prefix of colsum inside g's owner block,
//   sendoff[g] = base[g] + slots for g from sources < this rank,
//   ubase[o]   = unique rows sent to owner o by sources < this rank,
//   local_cnt  = colsum over this rank's own experts.
// Every matrix entry carries the low 8 bits of the step's epoch above its
// count (counts < 2^24): a 32-bit store arrives whole, so a receiver that
// reads this step's tag in an entry has its count -- no fence and no
// separate signal.  Tags of the same matrix buffer (parity) two steps apart
// differ, and no rank runs two steps ahead of another.  Loops over ranks
// issue their peer pointers and loads eight at a time before using them.
__global__ void __launch_bounds__(256) k_ep_publish(const qw6k_ep_desc d) {
    __shared__ uint32_t s_ep;
    __shared__ int s_bad;
    __shared__ int colsum[256];
    __shared__ int pre[257];
    __shared__ int wsum[8];
    pdl_grid_wait();
    const int tid = threadIdx.x, ne = (int)d.ne, world = (int)d.world, epr = ne / world;
    if (tid == 0) {
        s_ep = *d.epoch + 1;
        *d.epoch = s_ep;
        s_bad = 0;
    }
    __syncthreads();
    const uint32_t ep = s_ep, par = ep & 1u, tag = (ep & 0xffu) << 24;
    if (*d.abort) {
        if (tid < epr) d.local_cnt[tid] = 0;
        for (int g = tid; g < ne; g += blockDim.x) d.cnt_self[g] = 0;
        if (tid < world) d.ucnt[tid] = 0;
        return;
    }
    // matrix row: per-expert counts, then per-owner unique rows; ne <= 256,
    // so entry tid + 256 (if any) is a unique-row count
    const int L = ne + world, g1 = tid + 256;
    const uint32_t v0 = tag | (uint32_t)(tid < ne ? d.cnt_self[tid] : tid < L ? d.ucnt[tid - ne] : 0);
    const uint32_t v1 = tag | (uint32_t)(g1 < L ? d.ucnt[g1 - ne] : 0);
    const size_t row = ((size_t)par * world + d.rank) * L;
    for (int p0 = 0; p0 < world; p0 += 8) {
        uint8_t* pp[8];
#pragma unroll
        for (int j = 0; j < 8; j++) pp[j] = p0 + j < world ? d.peers[p0 + j] : nullptr;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (p0 + j < world) {
                uint32_t* m = reinterpret_cast<uint32_t*>(pp[j] + d.o_cnt) + row;
                if (tid < L) st_relaxed_sys(m + tid, v0);
                if (g1 < L) st_relaxed_sys(m + g1, v1);
            }
    }
    __syncthreads();
    // the counters are consumed: zero them for the next step's count kernel
    if (tid < ne) d.cnt_self[tid] = 0;
    if (tid < world) d.ucnt[tid] = 0;
    // column tid over the sources: expert tid's slots, or (tid < world) the
    // unique rows for owner tid; poll until every entry carries this step's tag
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(d.peers[d.rank] + d.o_cnt) + (size_t)par * world * L;
    int cs = 0, before = 0, ub = 0, tot = 0;
    bool ok = true;
    const uint64_t t0 = ep_now_ns();
    for (int s0 = 0; s0 < world && ok; s0 += 8) {
        uint32_t v[8], u[8];
        for (;;) {
            bool ready = true;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const bool in = s0 + j < world;
                v[j] = in && tid < ne ? ld_relaxed_sys(mine + (size_t)(s0 + j) * L + tid) : tag;
                u[j] = in && tid < world ? ld_relaxed_sys(mine + (size_t)(s0 + j) * L + ne + tid) : tag;
                ready = ready && (v[j] & 0xff000000u) == tag && (u[j] & 0xff000000u) == tag;
            }
            if (ready) break;
            if (ep_now_ns() - t0 > ep_limit(d)) {
                ok = false;
                break;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int vc = (int)(v[j] & 0xffffffu), uc = (int)(u[j] & 0xffffffu);
            cs += vc;
            tot += uc;
            if (s0 + j < (int)d.rank) {
                before += vc;
                ub += uc;
            }
        }
    }
    if (!ok) {
        atomicExch(d.err, 41 + QW6K_EP_SIG_COUNTS);
        atomicExch(d.abort, 1);
    }
    if (!__syncthreads_and(ok)) {
        if (tid < epr) d.local_cnt[tid] = 0;
        return;
    }
    colsum[tid] = tid < ne ? cs : 0;
    if (tid < world) {  // this rank's base at owner tid; no owner may receive more rows than its buffer holds
        d.ubase[tid] = ub;
        if (tot > (int)d.cap) s_bad = 1;
    }
    __syncthreads();
    // exclusive prefix of colsum over all experts (warp scans + warp totals);
    // pre[ne] is the total, so an owner block [b0, b1) holds pre[b1] - pre[b0]
    // slots and the prefix inside it is pre[g] - pre[b0]
    {
        const int lane = tid & 31, wid = tid >> 5;
        const int v = colsum[tid];
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[wid] = x;
        __syncthreads();
        int wb = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) wb += w < wid ? wsum[w] : 0;
        pre[tid] = wb + x - v;
        if (tid == 255) pre[256] = wb + x;
        __syncthreads();
        if (tid < ne) {
            const int b0 = (tid / epr) * epr;
            d.sendoff[tid] = pre[tid] - pre[b0] + before;
            // an owner block can never hold more slots than the receive capacity
            if (tid == b0 && pre[b0 + epr] - pre[b0] > (int)d.cap) s_bad = 1;
        }
    }
    __syncthreads();
    if (s_bad) {
        if (tid == 0) {
            atomicExch(d.err, 44);
            atomicExch(d.abort, 1);
        }
        if (tid < epr) d.local_cnt[tid] = 0;
        return;
    }
    if (tid < epr) d.local_cnt[tid] = colsum[d.rank * epr + tid];
}

// phase 1: warps loop over the assignments (grid-stride): the token row goes
// to its owner's rx at its unique row (first slot of the token at that owner
// only), the slot's metadata as one 8-byte store; the last CTA to finish
// signals every owner.
__global__ void __launch_bounds__(256) k_ep_dispatch(const qw6k_ep_desc d) {
    __shared__ bool last;
    pdl_grid_wait();
    const int n = (int)(d.ntok * d.topk), epr = (int)(d.ne / d.world);
    const bool go = !*d.abort;
    const int lane = threadIdx.x & 31, nw = gridDim.x * (blockDim.x >> 5);
    for (int a = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); go && a < n; a += nw) {
        const int g = d.eslot[d.idx[a]], owner = g / epr, slot = d.sendoff[g] + d.pos[a], up = d.upos[a];
        const int urow = d.ubase[owner] + (up >= 0 ? up : -1 - up);
        if (up >= 0) {  // first slot of this token at this owner: send the row
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(d.x) +
                                                              (size_t)(a / (int)d.topk) * d.hidden);
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(d.peers[owner] + d.o_rx) +
                                                  (size_t)urow * d.hidden);
            // 4 KB rows per pass: all loads in flight before the stores
            const int nv = (int)d.hidden / 8;
            for (int i0 = 0; i0 < nv; i0 += 256) {
                uint4 v[8];
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (i0 + u * 32 + lane < nv) v[u] = __ldg(src + i0 + u * 32 + lane);
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (i0 + u * 32 + lane < nv) dst[i0 + u * 32 + lane] = v[u];
            }
        }
        if (lane == 0) {
            d.send_row[a] = slot;
            // the slot's token row at the owner and where its output goes, one 8-byte store
            reinterpret_cast<int2*>(d.peers[owner] + d.o_smeta)[slot] = make_int2(urow, (int)(d.rank * d.nmax) + a);
        }
    }
    // the barrier orders every thread's stores before thread 0's system-scope
    // fence, which orders them before the completion count and the signal
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(d.done_ctas, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last) {
        __threadfence_system();
        if (threadIdx.x == 0) *d.done_ctas = 0;
        if (go && threadIdx.x < d.world) st_release_sys(ep_sig(d, threadIdx.x, QW6K_EP_SIG_ROWS, d.rank), *d.epoch);
    }
}

// phases 2 and 4: wait for a signal from every rank
__global__ void k_ep_wait(const qw6k_ep_desc d, int kind) {
    pdl_grid_wait();
    if (*d.abort) return;
    ep_wait_all(d, kind, *d.epoch);
}

// phase 3: this rank's expert outputs are complete
__global__ void k_ep_signal_done(const qw6k_ep_desc d) {
    pdl_grid_wait();
    if (*d.abort) return;
    __threadfence_system();
    if (threadIdx.x < d.world) st_release_sys(ep_sig(d, threadIdx.x, QW6K_EP_SIG_DONE, d.rank), *d.epoch);
}

// phase 5: out[t] = sum_k w[a] * ret[a] (fp32 fma, slot order); the owners
// have written each assignment's bf16 output into this rank's ret
__global__ void k_ep_combine_ret(const qw6k_ep_desc d) {
    pdl_grid_wait();
    const int t = blockIdx.y, f = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (f >= (int)d.hidden || *d.abort) return;
    const int topk = (int)d.topk;
    const __nv_bfloat16* ret = reinterpret_cast<const __nv_bfloat16*>(d.peers[d.rank] + d.o_ret);
    // 8 features per thread: one 16-byte load per slot, all issued before the sums
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < topk; k0 += 8) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k0 + k < topk)
                v[k] = __ldcg(reinterpret_cast<const uint4*>(ret + ((size_t)t * topk + k0 + k) * d.hidden + f));
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (k0 + k >= topk) break;
            const float wk = d.w[(size_t)t * topk + k0 + k];
            const uint32_t u[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                o[2 * i] = fmaf(wk, __uint_as_float(u[i] << 16), o[2 * i]);
                o[2 * i + 1] = fmaf(wk, __uint_as_float(u[i] & 0xffff0000u), o[2 * i + 1]);
            }
        }
    }
    float4* op = reinterpret_cast<float4*>(d.out + (size_t)t * d.hidden + f);
    op[0] = make_float4(o[0], o[1], o[2], o[3]);
    op[1] = make_float4(o[4], o[5], o[6], o[7]);
}

}  // namespace qw6

using namespace qw6;

extern "C" int qw6k_ep_count(const int32_t* idx, uint32_t n, uint32_t ne, int32_t* cnt, int32_t* pos,
                             cudaStream_t st) {
    if (!idx || !cnt || !pos || !n || !ne || ne > 256) return QW6K_ERR_ARG;
    if (cudaMemsetAsync(cnt, 0, ne * sizeof(int32_t), st) != cudaSuccess) return QW6K_ERR_CUDA;
    k_ep_count<<<(n + 255) / 256, 256, 0, st>>>(idx, (int)n, cnt, pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_pack(const int32_t* idx, const int32_t* pos, const int32_t* cnt, uint32_t n, uint32_t topk,
                            uint32_t ne, const void* x_bf16, uint32_t hidden, void* send_x, int32_t* send_pos,
                            cudaStream_t st) {
    if (!idx || !pos || !cnt || !x_bf16 || !send_x || !send_pos || !n || !topk || !ne || ne > 256 || !hidden ||
        hidden % 8)
        return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(x_bf16) | reinterpret_cast<uintptr_t>(send_x)) & 15u) return QW6K_ERR_ALIGN;
    k_ep_pack<<<(n + 7) / 8, 256, 0, st>>>(idx, pos, cnt, (int)n, (int)topk, (int)ne, (const __nv_bfloat16*)x_bf16,
                                          (int)hidden, (__nv_bfloat16*)send_x, send_pos);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_expand(const int32_t* recv_cnt, uint32_t world, uint32_t epr, int32_t* row_expert,
                              cudaStream_t st) {
    if (!recv_cnt || !row_expert || !world || !epr || world * epr > 256) return QW6K_ERR_ARG;
    k_ep_expand<<<world * epr, 256, 0, st>>>(recv_cnt, (int)(world * epr), (int)epr, row_expert);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_combine(const void* ret_bf16, const float* w, const int32_t* send_pos, uint32_t ntok,
                               uint32_t topk, uint32_t hidden, float* out, cudaStream_t st) {
    if (!ret_bf16 || !w || !send_pos || !out || !ntok || !topk || !hidden || hidden % 2) return QW6K_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(ret_bf16) & 3u) || (reinterpret_cast<uintptr_t>(out) & 7u)) return QW6K_ERR_ALIGN;
    dim3 g((hidden / 2 + 255) / 256, ntok);
    k_ep_combine<<<g, 256, 0, st>>>((const __nv_bfloat16*)ret_bf16, w, send_pos, (int)topk, (int)hidden, out);
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}

extern "C" int qw6k_ep_p2p_phase(const qw6k_ep_desc* d, int phase, cudaStream_t st) {
    if (!d || !d->peers || !d->world || d->world > QW6K_EP_MAX_WORLD || d->rank >= d->world || !d->ne ||
        d->ne > 256 || d->ne % d->world || !d->topk || !d->ntok || !d->hidden || d->hidden % 8 || !d->epoch ||
        !d->abort || !d->done_ctas || !d->err || !d->idx || !d->w || !d->cnt_self || !d->pos || !d->sendoff ||
        !d->local_cnt || !d->send_row || !d->x || !d->out || !d->cap || !d->nmax || d->ntok * d->topk > d->nmax ||
        !d->ucnt || !d->upos || !d->ubase || !d->eslot)
        return QW6K_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(d->out) & 15u) return QW6K_ERR_ALIGN;  // 16-byte stores in the combine
    // every phase is launched as a programmatic dependent of the previous
    // kernel on the stream; the counters of phase 6 are zeroed at create and
    // re-zeroed by phase 0 once consumed
    cudaError_t e;
    switch (phase) {
    case 6:
        e = d->topk <= 8 ? launch_pdl(k_ep_count_u, dim3((d->ntok * 8 + 255) / 256), dim3(256), 0, st, *d)
                         : launch_pdl(k_ep_count_u, dim3((d->ntok + 127) / 128), dim3(128), 0, st, *d);
        break;
    case 0:
        e = launch_pdl(k_ep_publish, dim3(1), dim3(256), 0, st, *d);
        break;
    case 1: {
        // a warp per assignment up to a grid that stays resident (4 CTAs of
        // 256 threads per SM at the kernel's register count): each warp's
        // loop is a chain of dependent loads, so fewer rounds per warp is
        // what shortens the dispatch
        const uint32_t n = d->ntok * d->topk, ctas = (n + 7) / 8, cap = 4u * 148u;
        e = launch_pdl(k_ep_dispatch, dim3(ctas < cap ? ctas : cap), dim3(256), 0, st, *d);
        break;
    }
    case 2:
        e = launch_pdl(k_ep_wait, dim3(1), dim3(64), 0, st, *d, (int)QW6K_EP_SIG_ROWS);
        break;
    case 3:
        e = launch_pdl(k_ep_signal_done, dim3(1), dim3(64), 0, st, *d);
        break;
    case 4:
        e = launch_pdl(k_ep_wait, dim3(1), dim3(64), 0, st, *d, (int)QW6K_EP_SIG_DONE);
        break;
    case 5:
        e = launch_pdl(k_ep_combine_ret, dim3((d->hidden / 8 + 255) / 256, d->ntok), dim3(256), 0, st, *d);
        break;
    default:
        return QW6K_ERR_ARG;
    }
    if (e != cudaSuccess) return QW6K_ERR_CUDA;
    return cudaPeekAtLastError() == cudaSuccess ? 0 : QW6K_ERR_CUDA;
}
