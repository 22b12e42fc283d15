/* qw6_launch.h -- C-callable launchers of the CUDA kernels (internal).
 *
 * The host side of libqw6cuda is plain C (qw6_host.c); it reaches the
 * kernels only through these functions, which take device pointers and a
 * stream, validate shapes, and enqueue work without synchronizing.
 * All return 0 or a negative QW6K_ERR_* code.
 */
#ifndef QW6_LAUNCH_H
#define QW6_LAUNCH_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QW6K_ERR_ARG (-2)
#define QW6K_ERR_QUANT (-3)
#define QW6K_ERR_CUDA (-4)
#define QW6K_ERR_ALIGN (-5)
#define QW6K_ERR_TIMEOUT (-6)

/* 16 * block bytes of the format (0 if not a super-block format). */
size_t qw6k_tile_bytes(uint32_t quant);
/* Device bytes of the packed tile layout of a rows x cols matrix. */
size_t qw6k_packed_bytes(uint32_t quant, uint32_t rows, uint32_t cols);

/* Raw GGUF rows -> packed tile layout, nmat matrices at the given strides. */
int qw6k_pack(uint32_t quant, const void *raw, void *packed, uint32_t rows, uint32_t cols,
              uint32_t nmat, size_t raw_stride, size_t packed_stride, cudaStream_t st);

/* Bit-exact fp32 dequantization of raw GGUF rows (qw6.c:1674-1724). */
int qw6k_dequant(uint32_t quant, const void *raw, float *out, uint32_t rows, uint32_t cols,
                 cudaStream_t st);

/* y[t*ldy + r] = W[r] . x[t*ldx ...] for t < ntok (<= 32); W packed. */
int qw6k_matvec(uint32_t quant, const void *packed, const float *x, float *y, uint32_t rows,
                uint32_t cols, uint32_t ntok, uint32_t ldx, uint32_t ldy, cudaStream_t st);

/* LM head: keys[t] = max over rows r of the packed (logit, row_offset + r)
 * key of token t (qw6_argmax.cuh); y (nullable) also receives the logits.
 * keys are zeroed first.  Row shards combine with qw6k_argmax_keys_reduce. */
int qw6k_matvec_argmax(uint32_t quant, const void *packed, const float *x, float *y, unsigned long long *keys,
                       uint32_t rows, uint32_t cols, uint32_t ntok, uint32_t ldx, uint32_t ldy, uint32_t row_offset,
                       cudaStream_t st);
/* idx[t], val[t] (val nullable) from the max over nshards of keys[s*ntok + t]. */
int qw6k_argmax_keys_reduce(const unsigned long long *keys, uint32_t nshards, uint32_t ntok, uint32_t *idx,
                            float *val, cudaStream_t st);

/* D[M x N] fp32 = A[M x K] . B[N x K]^T, bf16 K-major operands, on tcgen05
 * (K % 64 == 0).  *err (device int) is set non-zero if a bounded wait timed out. */
int qw6k_gemm_bf16_nt(const void *A, const void *B, float *D, uint32_t M, uint32_t N, uint32_t K, int *err,
                      cudaStream_t st);

/* fp32 weights (row-major rows x cols). */
int qw6k_matvec_f32(const float *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                    cudaStream_t st);

/* Top-k routing, one token per row of logits (qw6.c:2796-2827). */
int qw6k_moe_route(const float *logits, uint32_t ntok, uint32_t n_experts, uint32_t top_k,
                   int32_t *idx, float *w, cudaStream_t st);

/* out[i] = sum_e w[e]*expert_out[e*dim+i] (+ shared_weight*shared[i]). */
int qw6k_moe_gather(const float *expert_out, const float *w, const float *shared,
                    float shared_weight, float *out, uint32_t dim, uint32_t top_k, cudaStream_t st);

/* out[i] = silu(gate[i]) * up[i]. */
int qw6k_silu_mul(const float *gate, const float *up, float *out, uint32_t n, cudaStream_t st);

/* Greedy argmax (lowest index on ties; NaN handling as qw6_cpu_argmax).
 * key64 is caller-provided device scratch of 8 bytes. */
int qw6k_argmax(const float *x, uint32_t n, unsigned long long *key64, uint32_t *out_idx,
                float *out_val, cudaStream_t st);

/* Routed MoE FFN for decode batches (ntok*top_k <= 4096, hidden and inter
 * multiples of 512, hidden <= 4096).  Expert e's packed matrices live at
 * base + e*stride.  The host runs qw6k_moe_nphases() launches in order on
 * one stream: for ntok <= 4 gate/up (self-routed), down, combine; otherwise
 * plan (route + group by expert), gate/up + silu, down, combine. */
typedef struct {
    uint32_t gq, dq;
    const void *gate, *up, *down;
    size_t gstride, ustride, dstride;
    const float *logits, *x;
    float *out;
    uint32_t ntok, hidden, inter, ne, topk;
    void *ws;
    size_t ws_bytes;
    /* prefill "rows" mode (logits == NULL, topk == 1, out unused): row r of
     * x goes to expert row_expert[r]; dout[r] (bf16, [ntok x hidden]) =
     * FFN_e(x[r]), unweighted */
    const int32_t *row_expert;
    void *dout;
    /* sorted rows mode (rows mode with row_expert == NULL): the rows of x are
     * grouped by expert in expert order, expert_counts[e] (device) rows each */
    const int32_t *expert_counts;
    /* sorted rows mode: x row of slot r is slot_row[r] (NULL: row r) --
     * received token rows are shared by the slots of one token's experts */
    const int32_t *slot_row;
    /* push mode (sorted rows, dout == NULL): the expert output of row r goes
     * to out_peers[s] + out_off + q * hidden * 2 bytes (bf16 row), where
     * slot_dst[r * slot_stride] = s * out_rows + q -- another GPU's memory
     * over NVLink; slot_row is read with the same stride */
    uint8_t *const *out_peers;
    size_t out_off;
    const int32_t *slot_dst;
    uint32_t out_rows;
    uint32_t slot_stride; /* 0 or 1: dense; 2: interleaved (row, dst) pairs */
} qw6k_moe_desc;

size_t qw6k_moe_ws_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t ne, uint32_t topk);
int qw6k_moe_check(const qw6k_moe_desc *d);
int qw6k_moe_nphases(const qw6k_moe_desc *d);
int qw6k_moe_phase_kind(const qw6k_moe_desc *d, int phase); /* 0 plan, 1 gate/up, 2 down, 3 combine */
int qw6k_moe_phase(const qw6k_moe_desc *d, int phase, cudaStream_t st);
/* Configure and load every decode kernel on the current device. */
int qw6k_moe_decode_setup(void);

/* MoE FFN block (k_block.cu).  pre: normed = rmsnorm(x') * norm_w with x' =
 * x, or x + add written to xsum when add is given; logits = router . normed
 * (fp32 router [ne x hidden]), sgate[t] = sigmoid(srouter . normed) or 1
 * when srouter is NULL.  post: out = x + (ffn + sgate * shared) (shared
 * nullable).  bad (nullable): set to 1 when x + add or out holds a NaN/Inf. */
int qw6k_block_pre(const float *x, const float *add, float *xsum, int *bad, const float *norm_w, const float *router,
                   const float *srouter, float *normed, float *logits, float *sgate, uint32_t ntok, uint32_t hidden,
                   uint32_t ne, cudaStream_t st);
int qw6k_block_post(const float *x, const float *ffn, const float *shared, const float *sgate, float *out, int *bad,
                    uint32_t ntok, uint32_t hidden, cudaStream_t st);
/* block_post, then normed = rmsnorm(out) * norm_w (hidden <= 4096) */
int qw6k_post_norm(const float *x, const float *ffn, const float *shared, const float *sgate, float *out, int *bad,
                   const float *norm_w, float *normed, uint32_t ntok, uint32_t hidden, cudaStream_t st);

/* Sampling (k_sample.cu): out[r] = qw6_sample's pick (qw6.c:2904-2982) over
 * logits row r (n floats, rows ld apart) with uniform draw u[r]; ws: device
 * scratch of qw6k_sample_ws_bytes(nrows) bytes (zeroed here). */
size_t qw6k_sample_ws_bytes(uint32_t nrows);
int qw6k_sample(const float *logits, uint32_t n, uint32_t ld, uint32_t nrows, float temp, float top_p, int top_k,
                const float *u, uint32_t *out, void *ws, size_t ws_bytes, cudaStream_t st);

/* Routed MoE FFN for prefill batches on tcgen05 (k_prefill.cu): desc->x is
 * bf16 [ntok x hidden]; gate/up/down Q4_K or Q6_K packed; hidden, inter
 * multiples of 256.  Phases 0..6 in order on one stream (route, count,
 * offsets, scatter, gate/up GEMM, down GEMM, slot-order combine into out).
 * *err records bounded-wait timeouts. */
size_t qw6k_moe_prefill_ws_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t ne, uint32_t topk);
int qw6k_moe_prefill_check(const qw6k_moe_desc *d, int *err);
int qw6k_moe_prefill_phase(const qw6k_moe_desc *d, int *err, int phase, cudaStream_t st);

/* Expert-parallel dispatch/combine helpers (k_ep.cu). */
int qw6k_ep_count(const int32_t *idx, uint32_t n, uint32_t ne, int32_t *cnt, int32_t *pos, cudaStream_t st);
int qw6k_ep_pack(const int32_t *idx, const int32_t *pos, const int32_t *cnt, uint32_t n, uint32_t topk, uint32_t ne,
                 const void *x_bf16, uint32_t hidden, void *send_x, int32_t *send_pos, cudaStream_t st);
int qw6k_ep_expand(const int32_t *recv_cnt, uint32_t world, uint32_t epr, int32_t *row_expert, cudaStream_t st);
int qw6k_ep_combine(const void *ret_bf16, const float *w, const int32_t *send_pos, uint32_t ntok, uint32_t topk,
                    uint32_t hidden, float *out, cudaStream_t st);

/* Expert parallelism over peer memory (k_ep.cu, phases of one layer).
 * Every rank holds one symmetric region with the same layout: signal words
 * (3 kinds x 64 sources, u32 epochs), a double-buffered count matrix
 * [2][world][ne + world] (u32: rows per expert, then unique token rows per
 * owner, each below 2^24 and tagged with the step's epoch in its top 8
 * bits, so that an entry is its own arrival signal), received token rows
 * rx [cap][hidden] (bf16, one per (source, token) pair), per received slot (expert-major) smeta [cap] (i32 pairs:
 * its row in rx, and the destination of its output as source rank * nmax +
 * source assignment), and the returned expert outputs of this rank's own
 * assignments ret [nmax][hidden] (bf16, written by the owners' down GEMM);
 * peers[p] is rank p's region as mapped in this process. */
#define QW6K_EP_MAX_WORLD 64
/* wait kinds (41 + kind is the timeout error); counts need no signal word */
enum { QW6K_EP_SIG_COUNTS = 0, QW6K_EP_SIG_ROWS = 1, QW6K_EP_SIG_DONE = 2 };
typedef struct {
    uint8_t *const *peers; /* device array [world] */
    size_t o_sig, o_cnt, o_rx, o_smeta, o_ret;
    uint32_t rank, world, ne, topk, hidden, ntok, cap, nmax;
    uint32_t *epoch;     /* private: step counter (phase 0 increments it) */
    int *abort;          /* private: set once any wait gives up; later phases do nothing */
    uint32_t *done_ctas; /* private: dispatch completion counter */
    int *err;            /* error word: 41 + phase kind of a wait that timed out */
    const int32_t *idx;  /* [ntok*topk] routing of this rank's tokens */
    const float *w;
    const int32_t *eslot; /* [ne] placed index of each routed expert id: rank eslot / (ne/world) owns it,
                             as its local expert eslot % (ne/world); everything below is in placed ids */
    int32_t *cnt_self, *pos;  /* [ne] rows per placed expert, [ntok*topk] position among its expert's */
    int32_t *ucnt, *upos;     /* [world] unique token rows per owner, [ntok*topk] position of the
                                 assignment's token row among them (-1 - position: a later slot of a
                                 token already sent to that owner) */
    int32_t *sendoff;    /* [ne] first slot of this rank's block for each expert at its owner */
    int32_t *ubase;      /* [world] first rx row of this rank's unique rows at each owner */
    int32_t *local_cnt;  /* [ne/world] rows per local expert this step */
    int32_t *send_row;   /* [ntok*topk] row of each assignment at its owner */
    const void *x;       /* bf16 [ntok][hidden] */
    float *out;          /* fp32 [ntok][hidden] */
    uint64_t wait_ns;    /* limit of every cross-GPU wait (0: 2 s) */
} qw6k_ep_desc;
/* phases: 0 publish counts + wait + plan, 1 dispatch rows + signal,
 * 2 wait for all rows, 3 signal outputs delivered, 4 wait for all outputs,
 * 5 combine (local reads of ret), 6 count (per expert and per owner; runs
 * first) */
int qw6k_ep_p2p_phase(const qw6k_ep_desc *d, int phase, cudaStream_t st);

/* Fixed 1 MiB device scratch (k_static.cu) of the allocation-free MoE entry
 * point; *ptr is its device address on the current device (looked up with
 * cudaGetSymbolAddress on the first call per device, which also configures
 * every decode kernel there). */
/* ---- decode-step executor (k_fwd.cu, k_matvec.cu) ----
 * The token id and position of the step being computed, in device memory;
 * bad is set by the kernels that check for NaN/Inf as qw6 does
 * (qw6_check_nan_inf at qw6.c:2457, 2472, 2487). */
typedef struct {
    uint32_t token, pos;
    int bad;
    uint32_t reserved;
} qw6k_step;
#define QW6K_FA_SPLIT 128 /* sequence chunks per kv head of the attention kernel */
/* out[cols] = row *row_idx of a raw matrix (exact dequant); bad on an index
 * past rows or a NaN/Inf */
int qw6k_dequant_row(uint32_t quant, const void *raw, uint32_t rows, uint32_t cols, const uint32_t *row_idx,
                     float *out, int *bad, cudaStream_t st);
int qw6k_rmsnorm(const float *x, const float *w, float *out, uint32_t dim, cudaStream_t st);
/* Gated DeltaNet token step: proj = [qkv 8192 | z 4096 | beta 32 | alpha 32];
 * ring [4][8192]: row p % 4 holds position p's qkv (zero before position
 * 0); conv_w [8192][4], dt/a [32], dn_norm [128]; state [32][128][128]
 * updated in place; gated [4096] = rmsnorm(o) * silu(z) */
int qw6k_dn_token(const float *proj, const qw6k_step *step, float *ring, const float *conv_w, const float *dt,
                  const float *a, const float *dn_norm, float *state, float *gated, cudaStream_t st);
/* gated attention: proj = [16 x (q 256 | gate 256) | k 512 | v 512]; caches
 * [max_ctx][2][256]; freq[32] = powf(1e7, i / 64) for even i < 64 */
int qw6k_fa_prep(const float *proj, const float *q_norm, const float *k_norm, const float *freq,
                 const qw6k_step *step, float *k_cache, float *v_cache, float *q_rot, cudaStream_t st);
size_t qw6k_fa_part_floats(void);
int qw6k_fa_attn(const float *q_rot, const float *k_cache, const float *v_cache, const qw6k_step *step, float *part,
                 const float *proj, float *attn, cudaStream_t st);
int qw6k_check_finite(const float *x, uint32_t n, int *bad, cudaStream_t st);
/* step->token = the argmax of *key, step->pos += 1 */
int qw6k_step_next(qw6k_step *step, const unsigned long long *key, cudaStream_t st);

#define QW6K_STATIC_SCRATCH_BYTES (1u << 20)
#define QW6K_MAX_DEVICES 64
int qw6k_static_scratch(void **ptr, size_t *bytes);

#ifdef __cplusplus
}
#endif

#endif /* QW6_LAUNCH_H */
