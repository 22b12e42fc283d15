/* qw6_cuda.h -- device-resident API of libqw6cuda (B200 / sm_100a).
 *
 * The per-call qw6_vk_*_host entry points (qw6_vk.h) copy everything from
 * and to host memory on every call.  This API is the persistent form the
 * reference's pipeline uses (weights uploaded once, qw6_vk.c:2920-2958; one
 * queue): a context owns a CUDA stream and a grow-only workspace, all
 * tensors are DEVICE pointers, and calls only enqueue work on the context's
 * stream (synchronize with qw6cu_synchronize).  No torch or C++ types cross
 * this boundary.  Every function returns 0 or a negative error code;
 * qw6cu_last_error() gives a message for the calling thread.
 *
 * Quant codes are qw6's qw6_quant_t values (qw6.h:77-92): Q4_K_M 4,
 * Q4_K_S 5, Q5_K 6, Q6_K 7, IQ3_S 9, IQ2_S 11, IQ2_XXS 13.
 *
 * Weights for the quantized kernels live in the PACKED TILE layout: the
 * GGUF super-blocks of every 16 consecutive rows, byte-permuted so that
 * each GPU lane fetches its tensor-core fragments with 16-byte loads.  The
 * permutation has the same size as the raw bytes, except that the row count
 * is rounded up to a multiple of 16 (qw6cu_packed_bytes).  qw6cu_pack
 * converts raw GGUF rows already on the device.
 */
#ifndef QW6_CUDA_H
#define QW6_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QW6CU_OK 0
#define QW6CU_ERR_ARG (-2)     /* bad shape / pointer / unsupported option */
#define QW6CU_ERR_QUANT (-3)   /* quant type not handled */
#define QW6CU_ERR_CUDA (-4)    /* CUDA runtime or launch failure */
#define QW6CU_ERR_ALIGN (-5)   /* pointer or stride not 16-byte aligned */
#define QW6CU_ERR_TIMEOUT (-6) /* a bounded device-side wait gave up */
#define QW6CU_ERR_NOMEM (-7)   /* device allocation failed */

typedef struct qw6cu_ctx qw6cu_ctx;

/* Message describing the last error of the calling thread. */
const char *qw6cu_last_error(void);

/* Create a context on `device` (-1: $QW6_CUDA_DEVICE, else 0) with its own
 * non-blocking stream. */
int qw6cu_create(qw6cu_ctx **out, int device);
void qw6cu_destroy(qw6cu_ctx *ctx);
/* Make the context enqueue on an external cudaStream_t (NULL: its own). */
int qw6cu_set_stream(qw6cu_ctx *ctx, void *stream);
void *qw6cu_get_stream(qw6cu_ctx *ctx);
int qw6cu_synchronize(qw6cu_ctx *ctx);

/* ---- weights ---- */

/* Bytes of the packed tile layout of one rows x cols matrix (0: invalid). */
size_t qw6cu_packed_bytes(uint32_t quant, uint32_t rows, uint32_t cols);

/* Pack `count` matrices: raw GGUF matrix i at raw + i*raw_stride, packed i
 * written at packed + i*packed_stride (packed_stride >= packed_bytes). */
int qw6cu_pack(qw6cu_ctx *ctx, uint32_t quant, const void *raw, void *packed, uint32_t rows, uint32_t cols,
               uint32_t count, size_t raw_stride, size_t packed_stride);

/* out[rows x cols] fp32 = exact dequantization of RAW GGUF rows, bit-equal
 * to qw6_tensor_dequantize_row (qw6.c:1674-1724). */
int qw6cu_dequantize(qw6cu_ctx *ctx, uint32_t quant, const void *raw, float *out, uint32_t rows, uint32_t cols);

/* ---- matvec ---- */

/* y[t*rows + r] = W[r] . x[t*cols ...] for t < ntok (1..32), W packed.
 * x must be 16-byte aligned. */
int qw6cu_matvec(qw6cu_ctx *ctx, uint32_t quant, const void *packed, const float *x, float *y, uint32_t rows,
                 uint32_t cols, uint32_t ntok);

/* fp32 weights, row-major rows x cols, one token. */
int qw6cu_matvec_f32(qw6cu_ctx *ctx, const float *w, const float *x, float *y, uint32_t rows, uint32_t cols);

/* ---- MoE pieces ---- */

/* Per token t: indices idx[t*top_k ..] and softmax weights w[t*top_k ..]
 * of the top_k largest of logits[t*n_experts ..] (n_experts <= 256,
 * top_k <= 32); ties go to the lower expert index (qw6.c:2796-2827). */
int qw6cu_moe_route(qw6cu_ctx *ctx, const float *logits, uint32_t ntok, uint32_t n_experts, uint32_t top_k,
                    int32_t *idx, float *w);
int qw6cu_silu_mul(qw6cu_ctx *ctx, const float *gate, const float *up, float *out, uint32_t n);
int qw6cu_moe_gather(qw6cu_ctx *ctx, const float *expert_out, const float *w, const float *shared_out,
                     float shared_weight, float *out, uint32_t dim, uint32_t top_k);
/* argmax with qw6_cpu_argmax semantics; idx/val are device pointers. */
int qw6cu_argmax(qw6cu_ctx *ctx, const float *x, uint32_t n, uint32_t *idx, float *val);

/* ---- dense GEMM on the tensor cores ---- */

/* D[M x N] (fp32, row-major) = A[M x K] . B[N x K]^T with bf16 K-major A and
 * B (row-major with K contiguous), on tcgen05 tensor cores with TMEM
 * accumulators.  K % 64 == 0; A, B 16-byte aligned. */
int qw6cu_gemm_bf16_nt(qw6cu_ctx *ctx, const void *A, const void *B, float *D, uint32_t M, uint32_t N, uint32_t K);

/* Synchronize and report whether any kernel of this context gave up a
 * bounded device-side wait since the last check (QW6CU_ERR_TIMEOUT; the
 * affected outputs are invalid).  Waits give up after 2 s instead of hanging. */
int qw6cu_check_device_errors(qw6cu_ctx *ctx);

/* ---- LM head + greedy argmax ---- */

/* Fused output projection and argmax (qw6.c:2493 then qw6_cpu_argmax,
 * qw6.c:2858-2863) over one row shard [row_offset, row_offset + rows) of the
 * vocabulary: keys[t] (device, 8 bytes per token) receives the packed
 * (logit, global row index) maximum of token t's logits over the shard --
 * larger logit first, lower index on ties, NaN handled like the CPU scan.
 * logits (nullable) also receives the rows x ntok logits (token-major).
 * x: [ntok x cols] device fp32, ntok <= 32.  Shards of one vocabulary are
 * combined exactly by taking the max of their keys. */
int qw6cu_lm_head_argmax(qw6cu_ctx *ctx, uint32_t quant, const void *packed, const float *x, uint32_t ntok,
                         uint32_t rows, uint32_t cols, uint32_t row_offset, unsigned long long *keys, float *logits);
/* idx[t] / val[t] (val nullable; device) from the max over nshards of
 * keys[s*ntok + t] -- e.g. after all-gathering every shard's keys. */
int qw6cu_argmax_keys_reduce(qw6cu_ctx *ctx, const unsigned long long *keys, uint32_t nshards, uint32_t ntok,
                             uint32_t *idx, float *val);

/* ---- sampling ---- */

/* token[r] (device) = qw6_sample's pick (qw6.c:2904-2982) over logits row r
 * (device fp32, nrows rows of n, no NaN) with the uniform draw u[r] (device
 * fp32 in [0, 1); qw6 takes it from libc rand()): temp <= 0 is greedy
 * (qw6_cpu_argmax); otherwise scores logits/temp in descending order (lower
 * index first on ties), keep the first top_k (<= 0: all), then the shortest
 * prefix whose probabilities reach top_p (outside (0, 1]: 1), and pick the
 * first item whose running exp(score - max) reaches u * the kept sum -- with
 * no sort and no copy of the logits to the host.  The sums are double, in a
 * different order than qw6's loop: a pick can differ only when u * sum lies
 * within rounding of a cumulative boundary. */
int qw6cu_sample(qw6cu_ctx *ctx, const float *logits, uint32_t n, uint32_t nrows, float temp, float top_p, int top_k,
                 const float *u, uint32_t *token);

/* ---- routed MoE FFN (decode batches) ---- */

/* One GGUF expert pack in the packed tile layout: expert e's matrix starts at
 * base + e*stride (qw6's bind_expert_pack keeps experts at a fixed stride,
 * qw6.c:542-597).  quant is the pack's qw6_quant_t. */
typedef struct {
    uint32_t quant;
    const void *base;
    size_t stride;
} qw6cu_expert_pack;

/* out[t] = sum over the top_k experts e of token t (routing of
 * logits[t*n_experts ..], qw6.c:2796-2827) of w_e * down_e(silu(gate_e x_t) *
 * up_e x_t), composed as qw6_apply_layer_moe (qw6.c:2246-2264) without the
 * shared expert.  gate/up are [inter x hidden], down [hidden x inter];
 * gate and up must share one quant type.  ntok * top_k <= 4096; hidden and
 * inter multiples of 256 (512 when ntok > 4), hidden <= 4096; n_experts <= 256.  Routing,
 * grouping and the expert matvecs all run on the device (no host sync).
 * Uses the context workspace (grown on first use, which synchronizes). */
int qw6cu_moe_decode(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                     const qw6cu_expert_pack *down, const float *logits, const float *x, float *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k);

/* Same computation with HOST logits/x/out (copied in and out on the
 * context stream); synchronous: returns after out is written. */
int qw6cu_moe_decode_hostio(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                            const qw6cu_expert_pack *down, const float *logits, const float *x, float *out,
                            uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k);

/* Allocation-free qw6cu_moe_decode, for callers that cannot allocate device
 * memory at the point where they run the layer: a runtime or serving process
 * that hands out all device memory from its own pool, or one whose
 * device-memory footprint must stay fixed after start-up (an allocation there
 * can fail, or stall on device-wide synchronisation, at a point where neither
 * is acceptable).  It has no counterpart in the reference.  Scratch is a fixed
 * 1 MiB array in device memory that the library owns (every GPU that loads
 * the library holds it until the process exits), so shapes whose workspace
 * (qw6cu_moe_workspace_bytes) exceeds 1 MiB are rejected with QW6CU_ERR_ARG
 * -- for hidden 2048, inter 512, 256 experts, top-8 that is ntok > 12.
 * Inputs, outputs and weights are device pointers owned by the caller; work is
 * enqueued on `stream` (a cudaStream_t, NULL = the legacy default stream) on
 * the calling thread's current device.  The first call on a device does a
 * one-time set-up there: it looks up the array's device address
 * (cudaGetSymbolAddress) and configures and loads every kernel this entry
 * point can launch; make that first call before any stream capture.  Every
 * call shares the array and leaves its contents behind; nothing in it needs
 * to start at zero because each call writes every scratch byte it later
 * reads.  Calls that can overlap on the GPU (different streams, or graphs
 * replayed concurrently) race on the array and must be serialized by the
 * caller. */
int qw6cu_moe_decode_noalloc(const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                             const qw6cu_expert_pack *down, const float *logits, const float *x, float *out,
                             uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k,
                             void *stream);

/* ---- the MoE FFN block (decode batches) ---- */

/* The shared expert of a MoE layer: gate/up [inter x hidden] and down
 * [hidden x inter], each in the packed tile layout of its quant type
 * (qw6cu_pack) or FP16/BF16 row-major; router: fp32 [hidden] (its sigmoid
 * weighs the shared expert) or NULL (weight 1), as qw6.c:2266-2285. */
typedef struct {
    uint32_t gate_quant, up_quant, down_quant;
    const void *gate, *up, *down;
    uint32_t inter;
    const float *router;
} qw6cu_shared_expert;

/* One MoE FFN block for ntok token rows, as qw6's forward pass applies it
 * to every layer (qw6.c:2474-2484 around qw6_apply_layer_moe,
 * qw6.c:2226-2290):
 *   normed = rmsnorm(x) * norm_w (eps 1e-6), logits = router . normed,
 *   ffn = routed experts (qw6cu_moe_decode on normed and logits)
 *         + s * shared_down(silu(shared_gate normed) * shared_up normed),
 *   out = x + ffn.
 * router (and shared->router): fp32 [n_experts x hidden] row-major, 16-byte
 * aligned; norm_w fp32
 * [hidden]; shared: NULL for none.  x, out: fp32 [ntok x hidden]; all device
 * pointers, enqueued on the context's stream with no host synchronization
 * (the context workspace is grown on first use, which synchronizes).  The
 * router logits are computed in fp32 like qw6's, but with a different
 * summation order, so a token whose k-th and (k+1)-th logits differ by
 * rounding only may select a different expert than the CPU. */
int qw6cu_moe_block(qw6cu_ctx *ctx, const float *x, const float *norm_w, const float *router,
                    const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up, const qw6cu_expert_pack *down,
                    const qw6cu_shared_expert *shared, float *out, uint32_t ntok, uint32_t hidden, uint32_t inter,
                    uint32_t n_experts, uint32_t top_k);

/* Device workspace qw6cu_moe_decode needs for these dimensions. */
size_t qw6cu_moe_workspace_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts,
                                 uint32_t top_k);

/* ---- routed MoE FFN (prefill batches, tensor cores) ---- */

/* The same layer as qw6cu_moe_decode for large token batches, as grouped
 * GEMMs on the tcgen05 tensor cores: tokens are grouped by selected expert,
 * each expert's packed Q4_K/Q6_K rows are dequantized to bf16 tiles in shared
 * memory and multiplied against the expert's bf16 token rows (fp32
 * accumulation in TMEM); silu(g)*u is kept in bf16; the down projection
 * writes every assignment's bf16 expert output and a combine sums
 * w_e * output in slot order with fp32 fma, so results do not depend on
 * scheduling.  x_bf16: [ntok x hidden] bf16 (device); out: fp32
 * [ntok x hidden], overwritten; both 16-byte aligned.  Tolerance vs the fp32 CPU composition:
 * 2e-2.  gate/up/down quant: Q4_K or Q6_K; hidden, inter multiples of 256. */
int qw6cu_moe_prefill(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                      const qw6cu_expert_pack *down, const float *logits, const void *x_bf16, float *out,
                      uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k);
size_t qw6cu_moe_prefill_workspace_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts,
                                         uint32_t top_k);

/* qw6cu_moe_prefill over n_batches batches of ntok tokens in HOST memory:
 * batch b reads logits[b] (fp32 [ntok x n_experts]) and x_bf16[b] (bf16
 * [ntok x hidden]) and writes out[b] (fp32 [ntok x hidden]); entries may
 * repeat.  Every batch is copied in, run and copied back, pipelined over two
 * device slots and two copy streams: the copy-in of batch b+1 and the
 * read-back of batch b-1 run while the experts of batch b run on the context
 * stream, so a long call streams at the rate of the slowest of the three.
 * The copies overlap only from page-locked host memory (cudaHostAlloc /
 * cudaHostRegister); pageable buffers give the same results, serialized.
 * Synchronous: returns once every out[b] is written (or on the first error).
 * Each batch's result is bit for bit that of qw6cu_moe_prefill. */
int qw6cu_moe_prefill_hostio(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                             const qw6cu_expert_pack *down, const float *const *logits, const void *const *x_bf16,
                             float *const *out, uint32_t n_batches, uint32_t ntok, uint32_t hidden, uint32_t inter,
                             uint32_t n_experts, uint32_t top_k);

/* Expert-parallel building block: the same grouped GEMMs with the routing
 * supplied per row instead of computed from logits.  Row r of x_bf16
 * ([nrows x hidden], device) is sent through expert row_expert[r] (an index
 * into these packs, < n_experts) and out_bf16[r] (bf16 [nrows x hidden],
 * overwritten) = down(silu(gate x_r) * up x_r), unweighted -- bit for bit the
 * per-assignment expert output qw6cu_moe_prefill forms before its combine.
 * Used on the rank that owns the experts after an all-to-all dispatch of
 * token rows. */
int qw6cu_moe_expert_rows(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                          const qw6cu_expert_pack *down, const void *x_bf16, const int32_t *row_expert,
                          void *out_bf16, uint32_t nrows, uint32_t hidden, uint32_t inter, uint32_t n_experts);

/* ---- expert parallelism (prefill) ----
 * Experts are sharded contiguously over `world` ranks: rank r owns experts
 * [r*experts_per_rank, (r+1)*experts_per_rank).  One layer on a rank:
 *   qw6cu_moe_route -> qw6cu_ep_count -> all-to-all of expert_count (each
 *   rank receives the counts of its own experts from every source) ->
 *   qw6cu_ep_pack -> all-to-all of the send rows -> qw6cu_ep_expand ->
 *   qw6cu_moe_expert_rows on the received rows (local packs) -> all-to-all
 *   of the bf16 expert outputs back in send-row order -> qw6cu_ep_combine.
 * The result equals qw6cu_moe_prefill on the same tokens: the same expert
 * outputs, weighted and summed in the same slot order.  (qw6_b200/ep.py runs
 * this with NCCL.) */

/* expert_count[n_experts] (zeroed here) = assignments routed to each global
 * expert; pos[a] = position of assignment a among those of its expert. */
int qw6cu_ep_count(qw6cu_ctx *ctx, const int32_t *idx, uint32_t nassign, uint32_t n_experts, int32_t *expert_count,
                   int32_t *pos);
/* Send row p = (exclusive prefix of expert_count)[idx[a]] + pos[a] gets the
 * token row (bf16, hidden) of assignment a = t*top_k + k; send_pos[a] = p.
 * Send rows are sorted by global expert, hence grouped by destination rank
 * and, inside each destination's block, by its local expert. */
int qw6cu_ep_pack(qw6cu_ctx *ctx, const int32_t *idx, const int32_t *pos, const int32_t *expert_count,
                  uint32_t nassign, uint32_t top_k, uint32_t n_experts, const void *x_bf16, uint32_t hidden,
                  void *send_x, int32_t *send_pos);
/* recv_count[s*experts_per_rank + e] rows from source rank s for local
 * expert e arrive in (s, e) order; row_expert[r] (overwritten) = e of
 * received row r.  world * experts_per_rank <= 256. */
int qw6cu_ep_expand(qw6cu_ctx *ctx, const int32_t *recv_count, uint32_t world, uint32_t experts_per_rank,
                    int32_t *row_expert);
/* out[t] (fp32, overwritten) = sum_k w[t*top_k+k] * ret_bf16[send_pos[t*top_k+k]]
 * as fp32 fma in slot order k (the single-GPU prefill combine). */
int qw6cu_ep_combine(qw6cu_ctx *ctx, const void *ret_bf16, const float *w, const int32_t *send_pos, uint32_t ntok,
                     uint32_t top_k, uint32_t hidden, float *out);

/* ---- expert parallelism over peer memory (prefill) ----
 * The same layer with no host round trip: one qw6cu_ep per rank (one
 * process per GPU) owns a symmetric device region that the other ranks map
 * through CUDA IPC.  Counts, token rows and expert outputs move through
 * peer memory (NVLink), ordered by epoch-stamped signal words; every wait
 * gives up after 2 s, records a timeout in the context's error word
 * (qw6cu_check_device_errors) and turns the rest of the layer into no-ops.
 * Setup: qw6cu_ep_create on every rank -> qw6cu_ep_handle -> all-gather the
 * handles in rank order -> qw6cu_ep_connect.  Then every rank calls
 * qw6cu_ep_layer once per layer step, in the same order; the call enqueues
 * all its kernels on the context's stream without synchronising, so a step
 * can be captured in a CUDA graph.  The result equals qw6cu_moe_prefill on
 * the union of the ranks' tokens, bit for bit. */
typedef struct qw6cu_ep qw6cu_ep;
/* bytes of one rank's handle (a cudaIpcMemHandle_t) */
size_t qw6cu_ep_handle_bytes(void);
/* Experts are sharded contiguously (n_experts / world per rank) unless
 * qw6cu_ep_set_placement says otherwise; up to max_tokens tokens per rank
 * and call.  Allocates the symmetric region
 * (2 * world * max_tokens * top_k * hidden * 2 bytes plus signals/counts)
 * and the private buffers. */
int qw6cu_ep_create(qw6cu_ctx *ctx, uint32_t rank, uint32_t world, uint32_t n_experts, uint32_t top_k,
                    uint32_t hidden, uint32_t inter, uint32_t max_tokens, qw6cu_ep **out);
int qw6cu_ep_handle(qw6cu_ep *ep, void *handle);
/* handles: world x qw6cu_ep_handle_bytes(), in rank order (own entry ignored) */
int qw6cu_ep_connect(qw6cu_ep *ep, const void *handles);
/* Expert placement (the same on every rank): experts[r * epr + j] is the
 * routed expert id that rank r holds as its local expert j, epr =
 * n_experts / world; a permutation of 0 .. n_experts-1.  Balancing the
 * ranks' rows by placing experts from routing statistics evens out the
 * grouped GEMMs without changing any output bit.  Synchronises the
 * context's stream; call between steps, with each rank's packs reordered
 * to match. */
int qw6cu_ep_set_placement(qw6cu_ep *ep, const uint32_t *experts);
/* gate/up/down: this rank's experts (local index 0 .. n_experts/world - 1);
 * logits fp32 [ntok x n_experts], x bf16 [ntok x hidden], out fp32 [ntok x
 * hidden] -- this rank's tokens, device memory; ntok <= max_tokens. */
int qw6cu_ep_layer(qw6cu_ep *ep, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                   const qw6cu_expert_pack *down, const float *logits, const void *x_bf16, float *out,
                   uint32_t ntok);
/* qw6cu_ep_layer over n_batches layer steps whose inputs and outputs are
 * in HOST memory (this rank's tokens; arrays of one host address per step),
 * pipelined as qw6cu_moe_prefill_hostio: the copy-in of step b+1 and the
 * read-back of step b-1 run beside step b.  Every rank makes the same call
 * with the same n_batches.  Synchronous: returns once every out[b] is
 * written (or on the first error). */
int qw6cu_ep_layer_hostio(qw6cu_ep *ep, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                          const qw6cu_expert_pack *down, const float *const *logits, const void *const *x_bf16,
                          float *const *out, uint32_t n_batches, uint32_t ntok);
/* Limit of every cross-GPU wait of this endpoint's later layers, in ms
 * (default 2000): a rank whose peer stops taking part gives up after it,
 * records the wait kind in the context's error word (41 counts, 42 rows,
 * 43 outputs; qw6cu_check_device_errors returns QW6CU_ERR_TIMEOUT) and skips
 * the rest of the layer. */
int qw6cu_ep_set_wait_limit(qw6cu_ep *ep, uint32_t ms);
/* rows this rank's experts processed in the last layer (synchronises) */
int qw6cu_ep_last_rows(qw6cu_ep *ep, uint32_t *rows);
void qw6cu_ep_destroy(qw6cu_ep *ep);

/* ---- GGUF files ----
 * qw6 keeps its model in one GGUF (v3) file (qw6.c:871-1240).  These calls
 * read its tensor table from a memory mapping of the file and upload tensors
 * to the GPU in the layout the kernels read; they synchronize the context's
 * stream. */
typedef struct qw6cu_gguf qw6cu_gguf;
typedef struct {
    const char *name;      /* owned by the qw6cu_gguf */
    uint32_t n_dims;
    uint64_t dims[4];      /* dims[0] = columns (contiguous), dims[1] = rows, dims[2] = experts */
    uint32_t ggml_type;
    int quant;             /* qw6_quant_t of the ggml type (qw6.c:1079-1094), -1 if qw6 has none */
    uint64_t file_offset;  /* absolute, aligned */
    uint64_t bytes;        /* data bytes (0 for an unknown type) */
    const void *data;      /* inside the mapping */
} qw6cu_gguf_tensor;
/* Parse header, metadata (general.alignment) and tensor table; every tensor
 * of a known type must fit in the file. */
int qw6cu_gguf_open(const char *path, qw6cu_gguf **out);
void qw6cu_gguf_close(qw6cu_gguf *g);
uint32_t qw6cu_gguf_tensor_count(const qw6cu_gguf *g);
int qw6cu_gguf_tensor_info(const qw6cu_gguf *g, uint32_t i, qw6cu_gguf_tensor *info);
/* index of the tensor called name, or -1 */
int qw6cu_gguf_find(const qw6cu_gguf *g, const char *name);
/* Device bytes tensor i takes uploaded (0: not uploadable): block formats in
 * the packed tile layout, FP16/BF16 and FP32 rows as stored; a 3-D tensor
 * [cols, rows, n] holds n matrices at a 256-byte aligned stride. */
size_t qw6cu_gguf_upload_bytes(const qw6cu_gguf *g, uint32_t i);
/* Upload tensor i to dst (device, 256-byte aligned, >= upload_bytes); *out
 * receives its quant, base and per-matrix stride -- for an expert pack the
 * qw6cu_expert_pack the MoE calls take (qw6's bind_expert_pack addressing,
 * qw6.c:542-597, with the packed stride). */
int qw6cu_gguf_upload(qw6cu_ctx *ctx, const qw6cu_gguf *g, uint32_t i, void *dst, size_t dst_bytes,
                      qw6cu_expert_pack *out);
/* The routed-expert tensors of layers 0 .. n_layers-1 (blk.L.ffn_gate_exps,
 * ffn_up_exps, ffn_down_exps) in one device allocation, and the table of
 * their packs: packs[3 * L + k] for k = gate, up, down, on the host and as
 * a device array of qw6cu_expert_pack for kernels that pick a layer's packs
 * on the GPU. */
typedef struct {
    uint32_t n_layers;
    qw6cu_expert_pack *packs;  /* host [n_layers * 3] */
    void *packs_dev;           /* device copy of packs */
    void *weights;             /* device allocation holding every pack */
    size_t bytes;
} qw6cu_moe_table;
int qw6cu_gguf_upload_moe(qw6cu_ctx *ctx, const qw6cu_gguf *g, uint32_t n_layers, qw6cu_moe_table *tab);
void qw6cu_moe_table_free(qw6cu_moe_table *tab);

/* ---- decode-step executor ----
 * qw6's per-token forward pass (qw6_forward_token, qw6.c:2426-2500; the
 * reference's GPU pipeline is qw6_vk_pipe_forward, qw6_vk.c:3041-3462) with
 * every weight resident on the device and one CUDA graph per step: the
 * embedding row, 40 (n_layers) decoder layers -- Gated DeltaNet token mixing
 * on layers l % 4 != 3, gated GQA attention with RoPE and a KV cache on
 * l % 4 == 3, then the MoE FFN block -- the final norm, the LM head and the
 * greedy argmax.  Dimensions are qw6's (qw6.h:24-55): hidden 2048, 256
 * experts (top 8, inter 512), shared expert inter 512.
 *
 * The model is given as a list of host tensors, raw GGUF rows as qw6's
 * qw6_tensor_t holds them (field = the tensor's role, the fields of
 * qw6_model_t's layers, qw6.h:126-170; layer -1 for the model-level ones).
 * Expert packs give the first expert and the byte stride between experts
 * (bind_expert_pack, qw6.c:542-597).  Tensors sharing one host pointer are
 * uploaded once. */
enum {
    QW6CU_F_NORM = 0, QW6CU_F_POST_NORM, QW6CU_F_ATTN_Q, QW6CU_F_ATTN_K, QW6CU_F_ATTN_V, QW6CU_F_ATTN_O,
    QW6CU_F_ATTN_Q_NORM, QW6CU_F_ATTN_K_NORM, QW6CU_F_ATTN_GATE, QW6CU_F_CONV1D, QW6CU_F_DN_OUT, QW6CU_F_DN_NORM,
    QW6CU_F_DN_ALPHA, QW6CU_F_DN_BETA, QW6CU_F_DN_DT, QW6CU_F_DN_A, QW6CU_F_MOE_ROUTER, QW6CU_F_SHARED_ROUTER,
    QW6CU_F_SHARED_GATE, QW6CU_F_SHARED_UP, QW6CU_F_SHARED_DOWN, QW6CU_F_EXPERT_GATE, QW6CU_F_EXPERT_UP,
    QW6CU_F_EXPERT_DOWN,
    QW6CU_F_TOK_EMBD = 100, QW6CU_F_OUTPUT, QW6CU_F_OUTPUT_NORM
};
typedef struct {
    uint32_t field;
    int32_t layer;         /* -1 for QW6CU_F_TOK_EMBD / OUTPUT / OUTPUT_NORM */
    uint32_t quant;        /* qw6_quant_t */
    uint32_t rows, cols;   /* of one matrix; vectors are one row */
    const void *data;      /* host memory */
    size_t stride;         /* expert packs: bytes from one expert to the next */
} qw6cu_model_tensor;
/* Shapes (rows x cols) it checks: norm, post_norm, output_norm 1 x 2048;
 * DeltaNet layers: attn_q (qkv) 8192 x 2048, attn_gate (z) 4096 x 2048,
 * dn_beta, dn_alpha 32 x 2048, dn_out 2048 x 4096, conv1d 8192 x 4 FP32,
 * dn_dt, dn_a 1 x 32, dn_norm 1 x 128; attention layers: attn_q 8192 x 2048
 * (q and gate per head), attn_k, attn_v 512 x 2048, attn_o 2048 x 4096,
 * attn_q_norm, attn_k_norm 1 x 256; every layer: moe_router 256 x 2048,
 * experts 512 x 2048 (gate, up) and 2048 x 512 (down), optional shared
 * expert 512 x 2048, 512 x 2048, 2048 x 512 and shared_router 1 x 2048;
 * tok_embd V' x 2048, output V x 2048 (V <= 248320 logits per step).
 * Weight matrices: the six block formats, FP16, BF16 (FP32 for the small
 * projections); vectors and the router: any format qw6 dequantizes. */
typedef struct qw6cu_decoder qw6cu_decoder;
/* Upload the model, allocate the recurrent state for positions < max_ctx,
 * run one step to set everything up, capture the step graph and clear the
 * state.  Synchronizes the context's stream. */
int qw6cu_decoder_create(qw6cu_ctx *ctx, const qw6cu_model_tensor *tensors, uint32_t n_tensors, uint32_t n_layers,
                         uint32_t max_ctx, qw6cu_decoder **out);
/* One step: token at position pos (0 .. max_ctx-1; the DeltaNet state moves
 * on by one token per call, as qw6's does).  logits (host, output rows
 * floats) and greedy (host: the argmax, lowest index on ties, as
 * qw6_cpu_argmax) are optional.  Synchronous; QW6CU_ERR_CUDA with
 * "non-finite" in qw6cu_last_error() when the hidden state or the logits
 * hold a NaN/Inf, as qw6's forward returns -1 (qw6.c:2457-2498). */
int qw6cu_decoder_forward(qw6cu_decoder *dec, uint32_t token, uint32_t pos, float *logits, uint32_t *greedy);
/* n greedy steps from token at pos with no host round trip between them
 * (each step's argmax is the next step's token, on the device); tokens
 * (host, n) receives the picked ids. */
int qw6cu_decoder_generate(qw6cu_decoder *dec, uint32_t token, uint32_t pos, uint32_t n, uint32_t *tokens);
/* Device logits of the last step (fp32, *rows of them), e.g. for
 * qw6cu_sample. */
const float *qw6cu_decoder_logits(qw6cu_decoder *dec, uint32_t *rows);
/* Clear the DeltaNet states, conv windows and KV caches (a new sequence). */
int qw6cu_decoder_reset(qw6cu_decoder *dec);
/* Device bytes the decoder holds (weights + state + scratch). */
size_t qw6cu_decoder_device_bytes(const qw6cu_decoder *dec);
void qw6cu_decoder_destroy(qw6cu_decoder *dec);

/* ---- profiling ----
 * Per-launch CUDA events around every kernel this context enqueues (the
 * counterpart of qw6's QW6_PROFILE timestamp queries, qw6_vk.c:2315-2357).
 * begin: allocate events for up to max_launches launches and start
 * recording; end: synchronize, then write per-kernel-id total milliseconds
 * and launch counts into arrays of QW6CU_NKERNELS entries and stop. */
#define QW6CU_NKERNELS 21
int qw6cu_profile_begin(qw6cu_ctx *ctx, uint32_t max_launches);
int qw6cu_profile_end(qw6cu_ctx *ctx, double *ms_total, uint32_t *launches);
const char *qw6cu_kernel_name(int kernel_id);

#ifdef __cplusplus
}
#endif

#endif /* QW6_CUDA_H */
