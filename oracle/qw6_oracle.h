/* qw6_oracle.h -- CPU restatement of qw6's quantized-matvec + MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the parity tests, smoke()
 * and bench.py's cpu_baseline leg compare the CUDA library against; no
 * product code path may link or call it.
 *
 * Every function restates one function of qw6's CPU reference (qw6.c) with
 * the same floating-point evaluation order, so that dequantized weights are
 * bit-identical and fp32 matvec results follow the same single-accumulator
 * sequence.  Pinning: tests/test_oracle.py checks these functions against
 * (a) qw6's own code compiled from its sources into oracle/_ref (bit-exact
 * dequant, identical matvec/routing), (b) the committed fixtures in
 * tests/golden/ that were produced by that build, and (c) the closed-form
 * known-answer tests of qw6's Vulkan self-test (qw6_vk.c:1609-1954).
 *
 * Build: oracle/Makefile with -std=c11 -O2 -ffp-contract=off (no FMA
 * contraction, as in the reference's x86-64 build).
 */
#ifndef QW6_ORACLE_H
#define QW6_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* qw6_fp16_to_f32, qw6.c:1448-1471 (exact, subnormals normalised). */
float qo_fp16_to_f32(uint16_t h);

/* qw6_tensor_dequantize_row, qw6.c:1674-1724.  w is the whole matrix
 * (rows x cols), row selects the row.  Returns 0, or -1 for an unsupported
 * quant / bad shape (the reference returns -1 for Q8_0 and IQ2_M too). */
int qo_dequantize_row(uint32_t quant, const void *w, uint32_t cols,
                      uint32_t row, float *dst);

/* qw6_tensor_matvec, qw6.c:1769-1791: per row, dequantize then a single
 * sequential fp32 accumulator.  y[rows]. */
int qo_matvec(uint32_t quant, const void *w, const float *x, float *y,
              uint32_t rows, uint32_t cols);

/* Same dequantized weights, double accumulation (error reference). */
int qo_matvec_f64(uint32_t quant, const void *w, const float *x, double *y,
                  uint32_t rows, uint32_t cols);

/* Batched form: y[t*rows + r] = W[r] . x[t*cols : ...] for t < ntok. */
int qo_matvec_batch(uint32_t quant, const void *w, const float *x, float *y,
                    uint32_t rows, uint32_t cols, uint32_t ntok);

/* qw6_cpu_moe_route, qw6.c:2796-2827: top_k by repeated strict-greater
 * argmax (ties -> lower index), softmax over the selected logits. */
int qo_moe_route(const float *logits, uint32_t n_experts, uint32_t top_k,
                 int32_t *idx, float *w);

/* qw6_cpu_argmax, qw6.c:2858-2863: strict '>' so the lowest index wins. */
int32_t qo_argmax(const float *x, uint32_t n);

/* moe_gather semantics (vulkan/moe_gather.comp:17-29):
 * out[i] = sum_e w[e]*expert_out[e*dim+i] (+ shared_weight*shared[i]). */
void qo_moe_gather(const float *expert_out, const float *w,
                   const float *shared_out, float shared_weight, float *out,
                   uint32_t dim, uint32_t top_k);

/* silu_mul semantics (qw6.c:2258 with qw6_silu, qw6.h:292-294). */
void qo_silu_mul(const float *gate, const float *up, float *out, uint32_t n);

/* Routed MoE FFN for ntok tokens, composed as qw6_apply_layer_moe does
 * (qw6.c:2246-2264) without the shared expert:
 *   route(logits[t]) -> for each selected e in selection order:
 *   g = Wg[e].x, u = Wu[e].x, mid = silu(g)*u, d = Wd[e].mid, out += w_e*d.
 * Expert e's matrices start at base + e*stride (bind_expert_pack,
 * qw6.c:542-597).  Gate/up are [inter x hidden], down is [hidden x inter].
 * idx_out/w_out (optional, [ntok*top_k]) receive the routing. */
typedef struct {
    uint32_t quant;
    const void *base;
    size_t stride;
} qo_expert_pack;

int qo_moe_layer(const qo_expert_pack *gate, const qo_expert_pack *up,
                 const qo_expert_pack *down, const float *logits,
                 const float *x, float *out, uint32_t ntok,
                 uint32_t hidden, uint32_t inter, uint32_t n_experts,
                 uint32_t top_k, int32_t *idx_out, float *w_out);

/* Same composition in double precision on the bit-exact weights (error
 * reference for the fp32 and bf16 paths). Routing uses the fp32 rule. */
int qo_moe_layer_f64(const qo_expert_pack *gate, const qo_expert_pack *up,
                     const qo_expert_pack *down, const float *logits,
                     const float *x, double *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t n_experts,
                     uint32_t top_k);

/* qw6_cpu_rmsnorm, qw6.c:2502-2512: ss = sum x[i]^2 (one fp32
 * accumulator), scale = 1 / sqrtf(ss / dim + 1e-6f) (QW6_RMS_EPS,
 * qw6.h:67), out[i] = x[i] * scale * weight[i] evaluated left to right. */
void qo_rmsnorm(const float *x, const float *weight, float *out, uint32_t dim);

/* One dense matrix of a block (FP32/FP16/BF16 or a GGUF block format),
 * rows x cols as its use implies. */
typedef struct {
    uint32_t quant;
    const void *w;
} qo_matrix;

/* The MoE FFN block as qw6's forward pass runs it around
 * qw6_apply_layer_moe (qw6.c:2474-2484, 2226-2290), per token t:
 *   normed = rmsnorm(x[t], norm_w)
 *   logits = router . normed                (router: [n_experts x hidden])
 *   ffn    = routed experts on normed       (as qo_moe_layer)
 *   with a shared expert (sgate, sup: [shared_inter x hidden], sdown:
 *   [hidden x shared_inter]): s = sigmoid(srouter . normed), or 1 without
 *   srouter ([1 x hidden]); ffn[i] += s * (sdown . (silu(sgate . normed) *
 *   (sup . normed)))[i]
 *   out[t][i] = x[t][i] + ffn[i]            (the residual add)
 * sgate/sup/sdown: all or none (NULL). */
int qo_moe_block(const float *x, const float *norm_w, const qo_matrix *router,
                 const qo_expert_pack *gate, const qo_expert_pack *up,
                 const qo_expert_pack *down, const qo_matrix *sgate,
                 const qo_matrix *sup, const qo_matrix *sdown,
                 const qo_matrix *srouter, float *out, uint32_t ntok,
                 uint32_t hidden, uint32_t inter, uint32_t shared_inter,
                 uint32_t n_experts, uint32_t top_k);

/* The same block in double precision on the bit-exact weights (error
 * reference): RMSNorm, the expert and shared-expert contractions, the
 * sigmoid gate and the residual in double; the experts and their weights
 * are chosen by the fp32 rule on the fp32 router logits (qo_rmsnorm +
 * qo_matvec), so both forms route identically. */
int qo_moe_block_f64(const float *x, const float *norm_w, const qo_matrix *router,
                     const qo_expert_pack *gate, const qo_expert_pack *up,
                     const qo_expert_pack *down, const qo_matrix *sgate,
                     const qo_matrix *sup, const qo_matrix *sdown,
                     const qo_matrix *srouter, double *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t shared_inter,
                     uint32_t n_experts, uint32_t top_k);

/* qw6_sample, qw6.c:2904-2982, with its one uniform draw u in [0, 1) given
 * (qw6 takes it from libc: (float)rand() / ((float)RAND_MAX + 1.0f)):
 * temp <= 0 -> argmax; else scores logits/temp (fp32) sorted descending
 * (ties: lower index first), top_k (<= 0: all) limits them, top_p
 * (outside (0, 1]: 1) takes the shortest prefix whose double-precision
 * probabilities reach it, and the token is the first whose cumulative
 * exp(score - max) reaches u * (sum over the kept prefix). */
int32_t qo_sample(const float *logits, uint32_t n, float temp, float top_p, int top_k, float u);

/* ---- the per-token forward pass (qw6_forward_token, qw6.c:2426-2500) ----
 * One tensor of qw6's model as qw6_tensor_t carries it: raw GGUF rows of
 * `cols` values (quant = qw6_quant_t), `rows` of them; for the expert packs
 * expert e's matrix starts at data + e * stride (bind_expert_pack,
 * qw6.c:542-597).  Vectors (norm weights, dt bias, a) are one row. */
typedef struct {
    uint32_t quant, rows, cols;
    const void *data;
    size_t stride;
} qo_tensor;

/* Per-layer tensors, in the roles of qw6_model_t's layer fields (qw6.h:126-170);
 * the linear-attention layers keep their qkv projection in ATTN_Q and the
 * output gate z in ATTN_GATE, as qw6's GGUF binding does (qw6.c:599-680). */
enum {
    QO_F_NORM = 0, QO_F_POST_NORM, QO_F_ATTN_Q, QO_F_ATTN_K, QO_F_ATTN_V, QO_F_ATTN_O, QO_F_ATTN_Q_NORM,
    QO_F_ATTN_K_NORM, QO_F_ATTN_GATE, QO_F_CONV1D, QO_F_DN_OUT, QO_F_DN_NORM, QO_F_DN_ALPHA, QO_F_DN_BETA,
    QO_F_DN_DT, QO_F_DN_A, QO_F_MOE_ROUTER, QO_F_SHARED_ROUTER, QO_F_SHARED_GATE, QO_F_SHARED_UP,
    QO_F_SHARED_DOWN, QO_F_EXPERT_GATE, QO_F_EXPERT_UP, QO_F_EXPERT_DOWN, QO_NF
};
#define QO_FWD_HIDDEN 2048

typedef struct {
    uint32_t n_layers;       /* qw6 runs 40; layer l is full attention when l % 4 == 3 */
    qo_tensor tok_embd, output, output_norm;
    const qo_tensor *layers; /* [n_layers][QO_NF] */
} qo_model;

int qo_fwd_is_full(uint32_t layer);
/* floats of the recurrent state of n_layers layers: per DeltaNet layer its
 * [32][128][128] state and [4][8192] conv window, per attention layer its
 * key and value caches of max_ctx positions ([max_ctx][2][256] each);
 * zero it before position 0 */
size_t qo_fwd_state_floats(uint32_t n_layers, uint32_t max_ctx);
/* logits[output.rows] of token at position pos; -1 on bad input or, as qw6,
 * on a NaN/Inf in the hidden state or the logits */
int qo_forward(const qo_model *m, float *state, uint32_t max_ctx, uint32_t token, uint32_t pos, float *logits);

#ifdef __cplusplus
}
#endif

#endif /* QW6_ORACLE_H */
