/* qw6_vk.h -- drop-in replacement of qw6's Vulkan backend header, backed by
 * libqw6cuda (hand-written CUDA for B200 / sm_100a).
 *
 * Every prototype below keeps the name, argument order and meaning of the
 * declaration in qw6's own qw6_vk.h, so qw6.c links against libqw6cuda.so
 * with -DQW6_VULKAN unchanged.  Conventions kept from the reference
 * (qw6_vk.c:1186-1362):
 *   - all pointers are caller-owned HOST memory; the call is synchronous and
 *     the result is in the output buffer when it returns;
 *   - return 0 on success, -1 on any error (bad shape, unsupported
 *     argument, CUDA failure); qw6cu_last_error() (qw6_cuda.h) describes it;
 *   - `w` of the quantized matmuls is raw GGUF super-block bytes, row-major,
 *     rows * (cols/256) * block_bytes; cols must be a multiple of 256.
 * Difference: the reference brings a Vulkan device up and down on every
 * call (qw6_vk.c:1195-1202); here the first call creates one process-wide
 * CUDA context (device QW6_CUDA_DEVICE, default 0) that later calls reuse.
 * Calls are serialized by an internal mutex.  There is no CPU fallback:
 * without a usable GPU every entry point returns -1.
 */
#ifndef QW6_VK_H
#define QW6_VK_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* qw6_vk.h:9 -- runs the known-answer tests of this library on the GPU;
 * returns 0 when all pass (the reference returns 0/1 the same way). */
int qw6_vk_selftest(void);

/* qw6_vk.h:10-11 -- y[rows] = W[rows x cols] (fp32) . x[cols]. */
int qw6_vk_matvec_f32_host(const float *w, const float *x, float *y, uint32_t rows, uint32_t cols);

/* qw6_vk.h:12-19 -- fused GGUF dequant + matvec, Q4_K / Q5_K / Q6_K /
 * IQ2_XXS (dispatch of qw6_vk_pipe_matvec, qw6_vk.c:2386-2430). */
int qw6_vk_matmul_q4k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);
int qw6_vk_matmul_q5k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);
int qw6_vk_matmul_q6k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);
int qw6_vk_matmul_iq2xxs_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);

/* Added: the reference reaches IQ2_S and IQ3_S only through its pipeline
 * dispatch (qw6_vk.c:2414-2425) and declares no host entry for them. */
int qw6_vk_matmul_iq2s_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);
int qw6_vk_matmul_iq3s_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols);

/* qw6_vk.h:24-25 -- out[i] = silu(gate[i]) * up[i]. */
int qw6_vk_silu_mul_host(const float *gate, const float *up, float *out, uint32_t n);

/* qw6_vk.h:26-27 -- index and value of the maximum (lowest index on ties). */
int qw6_vk_argmax_host(const float *x, uint32_t n, uint32_t *out_idx, float *out_val);

/* qw6_vk.h:28-29 -- greedy token = argmax(logits); error when n == 0. */
int qw6_vk_sampling_greedy_host(const float *logits, uint32_t n, uint32_t *token);

/* qw6_vk.h:34-36 -- top_k of n_experts (n_experts <= 256, top_k <= 8),
 * softmax over the selected logits, indices in selection order. */
int qw6_vk_moe_route_host(const float *logits, uint32_t *indices, float *weights, uint32_t n_experts,
                          uint32_t top_k);

/* qw6_vk.h:37-40 -- out[i] = sum_e w[e] * expert_out[e*dim + i]
 * (+ shared_weight * shared_out[i] when shared_out != NULL); top_k <= 8. */
int qw6_vk_moe_gather_host(const float *expert_out, const float *expert_weights, const float *shared_out,
                           float shared_weight, float *out, uint32_t dim, uint32_t top_k);

/* qw6_vk.h:20-23, 30-33, 41-55 -- entry points of the reference header that
 * lie outside the quantized-matvec / MoE path (RMSNorm, attention, DeltaNet,
 * MRoPE, MTP).  They exist so that qw6.c and other consumers link; each
 * returns -1 ("not provided by this library"), which qw6's callers already
 * treat as a backend failure. */
int qw6_vk_rmsnorm_host(const float *x, const float *w, float *y, uint32_t n, float eps);
int qw6_vk_rmsnorm_chunked_host(const float *x, const float *w, float *y, uint32_t n, float eps,
                                uint32_t n_groups);
int qw6_vk_attention_gqa_host(const float *q, const float *k_cache, const float *v_cache, float *out,
                              uint32_t seq_len, uint32_t n_q_heads, uint32_t n_kv_heads, uint32_t head_dim);
int qw6_vk_deltanet_conv1d_host(const float *x, const uint16_t *w, float *out, uint32_t dim,
                                uint32_t kernel_size);
int qw6_vk_deltanet_retrieve_host(const float *state, const float *query, float *out, uint32_t key_heads,
                                  uint32_t key_dim, uint32_t val_heads, uint32_t val_dim);
int qw6_vk_deltanet_update_host(float *state, const float *key, const float *value, const float *query,
                                const float *beta, uint32_t key_heads, uint32_t key_dim, uint32_t val_heads,
                                uint32_t val_dim);
int qw6_vk_mrope_host(float *q, float *k, uint32_t q_dim, uint32_t kv_dim, uint32_t n_heads, uint32_t n_kv_heads,
                      uint32_t position, uint32_t rotary_dim);
int qw6_vk_mtp_draft_host(const float *w, const float *hidden, float *logits, uint32_t vocab_size,
                          uint32_t hidden_size);

/* qw6_vk.h:57-83 -- whole-model pipeline.  The decode-step executor is not
 * part of this library (its attention/DeltaNet layers are out of scope), so
 * qw6_vk_pipe_init returns -1 and qw6.c takes its documented CPU path in
 * non-strict mode (qw6.c:3696-3707).  Declared only after qw6.h, which
 * defines qw6_model_t. */
#ifdef QW6_H
typedef struct qw6_vk_pipe_s qw6_vk_pipe_t;
int qw6_vk_pipe_init(qw6_vk_pipe_t **p, qw6_model_t *m, bool strict);
int qw6_vk_pipe_forward(qw6_vk_pipe_t *p, qw6_model_t *m, uint32_t token, uint32_t pos, float *logits_out);
int qw6_vk_pipe_forward_greedy(qw6_vk_pipe_t *p, qw6_model_t *m, uint32_t token, uint32_t pos,
                               uint32_t *out_token, float *dump_logits_buf);
void qw6_vk_pipe_free(qw6_vk_pipe_t *p);
#endif

#ifdef __cplusplus
}
#endif

#endif /* QW6_VK_H */
