/* ref_shim.c -- flat entry points into qw6's own CPU code.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled together with the unmodified
 * reference sources (qw6.c, qw6_tok.c, where they lie) into
 * oracle/_ref/libqw6ref.so by oracle/Makefile, so that tests and the
 * CPU-baseline leg of bench.py can call qw6's real implementation:
 *   qw6_tensor_dequantize_row (qw6.c:1674), qw6_tensor_matvec (qw6.c:1769),
 *   qw6_cpu_moe_route (qw6.c:2796), qw6_cpu_argmax (qw6.c:2858),
 *   qw6_cpu_rmsnorm (qw6.c:2502), qw6_sample (qw6.c:2921, over qw6's full
 *   QW6_VOCAB_SIZE logits, with libc's rand() seeded first), the
 *   qw6_silu / qw6_sigmoid inlines (qw6.h:292-297), and the routed-expert
 *   loop of qw6_apply_layer_moe (qw6.c:2246-2264) over a range of tokens.
 * The shim only wraps raw block bytes in a qw6_tensor_t and validates
 * arguments first, because the reference asserts (exit(1)) on bad input.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qw6.h"
#ifdef QW6_VULKAN
#include "qw6_vk.h"
#endif

static int block_ok(int quant, uint32_t cols) {
    switch (quant) {
    case QW6_Q_FP32:
    case QW6_Q_FP16:
    case QW6_Q_BF16: return cols > 0;
    case QW6_Q_Q4_K_M:
    case QW6_Q_Q4_K_S:
    case QW6_Q_Q5_K:
    case QW6_Q_Q6_K:
    case QW6_Q_IQ2_XXS:
    case QW6_Q_IQ2_S:
    case QW6_Q_IQ3_S: return cols > 0 && cols % 256 == 0;
    default: return 0;
    }
}

static void wrap(qw6_tensor_t *t, int quant, const void *w, uint32_t rows,
                 uint32_t cols) {
    memset(t, 0, sizeof(*t));
    t->rows = rows;
    t->cols = cols;
    t->quant = (qw6_quant_t)quant;
    t->data = (void *)w;
}

int ref_dequantize_row(int quant, const void *w, uint32_t rows, uint32_t cols,
                       uint32_t row, float *dst) {
    if (!w || !dst || rows == 0 || row >= rows || !block_ok(quant, cols)) return -1;
    qw6_tensor_t t;
    wrap(&t, quant, w, rows, cols);
    return qw6_tensor_dequantize_row(&t, row, dst);
}

int ref_matvec(int quant, const void *w, const float *x, float *y,
               uint32_t rows, uint32_t cols) {
    if (!w || !x || !y || rows == 0 || !block_ok(quant, cols)) return -1;
    qw6_tensor_t t;
    wrap(&t, quant, w, rows, cols);
    return qw6_tensor_matvec(y, &t, x, 0);
}

int ref_moe_route(const float *logits, int n_experts, int top_k, int *idx,
                  float *w) {
    if (!logits || !idx || !w || n_experts <= 0 || n_experts > 256 ||
        top_k <= 0 || top_k > n_experts)
        return -1;
    qw6_cpu_moe_route(idx, w, logits, n_experts, top_k);
    return 0;
}

int ref_argmax(const float *x, int n) {
    if (!x || n <= 0) return -1;
    return qw6_cpu_argmax(x, n);
}

float ref_silu(float v) { return qw6_silu(v); }

float ref_sigmoid(float v) { return qw6_sigmoid(v); }

int ref_rmsnorm(const float *x, const float *w, float *out, int dim) {
    if (!x || !w || !out || dim <= 0) return -1;
    qw6_cpu_rmsnorm(out, x, w, dim);
    return 0;
}

int ref_vocab_size(void) { return QW6_VOCAB_SIZE; }

/* logits: QW6_VOCAB_SIZE floats (qw6_sample reads the session's whole row) */
int ref_sample(const float *logits, float temp, float top_p, int top_k, unsigned seed) {
    if (!logits) return -1;
    qw6_session_t s;
    memset(&s, 0, sizeof(s));
    s.logits = (float *)logits;
    srand(seed);
    return (int)qw6_sample(&s, temp, top_p, top_k);
}

/* the uniform draw qw6_sample makes after srand(seed) (qw6.c:2917-2919) */
float ref_rand_unit(unsigned seed) {
    srand(seed);
    return (float)rand() / ((float)RAND_MAX + 1.0f);
}

/* Tokens [t0, t1) of a routed-MoE layer exactly as qw6_apply_layer_moe's
 * expert loop runs them (qw6.c:2246-2264): per token, qw6_cpu_moe_route of
 * its logits row, then for each selected expert in selection order
 * g = Wg[e].x, u = Wu[e].x, mid = silu(g)*u, t = Wd[e].mid, out += w_e*t.
 * Expert e's matrices are at base + e*stride (bind_expert_pack, qw6.c:542-597);
 * x and out are [ntok][hidden] rows, logits [ntok][n_experts].  No shared
 * expert (the benchmark configurations have none).  The whole loop runs in C,
 * so a caller can time qw6's CPU path without interpreter work per element. */
int ref_moe_tokens(int gq, const void *gate, const void *up, size_t gstride, int dq,
                   const void *down, size_t dstride, const float *logits, const float *x,
                   float *out, uint32_t t0, uint32_t t1, uint32_t hidden, uint32_t inter,
                   int n_experts, int top_k) {
    if (!gate || !up || !down || !logits || !x || !out || t1 < t0 || !block_ok(gq, hidden) ||
        !block_ok(dq, inter) || n_experts <= 0 || n_experts > 256 || top_k <= 0 || top_k > n_experts ||
        top_k > 32)
        return -1;
    float *g = malloc(sizeof(float) * inter), *u = malloc(sizeof(float) * inter);
    float *mid = malloc(sizeof(float) * inter), *tmp = malloc(sizeof(float) * hidden);
    int rc = (g && u && mid && tmp) ? 0 : -1;
    for (uint32_t t = t0; t < t1 && rc == 0; t++) {
        int idx[32];
        float w[32];
        const float *xt = x + (size_t)t * hidden;
        float *ot = out + (size_t)t * hidden;
        memset(ot, 0, sizeof(float) * hidden);
        qw6_cpu_moe_route(idx, w, logits + (size_t)t * n_experts, n_experts, top_k);
        for (int k = 0; k < top_k && rc == 0; k++) {
            const size_t e = (size_t)idx[k];
            qw6_tensor_t tg, tu, td;
            wrap(&tg, gq, (const uint8_t *)gate + e * gstride, inter, hidden);
            wrap(&tu, gq, (const uint8_t *)up + e * gstride, inter, hidden);
            wrap(&td, dq, (const uint8_t *)down + e * dstride, hidden, inter);
            rc = qw6_tensor_matvec(g, &tg, xt, 0);
            if (rc == 0) rc = qw6_tensor_matvec(u, &tu, xt, 0);
            if (rc == 0) {
                for (uint32_t i = 0; i < inter; i++) mid[i] = qw6_silu(g[i]) * u[i];
                rc = qw6_tensor_matvec(tmp, &td, mid, 0);
            }
            if (rc == 0)
                for (uint32_t i = 0; i < hidden; i++) ot[i] += w[k] * tmp[i];
        }
    }
    free(g);
    free(u);
    free(mid);
    free(tmp);
    return rc;
}

/* ---- a qw6_model_t for qw6's own forward pass ----
 * ref_model_set fills one tensor of a calloc'd qw6_model_t from raw GGUF
 * bytes (field ids: the per-layer roles of oracle/qw6_oracle.h's QO_F_*,
 * then 100/101/102 for token_embd/output/output_norm; the expert packs set
 * all QW6_NUM_EXPERTS tensors at data + e * stride, as bind_expert_pack
 * does, qw6.c:542-597).  ref_forward runs qw6_prefill (qw6.c:2867-2882)
 * one token at a time on a fresh session -- qw6's CPU forward pass, or, in
 * the library built with QW6_VULKAN, qw6_forward_token's pipeline branch
 * (qw6.c:2429-2445) after qw6_vk_pipe_init -- and copies out_rows logits
 * after every token. */
static qw6_tensor_t *model_field(qw6_model_t *m, int layer, int field) {
    if (field == 100) return &m->tok_embeddings;
    if (field == 101) return &m->output;
    if (field == 102) return &m->output_norm;
    if (layer < 0 || layer >= QW6_NUM_LAYERS) return NULL;
    switch (field) {
    case 0: return &m->layers[layer].norm;
    case 1: return &m->layers[layer].post_norm;
    case 2: return &m->layers[layer].attn_q;
    case 3: return &m->layers[layer].attn_k;
    case 4: return &m->layers[layer].attn_v;
    case 5: return &m->layers[layer].attn_o;
    case 6: return &m->layers[layer].attn_q_norm;
    case 7: return &m->layers[layer].attn_k_norm;
    case 8: return &m->layers[layer].attn_gate;
    case 9: return &m->layers[layer].conv1d;
    case 10: return &m->layers[layer].dn_out;
    case 11: return &m->layers[layer].dn_norm;
    case 12: return &m->layers[layer].dn_alpha;
    case 13: return &m->layers[layer].dn_beta;
    case 14: return &m->layers[layer].dn_dt;
    case 15: return &m->layers[layer].dn_a;
    case 16: return &m->layers[layer].moe_router;
    case 17: return &m->layers[layer].shared_router;
    case 18: return &m->layers[layer].shared_gate;
    case 19: return &m->layers[layer].shared_up;
    case 20: return &m->layers[layer].shared_down;
    case 21: return m->layers[layer].expert_gate;
    case 22: return m->layers[layer].expert_up;
    case 23: return m->layers[layer].expert_down;
    default: return NULL;
    }
}

void *ref_model_new(void) {
    qw6_model_t *m = calloc(1, sizeof(qw6_model_t));
    if (m) {
        m->weight_fd = -1;
        m->max_context = QW6_DEFAULT_CTX;
    }
    return m;
}

int ref_model_set(void *model, int layer, int field, int quant, uint32_t rows, uint32_t cols, const void *data,
                  size_t stride) {
    qw6_model_t *m = model;
    qw6_tensor_t *t = m ? model_field(m, layer, field) : NULL;
    if (!t || !data || !rows || !block_ok(quant, cols)) return -1;
    const int n = (field >= 21 && field <= 23) ? QW6_NUM_EXPERTS : 1;
    for (int e = 0; e < n; e++) {
        wrap(&t[e], quant, (const uint8_t *)data + (size_t)e * stride, rows, cols);
        t[e].ne[0] = cols;
        t[e].ne[1] = rows;
        t[e].n_dims = rows > 1 ? 2 : 1;
        snprintf(t[e].name, sizeof t[e].name, "f%d.l%d.e%d", field, layer, e);
#ifdef QW6_VULKAN
        t[e].vk_offset = (size_t)-1;
#endif
    }
    return 0;
}

static void model_states_free(qw6_model_t *m) {
    for (int l = 0; l < QW6_NUM_LAYERS; l++) {
        free(m->deltanet_state[l]);
        free(m->k_cache[l]);
        free(m->v_cache[l]);
        m->deltanet_state[l] = m->k_cache[l] = m->v_cache[l] = NULL;
    }
}

void ref_model_free(void *model) {
    if (!model) return;
    model_states_free(model);
    free(model);
}

int ref_forward(void *model, const uint32_t *tokens, uint32_t n, float *logits, uint32_t out_rows, int use_pipe) {
    qw6_model_t *m = model;
    if (!m || !tokens || !n || !logits || out_rows > QW6_VOCAB_SIZE) return -1;
#ifndef QW6_VULKAN
    if (use_pipe) return -1;
#endif
    qw6_session_t s;
    if (qw6_session_init(&s, m, n, use_pipe != 0) != 0) return -1;
    int rc = 0;
#ifdef QW6_VULKAN
    if (use_pipe) rc = qw6_vk_pipe_init((qw6_vk_pipe_t **)&s.vk_pipe, m, true);
#endif
    for (uint32_t i = 0; i < n && rc == 0; i++) {
        rc = qw6_prefill(&s, tokens + i, 1);
        if (rc == 0) memcpy(logits + (size_t)i * out_rows, s.logits, (size_t)out_rows * sizeof(float));
    }
#ifdef QW6_VULKAN
    if (s.vk_pipe) qw6_vk_pipe_free(s.vk_pipe);
    s.vk_pipe = NULL;
#endif
    qw6_session_free(&s);
    model_states_free(m);
    return rc;
}

#ifdef QW6_VULKAN
/* qw6_vk_pipe_forward_greedy over the tokens: the picked id after each and,
 * when logits is given, the logits the call returns with it */
int ref_pipe_greedy(void *model, const uint32_t *tokens, uint32_t n, uint32_t *picked, float *logits,
                    uint32_t out_rows) {
    qw6_model_t *m = model;
    if (!m || !tokens || !n || !picked || out_rows > QW6_VOCAB_SIZE) return -1;
    qw6_vk_pipe_t *p = NULL;
    if (qw6_vk_pipe_init(&p, m, true) != 0) return -1;
    float *buf = logits ? calloc(QW6_VOCAB_SIZE, sizeof(float)) : NULL;
    int rc = (logits && !buf) ? -1 : 0;
    for (uint32_t i = 0; i < n && rc == 0; i++) {
        rc = qw6_vk_pipe_forward_greedy(p, m, tokens[i], i, &picked[i], buf);
        if (rc == 0 && logits) memcpy(logits + (size_t)i * out_rows, buf, (size_t)out_rows * sizeof(float));
    }
    free(buf);
    qw6_vk_pipe_free(p);
    return rc;
}
#endif
