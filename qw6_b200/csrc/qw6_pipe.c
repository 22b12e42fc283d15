/* qw6_pipe.c -- qw6's whole-model pipeline entry points (qw6_vk.h:57-83) on
 * the decode-step executor (qw6_decoder.c).
 *
 * qw6_forward_token calls qw6_vk_pipe_forward / _forward_greedy for every
 * token once qw6_vk_pipe_init has succeeded (qw6.c:2429-2445, 3696-3707).
 * init reads the tensors of the caller's qw6_model_t (layout:
 * qw6_model_abi.h), uploads them once (the counterpart of the reference's
 * upload in qw6_vk_pipe_init, qw6_vk.c:2920-2958) and captures the step
 * graph; forward runs one step and copies the logits into qw6's buffer;
 * greedy returns the argmax and copies the logits only when asked.  The
 * pipeline owns its own context on device $QW6_CUDA_DEVICE (default 0).
 * Declared in include/qw6_vk.h with qw6's types; defined here with plain
 * pointers, which is ABI-identical. */
#define _POSIX_C_SOURCE 200809L

#include <stdbool.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "qw6_cuda.h"
#include "qw6_model_abi.h"

typedef struct {
    qw6cu_ctx *ctx;
    qw6cu_decoder *dec;
} pipe_t;

static void put(qw6cu_model_tensor *v, uint32_t *n, uint32_t field, int layer, const qw6abi_tensor *t,
                size_t stride) {
    if (!t->data) return;
    qw6cu_model_tensor *o = &v[(*n)++];
    o->field = field;
    o->layer = layer;
    o->quant = (uint32_t)t->quant;
    o->rows = t->rows;
    o->cols = t->cols;
    o->data = t->data;
    o->stride = stride;
}

/* bytes between consecutive experts when all of them are evenly spaced
 * (bind_expert_pack, qw6.c:542-597), else 0 */
static size_t expert_stride(const qw6abi_tensor *e) {
    if (!e[0].data || !e[1].data) return 0;
    const ptrdiff_t s = (const char *)e[1].data - (const char *)e[0].data;
    if (s <= 0) return 0;
    for (int i = 1; i < QW6ABI_EXPERTS; i++)
        if ((const char *)e[i].data - (const char *)e[0].data != (ptrdiff_t)i * s || e[i].quant != e[0].quant)
            return 0;
    return (size_t)s;
}

static int fail(const char *what) {
    fprintf(stderr, "qw6_cuda pipe: %s: %s\n", what, qw6cu_last_error());
    return -1;
}

int qw6_vk_pipe_init(void **p, void *model, bool strict) {
    (void)strict; /* init either succeeds or reports -1; qw6 decides what a failure means */
    if (!p || !model) return -1;
    *p = NULL;
    const qw6abi_model *m = model;
    const uint32_t cap = 3 + QW6ABI_LAYERS * 32;
    qw6cu_model_tensor *v = calloc(cap, sizeof *v);
    pipe_t *pp = calloc(1, sizeof *pp);
    if (!v || !pp) {
        free(v);
        free(pp);
        return -1;
    }
    uint32_t n = 0;
    put(v, &n, QW6CU_F_TOK_EMBD, -1, &m->tok_embeddings, 0);
    put(v, &n, QW6CU_F_OUTPUT, -1, &m->output, 0);
    put(v, &n, QW6CU_F_OUTPUT_NORM, -1, &m->output_norm, 0);
    int rc = 0;
    for (int l = 0; l < QW6ABI_LAYERS && !rc; l++) {
        const qw6abi_layer *L = &m->layers[l];
        put(v, &n, QW6CU_F_NORM, l, &L->norm, 0);
        put(v, &n, QW6CU_F_POST_NORM, l, &L->post_norm, 0);
        put(v, &n, QW6CU_F_ATTN_Q, l, &L->attn_q, 0);
        put(v, &n, QW6CU_F_ATTN_K, l, &L->attn_k, 0);
        put(v, &n, QW6CU_F_ATTN_V, l, &L->attn_v, 0);
        put(v, &n, QW6CU_F_ATTN_O, l, &L->attn_o, 0);
        put(v, &n, QW6CU_F_ATTN_Q_NORM, l, &L->attn_q_norm, 0);
        put(v, &n, QW6CU_F_ATTN_K_NORM, l, &L->attn_k_norm, 0);
        put(v, &n, QW6CU_F_ATTN_GATE, l, &L->attn_gate, 0);
        put(v, &n, QW6CU_F_CONV1D, l, &L->conv1d, 0);
        put(v, &n, QW6CU_F_DN_OUT, l, &L->dn_out, 0);
        put(v, &n, QW6CU_F_DN_NORM, l, &L->dn_norm, 0);
        put(v, &n, QW6CU_F_DN_ALPHA, l, &L->dn_alpha, 0);
        put(v, &n, QW6CU_F_DN_BETA, l, &L->dn_beta, 0);
        put(v, &n, QW6CU_F_DN_DT, l, &L->dn_dt, 0);
        put(v, &n, QW6CU_F_DN_A, l, &L->dn_a, 0);
        put(v, &n, QW6CU_F_MOE_ROUTER, l, &L->moe_router, 0);
        put(v, &n, QW6CU_F_SHARED_ROUTER, l, &L->shared_router, 0);
        put(v, &n, QW6CU_F_SHARED_GATE, l, &L->shared_gate, 0);
        put(v, &n, QW6CU_F_SHARED_UP, l, &L->shared_up, 0);
        put(v, &n, QW6CU_F_SHARED_DOWN, l, &L->shared_down, 0);
        const size_t sg = expert_stride(L->expert_gate), su = expert_stride(L->expert_up),
                     sd = expert_stride(L->expert_down);
        if (!sg || !su || !sd) {
            fprintf(stderr, "qw6_cuda pipe: layer %d experts are not one evenly spaced pack\n", l);
            rc = -1;
        }
        put(v, &n, QW6CU_F_EXPERT_GATE, l, &L->expert_gate[0], sg);
        put(v, &n, QW6CU_F_EXPERT_UP, l, &L->expert_up[0], su);
        put(v, &n, QW6CU_F_EXPERT_DOWN, l, &L->expert_down[0], sd);
    }
    const char *dev = getenv("QW6_CUDA_DEVICE");
    if (!rc && qw6cu_create(&pp->ctx, dev ? atoi(dev) : 0) != 0) rc = fail("context");
    const uint32_t max_ctx = m->max_context ? m->max_context : 4096;
    if (!rc && qw6cu_decoder_create(pp->ctx, v, n, QW6ABI_LAYERS, max_ctx, &pp->dec) != 0) rc = fail("init");
    free(v);
    if (rc) {
        if (pp->ctx) qw6cu_destroy(pp->ctx);
        free(pp);
        return -1;
    }
    *p = pp;
    return 0;
}

int qw6_vk_pipe_forward(void *p, void *model, uint32_t token, uint32_t pos, float *logits_out) {
    (void)model;
    pipe_t *pp = p;
    if (!pp || !logits_out) return -1;
    return qw6cu_decoder_forward(pp->dec, token, pos, logits_out, NULL) == 0 ? 0 : fail("forward");
}

int qw6_vk_pipe_forward_greedy(void *p, void *model, uint32_t token, uint32_t pos, uint32_t *out_token,
                               float *dump_logits_buf) {
    (void)model;
    pipe_t *pp = p;
    if (!pp || !out_token) return -1;
    return qw6cu_decoder_forward(pp->dec, token, pos, dump_logits_buf, out_token) == 0 ? 0 : fail("forward");
}

void qw6_vk_pipe_free(void *p) {
    pipe_t *pp = p;
    if (!pp) return;
    qw6cu_decoder_destroy(pp->dec);
    qw6cu_destroy(pp->ctx);
    free(pp);
}
