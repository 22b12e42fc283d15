/* qw6_oracle_fwd.c -- CPU restatement of qw6's per-token forward pass.
 *
 * TEST INFRASTRUCTURE ONLY: the checker of the library's decode-step
 * executor; no product code path may link or call it.
 *
 * Follows qw6_forward_token (qw6.c:2426-2500) and the layer functions it
 * calls, in qw6's floating-point evaluation order:
 *   qw6_apply_linear_attn       qw6.c:2292-2360 (Gated DeltaNet layer)
 *   qw6_gated_delta_net_single  qw6.c:2079-2108
 *   qw6_l2_norm_heads           qw6.c:2055-2063
 *   qw6_apply_full_attn         qw6.c:2368-2424 (gated GQA attention layer)
 *   qw6_cpu_mrope               qw6.c:2711-2745
 *   qw6_cpu_attention_gqa       qw6.c:2750-2793
 *   qw6_apply_layer_moe         qw6.c:2226-2290 (via qo_moe_block)
 *   qw6_softplus / qw6_sigmoid  qw6.h:295-302
 * with qw6's model dimensions (qw6.h:24-55) and any number of layers (qw6
 * runs its 40); layer l is full attention when l % 4 == 3 (qw6_layer_type,
 * qw6.h:320-324).  Pinned bit for bit against qw6's own forward pass
 * (oracle/_ref, tests/test_oracle_fwd.py).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "qw6_oracle.h"

enum {
    HID = QO_FWD_HIDDEN,
    QH = 16,        /* query heads */
    KVH = 2,        /* key/value heads of the full-attention layers */
    HD = 256,       /* their head dimension */
    KH = 16,        /* DeltaNet key heads */
    KD = 128,       /* their dimension */
    VH = 32,        /* DeltaNet value heads */
    VD = 128,       /* their dimension */
    CONV = 4,       /* causal conv1d taps */
    QKV = KH * KD * 2 + VH * VD,
    VDIM = VH * VD,
    NE = 256,
    TOPK = 8,
    INTER = 512,
    SINTER = 512,
    ROT = 64        /* (int)(HD * 0.25f): rotary dimensions */
};
#define ROPE_THETA 10000000.0f
#define RMS_EPS 1e-6f

static float silu(float v) { return v / (1.0f + expf(-v)); }
static float sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }
static float softplus(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return log1pf(expf(v));
}

int qo_fwd_is_full(uint32_t layer) { return layer % 4 == 3; }

size_t qo_fwd_state_floats(uint32_t n_layers, uint32_t max_ctx) {
    size_t n = 0;
    for (uint32_t l = 0; l < n_layers; l++)
        n += qo_fwd_is_full(l) ? (size_t)2 * max_ctx * KVH * HD : (size_t)VH * VD * VD + (size_t)CONV * QKV;
    return n;
}

static float *layer_state(float *state, uint32_t layer, uint32_t max_ctx) {
    size_t off = 0;
    for (uint32_t l = 0; l < layer; l++)
        off += qo_fwd_is_full(l) ? (size_t)2 * max_ctx * KVH * HD : (size_t)VH * VD * VD + (size_t)CONV * QKV;
    return state + off;
}

/* qw6_tensor_matvec with max_rows (qw6.c:1769-1791): rows beyond the
 * tensor's stay as the caller left them */
static int tmatvec(const qo_tensor *t, const float *x, float *y, uint32_t max_rows) {
    if (!t->data || !t->rows || !t->cols) return -1;
    const uint32_t rows = max_rows && max_rows < t->rows ? max_rows : t->rows;
    return qo_matvec(t->quant, t->data, x, y, rows, t->cols);
}

/* row 0 of a vector tensor, which must hold exactly n values */
static int tvector(const qo_tensor *t, float *dst, uint32_t n) {
    if (!t->data || t->cols != n) return -1;
    return qo_dequantize_row(t->quant, t->data, t->cols, 0, dst);
}

static int nonfinite(const float *x, uint32_t n) {
    for (uint32_t i = 0; i < n; i++)
        if (!isfinite(x[i])) return 1;
    return 0;
}

static void l2_norm_heads(float *x, int heads, int dim) {
    for (int h = 0; h < heads; h++) {
        float *row = x + h * dim, ss = 0.0f;
        for (int i = 0; i < dim; i++) ss += row[i] * row[i];
        const float scale = 1.0f / sqrtf(ss + RMS_EPS);
        for (int i = 0; i < dim; i++) row[i] *= scale;
    }
}

/* value head vh reads key/query head vh % KH (qw6.c:2084) */
static void gated_delta_net(float *out, float *state, const float *q16, const float *k16, const float *v,
                            const float *gate, const float *beta) {
    const float scale = 1.0f / sqrtf((float)VD);
    for (int vh = 0; vh < VH; vh++) {
        const int kh = vh % KH;
        const float *q = q16 + kh * KD, *k = k16 + kh * KD, *vv = v + vh * VD;
        float *oo = out + vh * VD, *s = state + (size_t)vh * VD * VD;
        const float decay = expf(gate[vh]), b = beta[vh];
        for (int j = 0; j < VD; j++) {
            float *row = s + j * VD;
            for (int i = 0; i < VD; i++) row[i] *= decay;
            float pred = 0.0f;
            for (int i = 0; i < VD; i++) pred += row[i] * k[i];
            const float delta = (vv[j] - pred) * b;
            for (int i = 0; i < VD; i++) row[i] += delta * k[i];
            float sum = 0.0f;
            for (int i = 0; i < VD; i++) sum += row[i] * q[i];
            oo[j] = sum * scale;
        }
    }
}

static int linear_attn(const qo_tensor *L, float *st, const float *x, float *out) {
    float *qkv = calloc(QKV, sizeof(float)), *conv = calloc(QKV, sizeof(float));
    float *z = calloc(VDIM, sizeof(float)), *gdn = calloc(VDIM, sizeof(float)), *gated = calloc(VDIM, sizeof(float));
    float beta[VH] = {0}, alpha[VH] = {0}, dt[VH] = {0}, a[VH] = {0}, nw[VD] = {0};
    int rc = (qkv && conv && z && gdn && gated) ? 0 : -1;
    if (!rc) rc = tmatvec(&L[QO_F_ATTN_Q], x, qkv, QKV);
    if (!rc) rc = tmatvec(&L[QO_F_ATTN_GATE], x, z, VDIM);
    if (!rc) rc = tmatvec(&L[QO_F_DN_BETA], x, beta, VH);
    if (!rc) rc = tmatvec(&L[QO_F_DN_ALPHA], x, alpha, VH);
    if (!rc) rc = tvector(&L[QO_F_DN_DT], dt, VH);
    if (!rc) rc = tvector(&L[QO_F_DN_A], a, VH);
    if (!rc) rc = tvector(&L[QO_F_DN_NORM], nw, VD);
    const qo_tensor *cw_t = &L[QO_F_CONV1D];
    if (!rc && (!cw_t->data || cw_t->quant != 0 || cw_t->rows != QKV || cw_t->cols != CONV)) rc = -1;
    if (!rc) {
        float *dn = st, *cs = st + (size_t)VH * VD * VD;
        memmove(cs, cs + QKV, (size_t)(CONV - 1) * QKV * sizeof(float));
        memcpy(cs + (size_t)(CONV - 1) * QKV, qkv, QKV * sizeof(float));
        const float *cw = (const float *)cw_t->data;
        for (int c = 0; c < QKV; c++) {
            float sum = 0.0f;
            for (int k = 0; k < CONV; k++) sum += cs[(size_t)k * QKV + c] * cw[(size_t)c * CONV + k];
            conv[c] = silu(sum);
        }
        float *q = conv, *k = conv + KH * KD, *v = conv + 2 * KH * KD;
        l2_norm_heads(q, KH, KD);
        l2_norm_heads(k, KH, KD);
        for (int h = 0; h < VH; h++) {
            beta[h] = sigmoid(beta[h]);
            alpha[h] = softplus(alpha[h] + dt[h]) * a[h];
        }
        gated_delta_net(gdn, dn, q, k, v, alpha, beta);
        for (int h = 0; h < VH; h++) {
            float *dst = gated + h * VD;
            qo_rmsnorm(gdn + h * VD, nw, dst, VD);
            for (int i = 0; i < VD; i++) dst[i] *= silu(z[h * VD + i]);
        }
        rc = tmatvec(&L[QO_F_DN_OUT], gated, out, HID);
    }
    free(qkv); free(conv); free(z); free(gdn); free(gated);
    return rc;
}

static void rope(float *x, int heads, int dim, uint32_t pos) {
    const int rot = ROT < dim ? ROT : dim;
    for (int h = 0; h < heads; h++) {
        float *xh = x + h * dim;
        for (int i = 0; i + 1 < rot; i += 2) {
            const float theta = (float)pos / powf(ROPE_THETA, (float)i / rot);
            const float c = cosf(theta), s = sinf(theta), a = xh[i], b = xh[i + 1];
            xh[i] = a * c - b * s;
            xh[i + 1] = a * s + b * c;
        }
    }
}

static int attention_gqa(float *out, const float *q, const float *kc, const float *vc, int seq) {
    const int group = QH / KVH;
    float *scores = malloc((size_t)seq * sizeof(float));
    if (!scores) return -1;
    for (int h = 0; h < QH; h++) {
        const int kv = h / group;
        const float *qh = q + (size_t)h * HD;
        float mx = -INFINITY;
        for (int t = 0; t < seq; t++) {
            const float *kh = kc + ((size_t)t * KVH + kv) * HD;
            float dot = 0.0f;
            for (int d = 0; d < HD; d++) dot += qh[d] * kh[d];
            scores[t] = dot / sqrtf((float)HD);
            if (scores[t] > mx) mx = scores[t];
        }
        float sum = 0.0f;
        for (int t = 0; t < seq; t++) {
            scores[t] = expf(scores[t] - mx);
            sum += scores[t];
        }
        for (int d = 0; d < HD; d++) out[(size_t)h * HD + d] = 0.0f;
        for (int t = 0; t < seq; t++) {
            const float w = scores[t] / sum;
            const float *vh = vc + ((size_t)t * KVH + kv) * HD;
            for (int d = 0; d < HD; d++) out[(size_t)h * HD + d] += w * vh[d];
        }
    }
    free(scores);
    return 0;
}

static int full_attn(const qo_tensor *L, float *st, uint32_t max_ctx, const float *x, uint32_t pos, float *out) {
    if (pos >= max_ctx) return -1;
    float *qfull = calloc(QH * HD * 2, sizeof(float)), *q = calloc(QH * HD, sizeof(float));
    float *gate = calloc(QH * HD, sizeof(float)), *attn = calloc(QH * HD, sizeof(float));
    float k[KVH * HD] = {0}, v[KVH * HD] = {0}, qw[HD] = {0}, kw[HD] = {0};
    int rc = (qfull && q && gate && attn) ? 0 : -1;
    if (!rc) rc = tmatvec(&L[QO_F_ATTN_Q], x, qfull, QH * HD * 2);
    if (!rc) rc = tmatvec(&L[QO_F_ATTN_K], x, k, KVH * HD);
    if (!rc) rc = tmatvec(&L[QO_F_ATTN_V], x, v, KVH * HD);
    if (!rc) rc = tvector(&L[QO_F_ATTN_Q_NORM], qw, HD);
    if (!rc) rc = tvector(&L[QO_F_ATTN_K_NORM], kw, HD);
    if (!rc) {
        for (int h = 0; h < QH; h++) {
            memcpy(q + h * HD, qfull + h * HD * 2, HD * sizeof(float));
            memcpy(gate + h * HD, qfull + h * HD * 2 + HD, HD * sizeof(float));
        }
        for (int h = 0; h < QH; h++) qo_rmsnorm(q + h * HD, qw, q + h * HD, HD);
        for (int h = 0; h < KVH; h++) qo_rmsnorm(k + h * HD, kw, k + h * HD, HD);
        rope(q, QH, HD, pos);
        rope(k, KVH, HD, pos);
        float *kc = st, *vc = st + (size_t)max_ctx * KVH * HD;
        memcpy(kc + (size_t)pos * KVH * HD, k, sizeof k);
        memcpy(vc + (size_t)pos * KVH * HD, v, sizeof v);
        rc = attention_gqa(attn, q, kc, vc, (int)pos + 1);
    }
    if (!rc) {
        for (int i = 0; i < QH * HD; i++) attn[i] *= sigmoid(gate[i]);
        rc = tmatvec(&L[QO_F_ATTN_O], attn, out, HID);
    }
    free(qfull); free(q); free(gate); free(attn);
    return rc;
}

static int moe(const qo_tensor *L, const float *x, float *out) {
    const qo_tensor *r = &L[QO_F_MOE_ROUTER], *g = &L[QO_F_EXPERT_GATE], *u = &L[QO_F_EXPERT_UP],
                    *d = &L[QO_F_EXPERT_DOWN], *sg = &L[QO_F_SHARED_GATE], *su = &L[QO_F_SHARED_UP],
                    *sd = &L[QO_F_SHARED_DOWN], *sr = &L[QO_F_SHARED_ROUTER];
    if (!r->data || !g->data || !u->data || !d->data) return -1;
    const qo_matrix router = {r->quant, r->data}, mg = {sg->quant, sg->data}, mu = {su->quant, su->data},
                    md = {sd->quant, sd->data}, msr = {sr->quant, sr->data};
    const qo_expert_pack pg = {g->quant, g->data, g->stride}, pu = {u->quant, u->data, u->stride},
                         pd = {d->quant, d->data, d->stride};
    const int shared = sg->data && su->data && sd->data;
    float nw[HID];
    int rc = tvector(&L[QO_F_POST_NORM], nw, HID);
    if (!rc)
        rc = qo_moe_block(x, nw, &router, &pg, &pu, &pd, shared ? &mg : NULL, shared ? &mu : NULL,
                          shared ? &md : NULL, shared && sr->data ? &msr : NULL, out, 1, HID, INTER, SINTER, NE, TOPK);
    return rc;
}

int qo_forward(const qo_model *m, float *state, uint32_t max_ctx, uint32_t token, uint32_t pos, float *logits) {
    if (!m || !m->layers || !state || !logits || !m->tok_embd.data || token >= m->tok_embd.rows ||
        m->tok_embd.cols != HID)
        return -1;
    float hidden[HID], normed[HID], nw[HID], attn[HID], next[HID];
    int rc = qo_dequantize_row(m->tok_embd.quant, m->tok_embd.data, HID, token, hidden);
    if (!rc && nonfinite(hidden, HID)) rc = -1;
    for (uint32_t l = 0; l < m->n_layers && !rc; l++) {
        const qo_tensor *L = m->layers + (size_t)l * QO_NF;
        float *st = layer_state(state, l, max_ctx);
        memset(attn, 0, sizeof attn);
        rc = tvector(&L[QO_F_NORM], nw, HID);
        if (!rc) {
            qo_rmsnorm(hidden, nw, normed, HID);
            rc = qo_fwd_is_full(l) ? full_attn(L, st, max_ctx, normed, pos, attn) : linear_attn(L, st, normed, attn);
        }
        if (!rc) {
            for (int i = 0; i < HID; i++) hidden[i] += attn[i];
            if (nonfinite(hidden, HID)) rc = -1;
        }
        if (!rc) rc = moe(L, hidden, next);
        if (!rc) {
            memcpy(hidden, next, sizeof hidden);
            if (nonfinite(hidden, HID)) rc = -1;
        }
    }
    if (!rc) rc = tvector(&m->output_norm, nw, HID);
    if (!rc) {
        qo_rmsnorm(hidden, nw, normed, HID);
        rc = tmatvec(&m->output, normed, logits, 0);
    }
    if (!rc && nonfinite(logits, m->output.rows)) rc = -1;
    return rc;
}
