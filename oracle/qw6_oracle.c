/* qw6_oracle.c -- CPU restatement of qw6's quantized-matvec + MoE path.
 *
 * TEST INFRASTRUCTURE ONLY (see qw6_oracle.h).  Each decoder below restates
 * the matching qw6 function with the same float evaluation order; all
 * arithmetic is IEEE binary32, left to right, no FMA (built with
 * -ffp-contract=off).
 */
#include "qw6_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../qw6_b200/csrc/qw6_formats.h"
#include "../qw6_b200/csrc/qw6_iq_grids.h"

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
           ((uint32_t)p[3] << 24);
}
static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* qw6.c:1448-1471 */
float qo_fp16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31u) return bits_f32(sign | 0x7f800000u | (m << 13));
    if (e == 0u) {
        if (m == 0u) return bits_f32(sign);
        /* subnormal: shift the mantissa up until the implicit bit appears */
        int32_t ex = 1;
        while (!(m & 1024u)) { m <<= 1; ex--; }
        return bits_f32(sign | ((uint32_t)(ex + 112) << 23) | ((m & 1023u) << 13));
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* qw6.c:1473-1478 */
static float bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* qw6_get_scale_min_k4, qw6.c:1480-1490: 8 (scale, min) 6-bit pairs packed
 * into 12 bytes; pairs 0..3 sit in the low 6 bits of bytes 0..7, pairs 4..7
 * take their low nibbles from bytes 8..11 and their top 2 bits from the top
 * of bytes 0..7. */
static void k4_scale_min(const uint8_t *s, int j, uint32_t *sc, uint32_t *mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
        *mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

/* qw6_dequantize_row_q4_k, qw6.c:1492-1516 (one 144-byte block). */
static void blk_q4_k(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b));
    const float dm = qo_fp16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qs = b + 16;
    for (int c = 0; c < 4; c++) {
        uint32_t s0, m0, s1, m1;
        k4_scale_min(sc, 2 * c, &s0, &m0);
        k4_scale_min(sc, 2 * c + 1, &s1, &m1);
        const float dl = d * (float)s0, ml = dm * (float)m0;
        const float dh = d * (float)s1, mh = dm * (float)m1;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++) o[64 * c + l] = dl * (float)(q[l] & 15) - ml;
        for (int l = 0; l < 32; l++) o[64 * c + 32 + l] = dh * (float)(q[l] >> 4) - mh;
    }
}

/* qw6_dequantize_row_q5_k, qw6.c:1518-1548 (one 176-byte block). */
static void blk_q5_k(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b));
    const float dm = qo_fp16_to_f32(rd16(b + 2));
    const uint8_t *sc = b + 4, *qh = b + 16, *qs = b + 48;
    for (int c = 0; c < 4; c++) {
        uint32_t s0, m0, s1, m1;
        k4_scale_min(sc, 2 * c, &s0, &m0);
        k4_scale_min(sc, 2 * c + 1, &s1, &m1);
        const float dl = d * (float)s0, ml = dm * (float)m0;
        const float dh = d * (float)s1, mh = dm * (float)m1;
        const uint8_t lo_bit = (uint8_t)(1u << (2 * c)), hi_bit = (uint8_t)(2u << (2 * c));
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++)
            o[64 * c + l] = dl * (float)((q[l] & 15) + ((qh[l] & lo_bit) ? 16 : 0)) - ml;
        for (int l = 0; l < 32; l++)
            o[64 * c + 32 + l] = dh * (float)((q[l] >> 4) + ((qh[l] & hi_bit) ? 16 : 0)) - mh;
    }
}

/* qw6_dequantize_row_q6_k, qw6.c:1550-1578 (one 210-byte block).  qw6 reads
 * scale sc[n/16 + 2*k] for the k-th 32-run of each 128-half, i.e. only the
 * even-indexed scales; that is reproduced here exactly. */
static void blk_q6_k(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b + 208));
    const int8_t *sc = (const int8_t *)(b + 192);
    for (int h = 0; h < 2; h++) {
        const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
        const int8_t *s = sc + 8 * h;
        float *oh = o + 128 * h;
        for (int l = 0; l < 32; l++) {
            const int q0 = (int)((ql[l] & 15) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q1 = (int)((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q2 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q3 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            oh[l] = d * (float)s[0] * (float)q0;
            oh[l + 32] = d * (float)s[2] * (float)q1;
            oh[l + 64] = d * (float)s[4] * (float)q2;
            oh[l + 96] = d * (float)s[6] * (float)q3;
        }
    }
}

static float sgn(uint32_t signs, int j) { return (signs >> j) & 1u ? -1.0f : 1.0f; }

/* qw6_dequantize_row_iq2_xxs, qw6.c:1580-1602 (one 66-byte block).  Each
 * 32-weight group is 8 bytes: 4 grid indices, then a word holding four 7-bit
 * sign indices and a 4-bit scale in its top nibble. */
static void blk_iq2_xxs(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b));
    for (int g = 0; g < 8; g++) {
        const uint8_t *grp = b + 2 + 8 * g;
        const uint32_t aux = rd32(grp + 4);
        const float db = d * (0.5f + (float)(aux >> 28)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint8_t *gr = QW6_IQ2XXS_GRID_BYTES + 8u * grp[l];
            const uint32_t s = qw6_ksigns((aux >> (7 * l)) & 127u);
            for (int j = 0; j < 8; j++) o[32 * g + 8 * l + j] = db * (float)gr[j] * sgn(s, j);
        }
    }
}

/* qw6_dequantize_row_iq2_s, qw6.c:1604-1630 (one 82-byte block). */
static void blk_iq2_s(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b));
    const uint8_t *qs = b + 2, *sg = b + 34, *qh = b + 66, *sc = b + 74;
    for (int g = 0; g < 8; g++) {
        const float d0 = d * (0.5f + (float)(sc[g] & 15)) * 0.25f;
        const float d1 = d * (0.5f + (float)(sc[g] >> 4)) * 0.25f;
        for (int l = 0; l < 4; l++) {
            const uint32_t gi = qs[4 * g + l] | (((uint32_t)qh[g] << (8 - 2 * l)) & 0x300u);
            const uint8_t *gr = QW6_IQ2S_GRID_BYTES + 8u * gi;
            const float dl = l < 2 ? d0 : d1;
            const uint32_t s = sg[4 * g + l];
            for (int j = 0; j < 8; j++) o[32 * g + 8 * l + j] = dl * (float)gr[j] * sgn(s, j);
        }
    }
}

/* qw6_dequantize_row_iq3_s, qw6.c:1632-1672 (one 110-byte block).  Pairs of
 * 32-weight groups share a scale byte (low nibble, high nibble); each 8
 * weights come from two 4-byte grid entries whose 9th index bit is taken
 * from the group's qh byte. */
static void blk_iq3_s(const uint8_t *b, float *o) {
    const float d = qo_fp16_to_f32(rd16(b));
    const uint8_t *qs = b + 2, *qh = b + 66, *sg = b + 74, *sc = b + 106;
    for (int g = 0; g < 8; g++) {
        const uint32_t nib = (g & 1) ? (sc[g >> 1] >> 4) : (sc[g >> 1] & 15u);
        const float db = d * (float)(int)(1 + 2 * nib);
        const uint8_t *q = qs + 8 * g, *s = sg + 4 * g;
        const uint32_t h = qh[g];
        for (int l = 0; l < 4; l++) {
            const uint32_t i1 = q[2 * l] | ((h << (8 - 2 * l)) & 256u);
            const uint32_t i2 = q[2 * l + 1] | ((h << (7 - 2 * l)) & 256u);
            const uint8_t *g1 = QW6_IQ3S_GRID_BYTES + 4u * i1;
            const uint8_t *g2 = QW6_IQ3S_GRID_BYTES + 4u * i2;
            for (int j = 0; j < 4; j++) {
                o[32 * g + 8 * l + j] = db * (float)g1[j] * sgn(s[l], j);
                o[32 * g + 8 * l + j + 4] = db * (float)g2[j] * sgn(s[l], j + 4);
            }
        }
    }
}

typedef void (*blk_fn)(const uint8_t *, float *);

static blk_fn block_decoder(uint32_t quant) {
    switch (quant) {
    case QW6F_Q4_K_M:
    case QW6F_Q4_K_S: return blk_q4_k;
    case QW6F_Q5_K: return blk_q5_k;
    case QW6F_Q6_K: return blk_q6_k;
    case QW6F_IQ2_XXS: return blk_iq2_xxs;
    case QW6F_IQ2_S: return blk_iq2_s;
    case QW6F_IQ3_S: return blk_iq3_s;
    default: return NULL;
    }
}

/* qw6.c:1674-1724 */
int qo_dequantize_row(uint32_t quant, const void *w, uint32_t cols,
                      uint32_t row, float *dst) {
    if (!w || !dst || cols == 0) return -1;
    const uint8_t *base = (const uint8_t *)w;
    if (quant == QW6F_FP32) {
        memcpy(dst, base + (size_t)row * cols * 4u, (size_t)cols * 4u);
        return 0;
    }
    if (quant == QW6F_FP16 || quant == QW6F_BF16) {
        const uint8_t *p = base + (size_t)row * cols * 2u;
        for (uint32_t i = 0; i < cols; i++)
            dst[i] = quant == QW6F_FP16 ? qo_fp16_to_f32(rd16(p + 2 * i)) : bf16_to_f32(rd16(p + 2 * i));
        return 0;
    }
    blk_fn f = block_decoder(quant);
    if (!f || cols % QW6_QK) return -1;
    const uint32_t bb = qw6_block_bytes(quant), nb = cols / QW6_QK;
    const uint8_t *r = base + (size_t)row * nb * bb;
    for (uint32_t i = 0; i < nb; i++) f(r + (size_t)i * bb, dst + (size_t)i * QW6_QK);
    return 0;
}

/* qw6.c:1769-1791 */
int qo_matvec(uint32_t quant, const void *w, const float *x, float *y,
              uint32_t rows, uint32_t cols) {
    if (!rows || !cols || !x || !y) return -1;
    float *buf = (float *)malloc((size_t)cols * sizeof(float));
    if (!buf) return -1;
    for (uint32_t r = 0; r < rows; r++) {
        if (qo_dequantize_row(quant, w, cols, r, buf)) { free(buf); return -1; }
        float acc = 0.0f;
        for (uint32_t c = 0; c < cols; c++) acc += buf[c] * x[c];
        y[r] = acc;
    }
    free(buf);
    return 0;
}

int qo_matvec_f64(uint32_t quant, const void *w, const float *x, double *y,
                  uint32_t rows, uint32_t cols) {
    if (!rows || !cols || !x || !y) return -1;
    float *buf = (float *)malloc((size_t)cols * sizeof(float));
    if (!buf) return -1;
    for (uint32_t r = 0; r < rows; r++) {
        if (qo_dequantize_row(quant, w, cols, r, buf)) { free(buf); return -1; }
        double acc = 0.0;
        for (uint32_t c = 0; c < cols; c++) acc += (double)buf[c] * (double)x[c];
        y[r] = acc;
    }
    free(buf);
    return 0;
}

int qo_matvec_batch(uint32_t quant, const void *w, const float *x, float *y,
                    uint32_t rows, uint32_t cols, uint32_t ntok) {
    for (uint32_t t = 0; t < ntok; t++)
        if (qo_matvec(quant, w, x + (size_t)t * cols, y + (size_t)t * rows, rows, cols)) return -1;
    return 0;
}

/* qw6.c:2796-2827 */
int qo_moe_route(const float *logits, uint32_t n_experts, uint32_t top_k,
                 int32_t *idx, float *w) {
    if (!n_experts || n_experts > 256 || !top_k || top_k > n_experts) return -1;
    float v[256];
    memcpy(v, logits, n_experts * sizeof(float));
    for (uint32_t k = 0; k < top_k; k++) {
        uint32_t best = 0;
        for (uint32_t i = 1; i < n_experts; i++)
            if (v[i] > v[best]) best = i;
        idx[k] = (int32_t)best;
        w[k] = v[best];
        v[best] = -INFINITY;
    }
    float mx = w[0];
    for (uint32_t k = 1; k < top_k; k++) if (w[k] > mx) mx = w[k];
    float sum = 0.0f;
    for (uint32_t k = 0; k < top_k; k++) { w[k] = expf(w[k] - mx); sum += w[k]; }
    for (uint32_t k = 0; k < top_k; k++) w[k] /= sum;
    return 0;
}

/* qw6.c:2858-2863 */
int32_t qo_argmax(const float *x, uint32_t n) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < n; i++) if (x[i] > x[best]) best = i;
    return (int32_t)best;
}

void qo_moe_gather(const float *expert_out, const float *w,
                   const float *shared_out, float shared_weight, float *out,
                   uint32_t dim, uint32_t top_k) {
    for (uint32_t i = 0; i < dim; i++) {
        float acc = 0.0f;
        for (uint32_t e = 0; e < top_k; e++) acc += w[e] * expert_out[(size_t)e * dim + i];
        if (shared_out) acc += shared_weight * shared_out[i];
        out[i] = acc;
    }
}

/* qw6_silu, qw6.h:292-294 */
static float silu(float v) { return v / (1.0f + expf(-v)); }

void qo_silu_mul(const float *gate, const float *up, float *out, uint32_t n) {
    for (uint32_t i = 0; i < n; i++) out[i] = silu(gate[i]) * up[i];
}

static const uint8_t *expert_ptr(const qo_expert_pack *p, int32_t e) {
    return (const uint8_t *)p->base + (size_t)e * p->stride;
}

/* qw6.c:2246-2264 */
int qo_moe_layer(const qo_expert_pack *gate, const qo_expert_pack *up,
                 const qo_expert_pack *down, const float *logits,
                 const float *x, float *out, uint32_t ntok,
                 uint32_t hidden, uint32_t inter, uint32_t n_experts,
                 uint32_t top_k, int32_t *idx_out, float *w_out) {
    if (top_k > 256) return -1;
    float *g = malloc(inter * sizeof(float)), *u = malloc(inter * sizeof(float));
    float *mid = malloc(inter * sizeof(float)), *tmp = malloc(hidden * sizeof(float));
    int rc = (g && u && mid && tmp) ? 0 : -1;
    int32_t idx[256];
    float w[256];
    for (uint32_t t = 0; t < ntok && rc == 0; t++) {
        const float *xt = x + (size_t)t * hidden;
        float *ot = out + (size_t)t * hidden;
        memset(ot, 0, hidden * sizeof(float));
        rc = qo_moe_route(logits + (size_t)t * n_experts, n_experts, top_k, idx, w);
        for (uint32_t k = 0; k < top_k && rc == 0; k++) {
            rc = qo_matvec(gate->quant, expert_ptr(gate, idx[k]), xt, g, inter, hidden);
            if (!rc) rc = qo_matvec(up->quant, expert_ptr(up, idx[k]), xt, u, inter, hidden);
            if (!rc) {
                for (uint32_t i = 0; i < inter; i++) mid[i] = silu(g[i]) * u[i];
                rc = qo_matvec(down->quant, expert_ptr(down, idx[k]), mid, tmp, hidden, inter);
            }
            if (!rc) for (uint32_t i = 0; i < hidden; i++) ot[i] += w[k] * tmp[i];
        }
        if (rc == 0 && idx_out) memcpy(idx_out + (size_t)t * top_k, idx, top_k * sizeof(int32_t));
        if (rc == 0 && w_out) memcpy(w_out + (size_t)t * top_k, w, top_k * sizeof(float));
    }
    free(g); free(u); free(mid); free(tmp);
    return rc;
}

int qo_moe_layer_f64(const qo_expert_pack *gate, const qo_expert_pack *up,
                     const qo_expert_pack *down, const float *logits,
                     const float *x, double *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t n_experts,
                     uint32_t top_k) {
    if (top_k > 256) return -1;
    double *g = malloc(inter * sizeof(double)), *u = malloc(inter * sizeof(double));
    double *tmp = malloc(hidden * sizeof(double));
    float *row = malloc((hidden > inter ? hidden : inter) * sizeof(float));
    double *mid = malloc(inter * sizeof(double));
    int rc = (g && u && tmp && row && mid) ? 0 : -1;
    int32_t idx[256];
    float w[256];
    for (uint32_t t = 0; t < ntok && rc == 0; t++) {
        const float *xt = x + (size_t)t * hidden;
        double *ot = out + (size_t)t * hidden;
        for (uint32_t i = 0; i < hidden; i++) ot[i] = 0.0;
        rc = qo_moe_route(logits + (size_t)t * n_experts, n_experts, top_k, idx, w);
        for (uint32_t k = 0; k < top_k && rc == 0; k++) {
            const uint8_t *pg = expert_ptr(gate, idx[k]), *pu = expert_ptr(up, idx[k]);
            for (uint32_t r = 0; r < inter && rc == 0; r++) {
                double ag = 0.0, au = 0.0;
                rc = qo_dequantize_row(gate->quant, pg, hidden, r, row);
                for (uint32_t c = 0; c < hidden && !rc; c++) ag += (double)row[c] * xt[c];
                if (!rc) rc = qo_dequantize_row(up->quant, pu, hidden, r, row);
                for (uint32_t c = 0; c < hidden && !rc; c++) au += (double)row[c] * xt[c];
                g[r] = ag;
                u[r] = au;
            }
            for (uint32_t i = 0; i < inter; i++) mid[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
            const uint8_t *pd = expert_ptr(down, idx[k]);
            for (uint32_t r = 0; r < hidden && rc == 0; r++) {
                double a = 0.0;
                rc = qo_dequantize_row(down->quant, pd, inter, r, row);
                for (uint32_t c = 0; c < inter && !rc; c++) a += (double)row[c] * mid[c];
                tmp[r] = a;
            }
            for (uint32_t i = 0; i < hidden && !rc; i++) ot[i] += (double)w[k] * tmp[i];
        }
    }
    free(g); free(u); free(tmp); free(row); free(mid);
    return rc;
}

/* qw6.c:2502-2512 */
void qo_rmsnorm(const float *x, const float *weight, float *out, uint32_t dim) {
    float ss = 0.0f;
    for (uint32_t i = 0; i < dim; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / (float)dim + 1e-6f);
    for (uint32_t i = 0; i < dim; i++) out[i] = x[i] * ss * weight[i];
}

/* qw6_sigmoid, qw6.h:295-297 */
static float sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }

/* qw6.c:2474-2484 around qw6.c:2226-2290 */
int qo_moe_block(const float *x, const float *norm_w, const qo_matrix *router,
                 const qo_expert_pack *gate, const qo_expert_pack *up,
                 const qo_expert_pack *down, const qo_matrix *sgate,
                 const qo_matrix *sup, const qo_matrix *sdown,
                 const qo_matrix *srouter, float *out, uint32_t ntok,
                 uint32_t hidden, uint32_t inter, uint32_t shared_inter,
                 uint32_t n_experts, uint32_t top_k) {
    if (!x || !norm_w || !router || !gate || !up || !down || !out || !hidden || !n_experts ||
        n_experts > 256 || !top_k || top_k > n_experts)
        return -1;
    const int shared = sgate && sup && sdown;
    if ((sgate || sup || sdown) && !shared) return -1;
    if (shared && !shared_inter) return -1;
    const uint32_t si = shared ? shared_inter : 1;
    float *normed = malloc(hidden * sizeof(float)), *ffn = malloc(hidden * sizeof(float));
    float *tmp = malloc(hidden * sizeof(float)), *logits = malloc(n_experts * sizeof(float));
    float *sg = malloc(si * sizeof(float)), *su = malloc(si * sizeof(float)), *smid = malloc(si * sizeof(float));
    int rc = (normed && ffn && tmp && logits && sg && su && smid) ? 0 : -1;
    for (uint32_t t = 0; t < ntok && rc == 0; t++) {
        const float *xt = x + (size_t)t * hidden;
        qo_rmsnorm(xt, norm_w, normed, hidden);
        rc = qo_matvec(router->quant, router->w, normed, logits, n_experts, hidden);
        if (!rc) rc = qo_moe_layer(gate, up, down, logits, normed, ffn, 1, hidden, inter, n_experts, top_k, NULL, NULL);
        if (!rc && shared) {
            float s = 1.0f;
            if (srouter) {
                rc = qo_matvec(srouter->quant, srouter->w, normed, &s, 1, hidden);
                s = sigmoid(s);
            }
            if (!rc) rc = qo_matvec(sgate->quant, sgate->w, normed, sg, shared_inter, hidden);
            if (!rc) rc = qo_matvec(sup->quant, sup->w, normed, su, shared_inter, hidden);
            if (!rc) {
                for (uint32_t i = 0; i < shared_inter; i++) smid[i] = silu(sg[i]) * su[i];
                rc = qo_matvec(sdown->quant, sdown->w, smid, tmp, hidden, shared_inter);
            }
            if (!rc)
                for (uint32_t i = 0; i < hidden; i++) ffn[i] += s * tmp[i];
        }
        if (!rc)
            for (uint32_t i = 0; i < hidden; i++) out[(size_t)t * hidden + i] = xt[i] + ffn[i];
    }
    free(normed); free(ffn); free(tmp); free(logits); free(sg); free(su); free(smid);
    return rc;
}

/* y[r] = sum_c W[r][c] * x[c] in double over the dequantized rows of W
 * ([rows x cols]); row is scratch of cols floats */
static int matvec_d(uint32_t quant, const void *w, const double *x, double *y, uint32_t rows, uint32_t cols,
                    float *row) {
    for (uint32_t r = 0; r < rows; r++) {
        if (qo_dequantize_row(quant, w, cols, r, row)) return -1;
        double a = 0.0;
        for (uint32_t c = 0; c < cols; c++) a += (double)row[c] * x[c];
        y[r] = a;
    }
    return 0;
}

int qo_moe_block_f64(const float *x, const float *norm_w, const qo_matrix *router,
                     const qo_expert_pack *gate, const qo_expert_pack *up,
                     const qo_expert_pack *down, const qo_matrix *sgate,
                     const qo_matrix *sup, const qo_matrix *sdown,
                     const qo_matrix *srouter, double *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t shared_inter,
                     uint32_t n_experts, uint32_t top_k) {
    if (!x || !norm_w || !router || !gate || !up || !down || !out || !hidden || !n_experts ||
        n_experts > 256 || !top_k || top_k > n_experts)
        return -1;
    const int shared = sgate && sup && sdown;
    if ((sgate || sup || sdown) && !shared) return -1;
    if (shared && !shared_inter) return -1;
    const uint32_t mi = inter > shared_inter ? inter : shared_inter, wide = hidden > mi ? hidden : mi;
    float *n32 = malloc(hidden * sizeof(float)), *logits = malloc(n_experts * sizeof(float));
    float *row = malloc(wide * sizeof(float));
    double *nd = malloc(hidden * sizeof(double)), *ffn = malloc(hidden * sizeof(double));
    double *tmp = malloc(hidden * sizeof(double)), *g = malloc(mi * sizeof(double));
    double *u = malloc(mi * sizeof(double)), *mid = malloc(mi * sizeof(double));
    int rc = (n32 && logits && row && nd && ffn && tmp && g && u && mid) ? 0 : -1;
    int32_t idx[256];
    float w[256];
    for (uint32_t t = 0; t < ntok && rc == 0; t++) {
        const float *xt = x + (size_t)t * hidden;
        /* routing exactly as the fp32 block */
        qo_rmsnorm(xt, norm_w, n32, hidden);
        rc = qo_matvec(router->quant, router->w, n32, logits, n_experts, hidden);
        if (!rc) rc = qo_moe_route(logits, n_experts, top_k, idx, w);
        /* the arithmetic in double */
        double ss = 0.0;
        for (uint32_t i = 0; i < hidden; i++) ss += (double)xt[i] * xt[i];
        const double scale = 1.0 / sqrt(ss / hidden + 1e-6);
        for (uint32_t i = 0; i < hidden; i++) nd[i] = (double)xt[i] * scale * norm_w[i];
        for (uint32_t i = 0; i < hidden; i++) ffn[i] = 0.0;
        for (uint32_t k = 0; k < top_k && rc == 0; k++) {
            rc = matvec_d(gate->quant, expert_ptr(gate, idx[k]), nd, g, inter, hidden, row);
            if (!rc) rc = matvec_d(up->quant, expert_ptr(up, idx[k]), nd, u, inter, hidden, row);
            for (uint32_t i = 0; i < inter && !rc; i++) mid[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
            if (!rc) rc = matvec_d(down->quant, expert_ptr(down, idx[k]), mid, tmp, hidden, inter, row);
            for (uint32_t i = 0; i < hidden && !rc; i++) ffn[i] += (double)w[k] * tmp[i];
        }
        if (!rc && shared) {
            double s = 1.0;
            if (srouter) {
                rc = matvec_d(srouter->quant, srouter->w, nd, &s, 1, hidden, row);
                s = 1.0 / (1.0 + exp(-s));
            }
            if (!rc) rc = matvec_d(sgate->quant, sgate->w, nd, g, shared_inter, hidden, row);
            if (!rc) rc = matvec_d(sup->quant, sup->w, nd, u, shared_inter, hidden, row);
            for (uint32_t i = 0; i < shared_inter && !rc; i++) mid[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
            if (!rc) rc = matvec_d(sdown->quant, sdown->w, mid, tmp, hidden, shared_inter, row);
            for (uint32_t i = 0; i < hidden && !rc; i++) ffn[i] += s * tmp[i];
        }
        for (uint32_t i = 0; i < hidden && !rc; i++) out[(size_t)t * hidden + i] = (double)xt[i] + ffn[i];
    }
    free(n32); free(logits); free(row); free(nd); free(ffn); free(tmp); free(g); free(u); free(mid);
    return rc;
}

typedef struct {
    int idx;
    float score;
} qo_sample_item;

/* qw6.c:2909-2915: descending score, then ascending index */
static int sample_item_cmp(const void *a, const void *b) {
    const qo_sample_item *ia = (const qo_sample_item *)a, *ib = (const qo_sample_item *)b;
    if (ia->score < ib->score) return 1;
    if (ia->score > ib->score) return -1;
    return ia->idx - ib->idx;
}

/* qw6.c:2921-2982 */
int32_t qo_sample(const float *logits, uint32_t n, float temp, float top_p, int top_k, float u) {
    if (!logits || !n) return -1;
    if (temp <= 0.0f) return qo_argmax(logits, n);
    if (top_k < 0) top_k = 0;
    if (top_p <= 0.0f || top_p > 1.0f) top_p = 1.0f;
    qo_sample_item *items = malloc((size_t)n * sizeof(*items));
    if (!items) return -1;
    float max_score = -INFINITY;
    for (uint32_t i = 0; i < n; i++) {
        const float score = logits[i] / temp;
        items[i].idx = (int)i;
        items[i].score = score;
        if (score > max_score) max_score = score;
    }
    qsort(items, n, sizeof(*items), sample_item_cmp);
    int limit = (int)n;
    if (top_k > 0 && top_k < limit) limit = top_k;
    double sum = 0.0;
    for (int i = 0; i < limit; i++) sum += exp((double)items[i].score - (double)max_score);
    if (sum <= 0.0) {
        const int32_t tok = items[0].idx;
        free(items);
        return tok;
    }
    int nucleus = limit;
    if (top_p < 1.0f) {
        double cum = 0.0;
        nucleus = 0;
        for (int i = 0; i < limit; i++) {
            cum += exp((double)items[i].score - (double)max_score) / sum;
            nucleus = i + 1;
            if (cum >= (double)top_p) break;
        }
        if (nucleus < 1) nucleus = 1;
    }
    double keep_sum = 0.0;
    for (int i = 0; i < nucleus; i++) keep_sum += exp((double)items[i].score - (double)max_score);
    const double target = u * keep_sum;
    double acc = 0.0;
    int32_t tok = items[nucleus - 1].idx;
    for (int i = 0; i < nucleus; i++) {
        acc += exp((double)items[i].score - (double)max_score);
        if (target <= acc) {
            tok = items[i].idx;
            break;
        }
    }
    free(items);
    return tok;
}
