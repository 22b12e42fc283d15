/* qw6_decoder.c -- the decode-step executor (host C11).
 *
 * qw6_forward_token (qw6.c:2426-2500) for one token, every weight resident on
 * the device, a whole step enqueued once and replayed as a CUDA graph:
 *   hidden = token_embd[token]                       (qw6.c:2456)
 *   per layer l:
 *     normed = rmsnorm(hidden) * norm                (qw6.c:2462-2463)
 *     attn   = DeltaNet(normed) if l % 4 != 3 else gated attention(normed, pos)
 *     hidden = hidden + attn                         (qw6.c:2469-2470)
 *     hidden = MoE FFN block(hidden)                 (qw6.c:2476-2484)
 *   logits = output . (rmsnorm(hidden) * output_norm) (qw6.c:2491-2495)
 * plus the greedy argmax of the logits (qw6_cpu_argmax, qw6.c:2858-2863),
 * which the graph also writes back as the next step's token, so that
 * qw6cu_decoder_generate chains steps with no host round trip.
 *
 * The step's token and position live in device memory (qw6k_step): the
 * graph does not depend on them.  Projections that read the same row are
 * packed into one matrix and run as one matvec ([qkv | z | beta | alpha] of
 * a DeltaNet layer, [q/gate | k | v] of an attention layer, the shared
 * expert's [gate | up]) when they share a quant type.
 */
#define _POSIX_C_SOURCE 200809L

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"
#include "qw6_formats.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"

enum {
    D_HID = 2048, D_QKV = 8192, D_Z = 4096, D_VH = 32, D_VD = 128, D_QFULL = 8192, D_KV = 512, D_HD = 256,
    D_NE = 256, D_TOPK = 8, D_INTER = 512, D_MAX_LAYERS = 40, D_VOCAB = 248320, D_PROJ = D_QKV + D_Z + 2 * D_VH
};

typedef struct {
    uint32_t quant, rows, cols;
    const void *w;
    uint32_t y_off; /* offset of the rows in the output vector */
} mv_job;

typedef struct {
    const void *key[4];
    uint32_t quant, rows, cols, count;
    void *dev;
    size_t dev_stride;
} upl_t;

typedef struct {
    int full;
    float *norm, *post_norm;
    mv_job in[4];
    int n_in;
    mv_job out;
    float *conv_w, *dt, *a, *dn_norm, *q_norm, *k_norm;
    float *router, *srouter;
    uint32_t gq, dq;
    const void *gate, *up, *down;
    size_t gstride, ustride, dstride;
    int shared, n_sgu;
    mv_job sgu[2], sdown;
    float *s0, *s1; /* DeltaNet state + conv window, or the k and v caches */
    size_t s0_bytes, s1_bytes;
} dlayer;

struct qw6cu_decoder {
    qw6cu_ctx *ctx;
    cudaStream_t st, st2;        /* st2: the shared expert, beside the routed experts */
    cudaEvent_t ev_fork, ev_join;
    uint32_t n_layers, max_ctx, vocab, embd_rows, embd_quant;
    const void *embd;
    float *out_norm;
    mv_job lm;
    dlayer L[D_MAX_LAYERS];
    void **allocs;
    size_t n_allocs, cap_allocs, bytes;
    upl_t *ups;
    size_t n_ups, cap_ups;
    uint8_t *stage;
    size_t stage_n;
    qw6k_step *step, *h_step;
    float *hid, *hid2, *normed, *proj, *gated, *qr, *part, *attn, *attn_out, *rlogits, *sgate, *ffn,
        *sgu, *smid, *sh, *logits, *freq;
    unsigned long long *keys;
    uint32_t *gen;
    uint32_t gen_cap;
    void *moe_ws;
    size_t moe_ws_bytes;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

static int cu(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 0;
    qw6h_set_err("qw6cu_decoder: %s: %s", what, cudaGetErrorString(e));
    return QW6CU_ERR_CUDA;
}

static int kr(int rc, const char *what) { return rc ? qw6h_rc(rc, what) : 0; }

static void *dalloc(qw6cu_decoder *d, size_t bytes) {
    if (d->n_allocs == d->cap_allocs) {
        const size_t cap = d->cap_allocs ? 2 * d->cap_allocs : 256;
        void **a = realloc(d->allocs, cap * sizeof *a);
        if (!a) return NULL;
        d->allocs = a;
        d->cap_allocs = cap;
    }
    void *p = NULL;
    if (cudaMalloc(&p, bytes ? (bytes + 255) & ~(size_t)255 : 256) != cudaSuccess) {
        qw6h_set_err("qw6cu_decoder: cudaMalloc of %zu bytes failed", bytes);
        return NULL;
    }
    d->allocs[d->n_allocs++] = p;
    d->bytes += bytes;
    return p;
}

/* host bytes into the staging buffer, ordered on the decoder's stream (a
 * plain cudaMemcpy from pageable memory may return before its DMA lands and
 * does not order against a non-blocking stream) */
static uint8_t *stage(qw6cu_decoder *d, const void *host, size_t bytes) {
    if (bytes > d->stage_n) {
        cudaStreamSynchronize(d->st);
        cudaFree(d->stage);
        d->stage = NULL;
        d->stage_n = 0;
        if (cudaMalloc((void **)&d->stage, bytes) != cudaSuccess) {
            qw6h_set_err("qw6cu_decoder: staging buffer of %zu bytes", bytes);
            return NULL;
        }
        d->stage_n = bytes;
    }
    if (cudaStreamSynchronize(d->st) != cudaSuccess ||
        cudaMemcpyAsync(d->stage, host, bytes, cudaMemcpyHostToDevice, d->st) != cudaSuccess) {
        qw6h_set_err("qw6cu_decoder: upload of %zu bytes failed", bytes);
        return NULL;
    }
    return d->stage;
}

static int is_block(uint32_t q) { return qw6_block_bytes(q) != 0; }
static int is_16(uint32_t q) { return q == QW6F_FP16 || q == QW6F_BF16; }

/* device bytes of `rows` x `cols` as the matvec reads them */
static size_t dev_bytes(uint32_t q, uint32_t rows, uint32_t cols) {
    if (q == QW6F_FP32) return (size_t)rows * cols * 4;
    return qw6k_packed_bytes(q, rows, cols);
}

static upl_t *find_upl(qw6cu_decoder *d, const void *const *key, uint32_t nkey, uint32_t quant, uint32_t rows,
                       uint32_t cols, uint32_t count) {
    for (size_t i = 0; i < d->n_ups; i++) {
        upl_t *u = &d->ups[i];
        if (u->quant != quant || u->rows != rows || u->cols != cols || u->count != count) continue;
        int same = 1;
        for (uint32_t k = 0; k < 4; k++) same &= u->key[k] == (k < nkey ? key[k] : NULL);
        if (same) return u;
    }
    return NULL;
}

static upl_t *add_upl(qw6cu_decoder *d, const void *const *key, uint32_t nkey, uint32_t quant, uint32_t rows,
                      uint32_t cols, uint32_t count, void *dev, size_t dev_stride) {
    if (d->n_ups == d->cap_ups) {
        const size_t cap = d->cap_ups ? 2 * d->cap_ups : 128;
        upl_t *u = realloc(d->ups, cap * sizeof *u);
        if (!u) return NULL;
        d->ups = u;
        d->cap_ups = cap;
    }
    upl_t *u = &d->ups[d->n_ups++];
    memset(u, 0, sizeof *u);
    for (uint32_t k = 0; k < nkey && k < 4; k++) u->key[k] = key[k];
    u->quant = quant;
    u->rows = rows;
    u->cols = cols;
    u->count = count;
    u->dev = dev;
    u->dev_stride = dev_stride;
    return u;
}

/* One matrix, or `count` of them `stride` bytes apart (an expert pack), into
 * the layout the kernels read. */
static void *upload_matrix(qw6cu_decoder *d, const qw6cu_model_tensor *t, uint32_t count, size_t *dev_stride) {
    const void *key[1] = {t->data};
    const upl_t *hit = find_upl(d, key, 1, t->quant, t->rows, t->cols, count);
    if (hit) {
        *dev_stride = hit->dev_stride;
        return hit->dev;
    }
    const size_t rb = qw6_row_bytes(t->quant, t->cols), one = (size_t)t->rows * rb;
    const size_t db = dev_bytes(t->quant, t->rows, t->cols), ds = count > 1 ? (db + 255) & ~(size_t)255 : db;
    const size_t raw_stride = count > 1 ? t->stride : one;
    if (!rb || !db || (count > 1 && t->stride < one)) {
        qw6h_set_err("qw6cu_decoder: tensor (field %u, layer %d) of quant %u, %u x %u cannot be uploaded", t->field,
                     t->layer, t->quant, t->rows, t->cols);
        return NULL;
    }
    void *dev = dalloc(d, ds * count);
    uint8_t *raw = dev ? stage(d, t->data, raw_stride * (count - 1) + one) : NULL;
    if (!raw) return NULL;
    if (t->quant == QW6F_FP32) {
        if (cu(cudaMemcpy2DAsync(dev, ds, raw, raw_stride, one, count, cudaMemcpyDeviceToDevice, d->st), "copy"))
            return NULL;
    } else if (kr(qw6k_pack(t->quant, raw, dev, t->rows, t->cols, count, raw_stride, ds, d->st), "pack")) {
        return NULL;
    }
    if (cu(cudaStreamSynchronize(d->st), "upload")) return NULL;
    *dev_stride = ds;
    return add_upl(d, key, 1, t->quant, t->rows, t->cols, count, dev, ds) ? dev : NULL;
}

/* Row 0 (or all rows: n = rows x cols) of a tensor as fp32 on the device. */
static float *upload_f32(qw6cu_decoder *d, const qw6cu_model_tensor *t, uint32_t n) {
    const void *key[1] = {t->data};
    const upl_t *hit = find_upl(d, key, 1, 1000u + t->quant, t->rows, t->cols, n);
    if (hit) return hit->dev;
    const size_t rb = qw6_row_bytes(t->quant, t->cols);
    const uint32_t rows = n / t->cols;
    if (!rb || !rows || (size_t)rows * t->cols != n || rows > t->rows) {
        qw6h_set_err("qw6cu_decoder: vector (field %u, layer %d) of quant %u, %u x %u", t->field, t->layer, t->quant,
                     t->rows, t->cols);
        return NULL;
    }
    float *dev = dalloc(d, (size_t)n * 4);
    uint8_t *raw = dev ? stage(d, t->data, rb * rows) : NULL;
    if (!raw) return NULL;
    if (t->quant == QW6F_FP32) {
        if (cu(cudaMemcpyAsync(dev, raw, (size_t)n * 4, cudaMemcpyDeviceToDevice, d->st), "copy")) return NULL;
    } else if (kr(qw6k_dequant(t->quant, raw, dev, rows, t->cols, d->st), "dequantize")) {
        return NULL;
    }
    if (cu(cudaStreamSynchronize(d->st), "upload")) return NULL;
    return add_upl(d, key, 1, 1000u + t->quant, t->rows, t->cols, n, dev, 0) ? (float *)dev : NULL;
}

/* Matrices read with the same input, stacked into as few matvecs as their
 * quant types allow; y_off[i] = where part i's rows go in the output. */
static int upload_group(qw6cu_decoder *d, const qw6cu_model_tensor *const *t, const uint32_t *y_off, int n,
                        mv_job *jobs, int *n_jobs) {
    *n_jobs = 0;
    for (int i = 0; i < n;) {
        int j = i + 1;
        /* a block-format part can only be followed when its rows fill whole 16-row tiles */
        while (j < n && t[j]->quant == t[i]->quant && t[j]->cols == t[i]->cols && y_off[j] == y_off[j - 1] + t[j - 1]->rows &&
               (!is_block(t[i]->quant) || t[j - 1]->rows % 16 == 0))
            j++;
        const void *key[4] = {0};
        uint32_t rows = 0;
        for (int k = i; k < j; k++) {
            if (k - i < 4) key[k - i] = t[k]->data;
            rows += t[k]->rows;
        }
        mv_job *jb = &jobs[(*n_jobs)++];
        jb->quant = t[i]->quant;
        jb->rows = rows;
        jb->cols = t[i]->cols;
        jb->y_off = y_off[i];
        const upl_t *hit = j - i <= 4 ? find_upl(d, key, (uint32_t)(j - i), t[i]->quant, rows, t[i]->cols, 0) : NULL;
        if (hit) {
            jb->w = hit->dev;
            i = j;
            continue;
        }
        uint8_t *dev = dalloc(d, dev_bytes(t[i]->quant, rows, t[i]->cols));
        if (!dev) return QW6CU_ERR_NOMEM;
        size_t off = 0;
        for (int k = i; k < j; k++) {
            const size_t one = (size_t)t[k]->rows * qw6_row_bytes(t[k]->quant, t[k]->cols);
            uint8_t *raw = stage(d, t[k]->data, one);
            if (!raw) return QW6CU_ERR_CUDA;
            int rc;
            if (t[k]->quant == QW6F_FP32)
                rc = cu(cudaMemcpyAsync(dev + off, raw, one, cudaMemcpyDeviceToDevice, d->st), "copy");
            else
                rc = kr(qw6k_pack(t[k]->quant, raw, dev + off, t[k]->rows, t[k]->cols, 1, one,
                                  dev_bytes(t[k]->quant, t[k]->rows, t[k]->cols), d->st),
                        "pack");
            if (rc) return rc;
            off += dev_bytes(t[k]->quant, t[k]->rows, t[k]->cols);
        }
        if (cu(cudaStreamSynchronize(d->st), "upload")) return QW6CU_ERR_CUDA;
        if (j - i <= 4 && !add_upl(d, key, (uint32_t)(j - i), t[i]->quant, rows, t[i]->cols, 0, dev, 0))
            return QW6CU_ERR_NOMEM;
        jb->w = dev;
        i = j;
    }
    return 0;
}

static int mv_on(cudaStream_t st, const mv_job *j, const float *x, float *y) {
    if (j->quant == QW6F_FP32)
        return kr(qw6k_matvec_f32((const float *)j->w, x, y + j->y_off, j->rows, j->cols, st), "matvec");
    return kr(qw6k_matvec(j->quant, j->w, x, y + j->y_off, j->rows, j->cols, 1, j->cols, j->rows, st), "matvec");
}

static int mv(const qw6cu_decoder *d, const mv_job *j, const float *x, float *y) { return mv_on(d->st, j, x, y); }

static const qw6cu_model_tensor *need(const qw6cu_model_tensor *const *tab, uint32_t field, int layer, uint32_t rows,
                                      uint32_t cols) {
    const qw6cu_model_tensor *t = tab[field];
    if (!t || !t->data) {
        qw6h_set_err("qw6cu_decoder: layer %d lacks tensor field %u", layer, field);
        return NULL;
    }
    if ((rows && t->rows != rows) || t->cols != cols) {
        qw6h_set_err("qw6cu_decoder: layer %d field %u is %u x %u, expected %u x %u", layer, field, t->rows, t->cols,
                     rows, cols);
        return NULL;
    }
    if (!qw6_row_bytes(t->quant, t->cols)) {
        qw6h_set_err("qw6cu_decoder: layer %d field %u has quant %u, which is not handled", layer, field, t->quant);
        return NULL;
    }
    return t;
}

static int weight_quant_ok(const qw6cu_model_tensor *t, int fp32_ok) {
    if (is_block(t->quant) || is_16(t->quant) || (fp32_ok && t->quant == QW6F_FP32)) return 1;
    qw6h_set_err("qw6cu_decoder: layer %d field %u: quant %u is not a matvec weight format", t->layer, t->field,
                 t->quant);
    return 0;
}

static int setup_layer(qw6cu_decoder *d, int l, const qw6cu_model_tensor *const *tab) {
    dlayer *L = &d->L[l];
    L->full = l % 4 == 3;
    const qw6cu_model_tensor *t;
    if (!(t = need(tab, QW6CU_F_NORM, l, 1, D_HID)) || !(L->norm = upload_f32(d, t, D_HID))) return QW6CU_ERR_ARG;
    if (!(t = need(tab, QW6CU_F_POST_NORM, l, 1, D_HID)) || !(L->post_norm = upload_f32(d, t, D_HID)))
        return QW6CU_ERR_ARG;
    const qw6cu_model_tensor *p[4];
    uint32_t off[4];
    int rc;
    if (!L->full) {
        if (!(p[0] = need(tab, QW6CU_F_ATTN_Q, l, D_QKV, D_HID)) || !(p[1] = need(tab, QW6CU_F_ATTN_GATE, l, D_Z, D_HID)) ||
            !(p[2] = need(tab, QW6CU_F_DN_BETA, l, D_VH, D_HID)) || !(p[3] = need(tab, QW6CU_F_DN_ALPHA, l, D_VH, D_HID)))
            return QW6CU_ERR_ARG;
        for (int i = 0; i < 4; i++)
            if (!weight_quant_ok(p[i], 1)) return QW6CU_ERR_QUANT;
        off[0] = 0, off[1] = D_QKV, off[2] = D_QKV + D_Z, off[3] = D_QKV + D_Z + D_VH;
        if ((rc = upload_group(d, p, off, 4, L->in, &L->n_in))) return rc;
        if (!(t = need(tab, QW6CU_F_DN_OUT, l, D_HID, D_Z)) || !weight_quant_ok(t, 1)) return QW6CU_ERR_ARG;
        p[0] = t, off[0] = 0;
        int one;
        if ((rc = upload_group(d, p, off, 1, &L->out, &one))) return rc;
        if (!(t = need(tab, QW6CU_F_CONV1D, l, D_QKV, 4))) return QW6CU_ERR_ARG;
        if (t->quant != QW6F_FP32) {  /* qw6 reads the conv weights as float (qw6.c:2333) */
            qw6h_set_err("qw6cu_decoder: layer %d conv1d must be FP32", l);
            return QW6CU_ERR_QUANT;
        }
        if (!(L->conv_w = upload_f32(d, t, D_QKV * 4))) return QW6CU_ERR_ARG;
        if (!(t = need(tab, QW6CU_F_DN_DT, l, 0, D_VH)) || !(L->dt = upload_f32(d, t, D_VH))) return QW6CU_ERR_ARG;
        if (!(t = need(tab, QW6CU_F_DN_A, l, 0, D_VH)) || !(L->a = upload_f32(d, t, D_VH))) return QW6CU_ERR_ARG;
        if (!(t = need(tab, QW6CU_F_DN_NORM, l, 0, D_VD)) || !(L->dn_norm = upload_f32(d, t, D_VD)))
            return QW6CU_ERR_ARG;
        L->s0_bytes = (size_t)D_VH * D_VD * D_VD * 4;
        L->s1_bytes = (size_t)4 * D_QKV * 4; /* conv window: ring of the 4 latest qkv rows */
    } else {
        if (!(p[0] = need(tab, QW6CU_F_ATTN_Q, l, D_QFULL, D_HID)) || !(p[1] = need(tab, QW6CU_F_ATTN_K, l, D_KV, D_HID)) ||
            !(p[2] = need(tab, QW6CU_F_ATTN_V, l, D_KV, D_HID)))
            return QW6CU_ERR_ARG;
        for (int i = 0; i < 3; i++)
            if (!weight_quant_ok(p[i], 1)) return QW6CU_ERR_QUANT;
        off[0] = 0, off[1] = D_QFULL, off[2] = D_QFULL + D_KV;
        if ((rc = upload_group(d, p, off, 3, L->in, &L->n_in))) return rc;
        if (!(t = need(tab, QW6CU_F_ATTN_O, l, D_HID, D_Z)) || !weight_quant_ok(t, 1)) return QW6CU_ERR_ARG;
        p[0] = t, off[0] = 0;
        int one;
        if ((rc = upload_group(d, p, off, 1, &L->out, &one))) return rc;
        if (!(t = need(tab, QW6CU_F_ATTN_Q_NORM, l, 0, D_HD)) || !(L->q_norm = upload_f32(d, t, D_HD)))
            return QW6CU_ERR_ARG;
        if (!(t = need(tab, QW6CU_F_ATTN_K_NORM, l, 0, D_HD)) || !(L->k_norm = upload_f32(d, t, D_HD)))
            return QW6CU_ERR_ARG;
        L->s0_bytes = L->s1_bytes = (size_t)d->max_ctx * D_KV * 4;
    }
    /* MoE FFN block */
    if (!(t = need(tab, QW6CU_F_MOE_ROUTER, l, D_NE, D_HID)) || !(L->router = upload_f32(d, t, D_NE * D_HID)))
        return QW6CU_ERR_ARG;
    const qw6cu_model_tensor *eg, *eu, *ed;
    if (!(eg = need(tab, QW6CU_F_EXPERT_GATE, l, D_INTER, D_HID)) || !(eu = need(tab, QW6CU_F_EXPERT_UP, l, D_INTER, D_HID)) ||
        !(ed = need(tab, QW6CU_F_EXPERT_DOWN, l, D_HID, D_INTER)))
        return QW6CU_ERR_ARG;
    if (eg->quant != eu->quant || !is_block(eg->quant) || !is_block(ed->quant)) {
        qw6h_set_err("qw6cu_decoder: layer %d experts: gate and up must share a block format, down a block format", l);
        return QW6CU_ERR_QUANT;
    }
    L->gq = eg->quant;
    L->dq = ed->quant;
    if (!(L->gate = upload_matrix(d, eg, D_NE, &L->gstride)) || !(L->up = upload_matrix(d, eu, D_NE, &L->ustride)) ||
        !(L->down = upload_matrix(d, ed, D_NE, &L->dstride)))
        return QW6CU_ERR_NOMEM;
    const qw6cu_model_tensor *sg = tab[QW6CU_F_SHARED_GATE], *su = tab[QW6CU_F_SHARED_UP], *sd = tab[QW6CU_F_SHARED_DOWN];
    L->shared = sg && su && sd && sg->data && su->data && sd->data; /* as qw6.c:2266-2267 */
    if (L->shared) {
        if (!(p[0] = need(tab, QW6CU_F_SHARED_GATE, l, D_INTER, D_HID)) ||
            !(p[1] = need(tab, QW6CU_F_SHARED_UP, l, D_INTER, D_HID)) ||
            !(t = need(tab, QW6CU_F_SHARED_DOWN, l, D_HID, D_INTER)) || !weight_quant_ok(p[0], 1) ||
            !weight_quant_ok(p[1], 1) || !weight_quant_ok(t, 1))
            return QW6CU_ERR_ARG;
        off[0] = 0, off[1] = D_INTER;
        if ((rc = upload_group(d, p, off, 2, L->sgu, &L->n_sgu))) return rc;
        p[0] = t, off[0] = 0;
        int one;
        if ((rc = upload_group(d, p, off, 1, &L->sdown, &one))) return rc;
        const qw6cu_model_tensor *sr = tab[QW6CU_F_SHARED_ROUTER];
        if (sr && sr->data) {
            if (!(t = need(tab, QW6CU_F_SHARED_ROUTER, l, 1, D_HID)) || !(L->srouter = upload_f32(d, t, D_HID)))
                return QW6CU_ERR_ARG;
        }
    }
    if (!(L->s0 = dalloc(d, L->s0_bytes)) || !(L->s1 = dalloc(d, L->s1_bytes))) return QW6CU_ERR_NOMEM;
    return 0;
}

static int enqueue_step(qw6cu_decoder *d) {
    cudaStream_t st = d->st;
    int *bad = &d->step->bad;
    int rc = kr(qw6k_dequant_row(d->embd_quant, d->embd, d->embd_rows, D_HID, &d->step->token, d->hid, bad, st),
                "embedding");
    /* the first layer's input norm; later ones come with the residual add that precedes them */
    if (!rc) rc = kr(qw6k_rmsnorm(d->hid, d->L[0].norm, d->normed, D_HID, st), "rmsnorm");
    for (uint32_t l = 0; l < d->n_layers && !rc; l++) {
        dlayer *L = &d->L[l];
        for (int j = 0; j < L->n_in && !rc; j++) rc = mv(d, &L->in[j], d->normed, d->proj);
        if (!rc && !L->full) {
            rc = kr(qw6k_dn_token(d->proj, d->step, L->s1, L->conv_w, L->dt, L->a, L->dn_norm, L->s0, d->gated, st),
                    "deltanet");
            if (!rc) rc = mv(d, &L->out, d->gated, d->attn_out);
        } else if (!rc) {
            rc = kr(qw6k_fa_prep(d->proj, L->q_norm, L->k_norm, d->freq, d->step, L->s0, L->s1, d->qr, st), "attention");
            if (!rc) rc = kr(qw6k_fa_attn(d->qr, L->s0, L->s1, d->step, d->part, d->proj, d->attn, st), "attention");
            if (!rc) rc = mv(d, &L->out, d->attn, d->attn_out);
        }
        if (!rc)
            rc = kr(qw6k_block_pre(d->hid, d->attn_out, d->hid2, bad, L->post_norm, L->router, L->srouter, d->normed,
                                   d->rlogits, d->sgate, 1, D_HID, D_NE, st),
                    "moe block");
        if (!rc && L->shared) rc = cu(cudaEventRecord(d->ev_fork, st), "fork");
        if (!rc) {
            qw6k_moe_desc m;
            memset(&m, 0, sizeof m);
            m.gq = L->gq, m.dq = L->dq, m.gate = L->gate, m.up = L->up, m.down = L->down;
            m.gstride = L->gstride, m.ustride = L->ustride, m.dstride = L->dstride;
            m.ntok = 1, m.hidden = D_HID, m.inter = D_INTER, m.ne = D_NE, m.topk = D_TOPK;
            m.logits = d->rlogits, m.x = d->normed, m.out = d->ffn, m.ws = d->moe_ws, m.ws_bytes = d->moe_ws_bytes;
            rc = kr(qw6k_moe_check(&m), "routed experts");
            const int np = rc ? 0 : qw6k_moe_nphases(&m);
            for (int ph = 0; ph < np && !rc; ph++) rc = kr(qw6k_moe_phase(&m, ph, st), "routed experts");
        }
        if (!rc && L->shared) { /* the shared expert on the second stream, joined before the residual add */
            rc = cu(cudaStreamWaitEvent(d->st2, d->ev_fork, 0), "fork");
            for (int j = 0; j < L->n_sgu && !rc; j++) rc = mv_on(d->st2, &L->sgu[j], d->normed, d->sgu);
            if (!rc) rc = kr(qw6k_silu_mul(d->sgu, d->sgu + D_INTER, d->smid, D_INTER, d->st2), "shared expert");
            if (!rc) rc = mv_on(d->st2, &L->sdown, d->smid, d->sh);
            if (!rc) rc = cu(cudaEventRecord(d->ev_join, d->st2), "join");
            if (!rc) rc = cu(cudaStreamWaitEvent(st, d->ev_join, 0), "join");
        }
        /* residual add, then the next layer's input norm (or the final norm) */
        const float *next_norm = l + 1 < d->n_layers ? d->L[l + 1].norm : d->out_norm;
        if (!rc)
            rc = kr(qw6k_post_norm(d->hid2, d->ffn, L->shared ? d->sh : NULL, d->sgate, d->hid, bad, next_norm,
                                   d->normed, 1, D_HID, st),
                    "moe block");
    }
    if (!rc)
        rc = kr(qw6k_matvec_argmax(d->lm.quant, d->lm.w, d->normed, d->logits, d->keys, d->vocab, D_HID, 1, D_HID,
                                   d->vocab, 0, st),
                "lm head");
    if (!rc) rc = kr(qw6k_check_finite(d->logits, d->vocab, bad, st), "lm head");
    if (!rc) rc = kr(qw6k_step_next(d->step, d->keys, st), "lm head");
    return rc;
}

int qw6cu_decoder_reset(qw6cu_decoder *d) {
    if (!d) return QW6CU_ERR_ARG;
    if (cu(cudaSetDevice(d->ctx->device), "set device")) return QW6CU_ERR_CUDA;
    for (uint32_t l = 0; l < d->n_layers; l++) {
        if (cu(cudaMemsetAsync(d->L[l].s0, 0, d->L[l].s0_bytes, d->st), "reset") ||
            cu(cudaMemsetAsync(d->L[l].s1, 0, d->L[l].s1_bytes, d->st), "reset"))
            return QW6CU_ERR_CUDA;
    }
    return cu(cudaStreamSynchronize(d->st), "reset");
}

/* one step with the step record already on the device; then read it back */
static int run(qw6cu_decoder *d, int graph) {
    int rc = graph ? cu(cudaGraphLaunch(d->exec, d->st), "graph launch") : enqueue_step(d);
    return rc;
}

int qw6cu_decoder_create(qw6cu_ctx *ctx, const qw6cu_model_tensor *tensors, uint32_t n_tensors, uint32_t n_layers,
                         uint32_t max_ctx, qw6cu_decoder **out) {
    if (!out) return QW6CU_ERR_ARG;
    *out = NULL;
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!tensors || !n_tensors || !n_layers || n_layers > D_MAX_LAYERS || !max_ctx || max_ctx > (1u << 24)) {
        qw6h_set_err("qw6cu_decoder_create: invalid arguments");
        return QW6CU_ERR_ARG;
    }
    const qw6cu_model_tensor *tab[D_MAX_LAYERS][QW6CU_F_EXPERT_DOWN + 1];
    const qw6cu_model_tensor *emb = NULL, *outw = NULL, *onorm = NULL;
    memset(tab, 0, sizeof tab);
    for (uint32_t i = 0; i < n_tensors; i++) {
        const qw6cu_model_tensor *t = &tensors[i];
        if (t->field == QW6CU_F_TOK_EMBD) emb = t;
        else if (t->field == QW6CU_F_OUTPUT) outw = t;
        else if (t->field == QW6CU_F_OUTPUT_NORM) onorm = t;
        else if (t->field <= QW6CU_F_EXPERT_DOWN && t->layer >= 0 && t->layer < (int32_t)n_layers)
            tab[t->layer][t->field] = t;
    }
    qw6cu_decoder *d = calloc(1, sizeof *d);
    if (!d) return QW6CU_ERR_NOMEM;
    d->ctx = ctx;
    d->n_layers = n_layers;
    d->max_ctx = max_ctx;
    if ((rc = cu(cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking), "stream")) ||
        (rc = cu(cudaStreamCreateWithFlags(&d->st2, cudaStreamNonBlocking), "stream")) ||
        (rc = cu(cudaEventCreateWithFlags(&d->ev_fork, cudaEventDisableTiming), "event")) ||
        (rc = cu(cudaEventCreateWithFlags(&d->ev_join, cudaEventDisableTiming), "event")))
        goto fail;
    rc = QW6CU_ERR_ARG;
    if (!emb || !emb->data || emb->cols != D_HID || !emb->rows || !qw6_row_bytes(emb->quant, D_HID)) {
        qw6h_set_err("qw6cu_decoder_create: token embeddings missing or not [rows x 2048] of a known quant");
        goto fail;
    }
    if (!outw || !outw->data || outw->cols != D_HID || !outw->rows || outw->rows > D_VOCAB || !is_block(outw->quant)) {
        qw6h_set_err("qw6cu_decoder_create: output weights missing or not [<= 248320 x 2048] of a block format");
        goto fail;
    }
    if (!onorm || !onorm->data || onorm->cols != D_HID) {
        qw6h_set_err("qw6cu_decoder_create: output norm missing or not 2048 wide");
        goto fail;
    }
    /* the embedding matrix stays in its raw form: a step dequantizes one row */
    d->embd_quant = emb->quant;
    d->embd_rows = emb->rows;
    {
        const size_t eb = (size_t)emb->rows * qw6_row_bytes(emb->quant, D_HID);
        void *e = dalloc(d, eb);
        if (!e || cu(cudaMemcpyAsync(e, emb->data, eb, cudaMemcpyHostToDevice, d->st), "embedding upload") ||
            cu(cudaStreamSynchronize(d->st), "embedding upload"))
            goto fail;
        d->embd = e;
    }
    if (!(d->out_norm = upload_f32(d, onorm, D_HID))) goto fail;
    {
        const qw6cu_model_tensor *p[1] = {outw};
        const uint32_t off[1] = {0};
        int one;
        if ((rc = upload_group(d, p, off, 1, &d->lm, &one))) goto fail;
        d->vocab = outw->rows;
        rc = QW6CU_ERR_ARG;
    }
    for (uint32_t l = 0; l < n_layers; l++)
        if ((rc = setup_layer(d, (int)l, tab[l]))) goto fail;
    rc = QW6CU_ERR_NOMEM;
    d->moe_ws_bytes = qw6k_moe_ws_bytes(1, D_HID, D_INTER, D_NE, D_TOPK);
    if (!(d->moe_ws = dalloc(d, d->moe_ws_bytes))) goto fail;
#define F32(ptr, n) if (!((ptr) = dalloc(d, (size_t)(n) * 4))) goto fail
    F32(d->hid, D_HID); F32(d->hid2, D_HID); F32(d->normed, D_HID); F32(d->proj, D_PROJ); F32(d->gated, D_Z); F32(d->qr, D_Z); F32(d->part, qw6k_fa_part_floats());
    F32(d->attn, D_Z); F32(d->attn_out, D_HID); F32(d->rlogits, D_NE); F32(d->sgate, 64); F32(d->ffn, D_HID);
    F32(d->sgu, 2 * D_INTER); F32(d->smid, D_INTER); F32(d->sh, D_HID); F32(d->logits, d->vocab); F32(d->freq, 32);
#undef F32
    if (!(d->keys = dalloc(d, 64)) || !(d->step = dalloc(d, sizeof(qw6k_step)))) goto fail;
    if ((rc = cu(cudaMallocHost((void **)&d->h_step, sizeof(qw6k_step)), "pinned step"))) goto fail;
    {
        /* RoPE frequencies as qw6 computes them: powf(theta, i / rotary_dims)
         * for even i < 64 (qw6.c:2727), with this host's libm */
        float f[32];
        for (int i = 0; i < 64; i += 2) f[i / 2] = powf(10000000.0f, (float)i / 64);
        if ((rc = cu(cudaMemcpyAsync(d->freq, f, sizeof f, cudaMemcpyHostToDevice, d->st), "rope table")) ||
            (rc = cu(cudaStreamSynchronize(d->st), "rope table")))
            goto fail;
    }
    /* one eager step sets up every kernel (attributes, module loading);
     * then the same step is captured and the state cleared */
    if ((rc = qw6cu_decoder_reset(d))) goto fail;
    memset(d->h_step, 0, sizeof *d->h_step);
    if ((rc = cu(cudaMemcpyAsync(d->step, d->h_step, sizeof *d->h_step, cudaMemcpyHostToDevice, d->st), "step")))
        goto fail;
    if ((rc = run(d, 0)) || (rc = cu(cudaStreamSynchronize(d->st), "first step"))) goto fail;
    if ((rc = cu(cudaStreamBeginCapture(d->st, cudaStreamCaptureModeThreadLocal), "capture"))) goto fail;
    rc = enqueue_step(d);
    {
        cudaGraph_t g = NULL;
        const int rc2 = cu(cudaStreamEndCapture(d->st, &g), "capture");
        if (!rc) rc = rc2;
        d->graph = g;
    }
    if (rc || (rc = cu(cudaGraphInstantiate(&d->exec, d->graph, 0), "graph instantiate"))) goto fail;
    if ((rc = qw6cu_decoder_reset(d))) goto fail;
    *out = d;
    return 0;
fail:
    qw6cu_decoder_destroy(d);
    return rc ? rc : QW6CU_ERR_ARG;
}

static int finish(qw6cu_decoder *d) {
    if (cu(cudaMemcpyAsync(d->h_step, d->step, sizeof *d->h_step, cudaMemcpyDeviceToHost, d->st), "step") ||
        cu(cudaStreamSynchronize(d->st), "step"))
        return QW6CU_ERR_CUDA;
    if (d->h_step->bad) {
        qw6h_set_err("qw6cu_decoder: non-finite value in the hidden state or the logits (or a token id past the "
                     "embedding rows)");
        return QW6CU_ERR_CUDA;
    }
    return 0;
}

int qw6cu_decoder_forward(qw6cu_decoder *d, uint32_t token, uint32_t pos, float *logits, uint32_t *greedy) {
    if (!d) return QW6CU_ERR_ARG;
    if (pos >= d->max_ctx || token >= d->embd_rows) {
        qw6h_set_err("qw6cu_decoder_forward: position %u or token %u out of range", pos, token);
        return QW6CU_ERR_ARG;
    }
    if (cu(cudaSetDevice(d->ctx->device), "set device")) return QW6CU_ERR_CUDA;
    d->h_step->token = token;
    d->h_step->pos = pos;
    d->h_step->bad = 0;
    int rc = cu(cudaMemcpyAsync(d->step, d->h_step, sizeof *d->h_step, cudaMemcpyHostToDevice, d->st), "step");
    if (!rc) rc = run(d, 1);
    if (!rc && logits)
        rc = cu(cudaMemcpyAsync(logits, d->logits, (size_t)d->vocab * 4, cudaMemcpyDeviceToHost, d->st), "logits");
    if (!rc) rc = finish(d);
    if (!rc && greedy) *greedy = d->h_step->token;
    return rc;
}

int qw6cu_decoder_generate(qw6cu_decoder *d, uint32_t token, uint32_t pos, uint32_t n, uint32_t *tokens) {
    if (!d || !tokens || !n) return QW6CU_ERR_ARG;
    if (pos >= d->max_ctx || n > d->max_ctx - pos || token >= d->embd_rows) {
        qw6h_set_err("qw6cu_decoder_generate: positions %u + %u past max_ctx or token %u out of range", pos, n, token);
        return QW6CU_ERR_ARG;
    }
    if (cu(cudaSetDevice(d->ctx->device), "set device")) return QW6CU_ERR_CUDA;
    if (n > d->gen_cap) {
        cudaFree(d->gen);
        d->gen = NULL;
        d->gen_cap = 0;
        if (cu(cudaMalloc((void **)&d->gen, (size_t)n * 4), "token buffer")) return QW6CU_ERR_NOMEM;
        d->gen_cap = n;
    }
    d->h_step->token = token;
    d->h_step->pos = pos;
    d->h_step->bad = 0;
    int rc = cu(cudaMemcpyAsync(d->step, d->h_step, sizeof *d->h_step, cudaMemcpyHostToDevice, d->st), "step");
    for (uint32_t i = 0; i < n && !rc; i++) {
        rc = run(d, 1);
        if (!rc)
            rc = cu(cudaMemcpyAsync(d->gen + i, &d->step->token, 4, cudaMemcpyDeviceToDevice, d->st), "token");
    }
    if (!rc) rc = cu(cudaMemcpyAsync(tokens, d->gen, (size_t)n * 4, cudaMemcpyDeviceToHost, d->st), "tokens");
    if (!rc) rc = finish(d);
    return rc;
}

const float *qw6cu_decoder_logits(qw6cu_decoder *d, uint32_t *rows) {
    if (!d) return NULL;
    if (rows) *rows = d->vocab;
    return d->logits;
}

size_t qw6cu_decoder_device_bytes(const qw6cu_decoder *d) { return d ? d->bytes : 0; }

void qw6cu_decoder_destroy(qw6cu_decoder *d) {
    if (!d) return;
    if (d->ctx) cudaSetDevice(d->ctx->device);
    if (d->st) cudaStreamSynchronize(d->st);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    for (size_t i = 0; i < d->n_allocs; i++) cudaFree(d->allocs[i]);
    cudaFree(d->stage);
    cudaFree(d->gen);
    if (d->h_step) cudaFreeHost(d->h_step);
    if (d->st2) cudaStreamSynchronize(d->st2);
    if (d->ev_fork) cudaEventDestroy(d->ev_fork);
    if (d->ev_join) cudaEventDestroy(d->ev_join);
    if (d->st2) cudaStreamDestroy(d->st2);
    if (d->st) cudaStreamDestroy(d->st);
    free(d->allocs);
    free(d->ups);
    free(d);
}
