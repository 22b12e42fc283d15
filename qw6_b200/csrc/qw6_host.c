/* qw6_host.c -- host side of libqw6cuda (C11 + CUDA runtime C API).
 *
 * Implements the drop-in entry points of include/qw6_vk.h (the per-call
 * host-memory API of qw6's Vulkan backend, qw6_vk.c:1186-1362) and the
 * device-resident API of include/qw6_cuda.h.  Kernels are reached through
 * the launchers of qw6_launch.h; nothing here computes on the CPU.
 */
#define _POSIX_C_SOURCE 200809L

#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"
#include "qw6_formats.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"
#include "qw6_vk.h"

/* ------------------------------------------------------------ errors --- */

static _Thread_local char g_err[512];

void qw6h_set_err(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

const char *qw6cu_last_error(void) { return g_err; }

static int cuda_fail(const char *what, cudaError_t e) {
    qw6h_set_err("%s: %s", what, cudaGetErrorString(e));
    return QW6CU_ERR_CUDA;
}

/* Map a launcher status to the public codes and record a message. */
int qw6h_rc(int rc, const char *what) {
    if (rc == 0) return 0;
    if (rc == QW6K_ERR_CUDA) {
        cudaError_t e = cudaGetLastError();
        qw6h_set_err("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
        return QW6CU_ERR_CUDA;
    }
    if (rc == QW6K_ERR_QUANT) qw6h_set_err("%s: unsupported quant type", what);
    else if (rc == QW6K_ERR_ALIGN) qw6h_set_err("%s: pointer or stride not 16-byte aligned", what);
    else if (rc == QW6K_ERR_TIMEOUT) qw6h_set_err("%s: bounded device wait timed out", what);
    else qw6h_set_err("%s: invalid argument", what);
    return rc;
}

/* ----------------------------------------------------------- context --- */

int qw6h_use(qw6cu_ctx *ctx) {
    if (!ctx) {
        qw6h_set_err("null context");
        return QW6CU_ERR_ARG;
    }
    cudaError_t e = cudaSetDevice(ctx->device);
    return e == cudaSuccess ? 0 : cuda_fail("cudaSetDevice", e);
}

int qw6cu_create(qw6cu_ctx **out, int device) {
    if (!out) {
        qw6h_set_err("qw6cu_create: null output");
        return QW6CU_ERR_ARG;
    }
    *out = NULL;
    if (device < 0) {
        const char *env = getenv("QW6_CUDA_DEVICE");
        device = env ? atoi(env) : 0;
    }
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail("cudaGetDeviceCount", e);
    if (device >= n) {
        qw6h_set_err("qw6cu_create: device %d not present (%d devices)", device, n);
        return QW6CU_ERR_ARG;
    }
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail("cudaSetDevice", e);
    struct cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail("cudaGetDeviceProperties", e);
    if (prop.major != 10) {
        qw6h_set_err("qw6cu_create: device %d is sm_%d%d; libqw6cuda is built for sm_100a only", device, prop.major,
                     prop.minor);
        return QW6CU_ERR_CUDA;
    }
    qw6cu_ctx *c = calloc(1, sizeof *c);
    if (!c) {
        qw6h_set_err("qw6cu_create: out of host memory");
        return QW6CU_ERR_NOMEM;
    }
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if ((e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking)) != cudaSuccess) {
        free(c);
        return cuda_fail("cudaStreamCreate", e);
    }
    c->st = c->own;
    *out = c;
    return 0;
}

static void prof_free(qw6cu_ctx *ctx) {
    for (int i = 0; i < ctx->prof_cap; i++) {
        cudaEventDestroy(ctx->prof[i].a);
        cudaEventDestroy(ctx->prof[i].b);
    }
    free(ctx->prof);
    ctx->prof = NULL;
    ctx->prof_cap = ctx->prof_n = ctx->prof_on = 0;
}

void qw6cu_destroy(qw6cu_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->st);
    if (ctx->io_ready) {
        cudaStreamSynchronize(ctx->io_in);
        cudaStreamSynchronize(ctx->io_out);
        for (int i = 0; i < 9; i++) cudaEventDestroy(ctx->io_ev[i]);
        cudaStreamDestroy(ctx->io_in);
        cudaStreamDestroy(ctx->io_out);
    }
    prof_free(ctx);
    for (int i = 0; i < QW6H_NBUF; i++) cudaFree(ctx->buf[i].p);
    cudaFreeHost(ctx->pinned);
    cudaStreamDestroy(ctx->own);
    free(ctx);
}

int qw6cu_set_stream(qw6cu_ctx *ctx, void *stream) {
    if (!ctx) {
        qw6h_set_err("null context");
        return QW6CU_ERR_ARG;
    }
    ctx->st = stream ? (cudaStream_t)stream : ctx->own;
    return 0;
}

void *qw6cu_get_stream(qw6cu_ctx *ctx) { return ctx ? (void *)ctx->st : NULL; }

int qw6cu_synchronize(qw6cu_ctx *ctx) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    cudaError_t e = cudaStreamSynchronize(ctx->st);
    return e == cudaSuccess ? 0 : cuda_fail("cudaStreamSynchronize", e);
}

/* Grow-only device buffer slot `i` of at least `bytes` (16-byte aligned).
 * Growing frees the old allocation, which synchronizes the device. */
void *qw6h_buf(qw6cu_ctx *ctx, int i, size_t bytes) {
    qw6h_buf_t *b = &ctx->buf[i];
    if (b->n >= bytes && b->p) return b->p;
    if (b->p) cudaFree(b->p);
    b->p = NULL;
    b->n = 0;
    size_t want = bytes < 256 ? 256 : bytes;
    cudaError_t e = cudaMalloc(&b->p, want);
    if (e != cudaSuccess) {
        b->p = NULL;
        qw6h_set_err("cudaMalloc(%zu): %s", want, cudaGetErrorString(e));
        return NULL;
    }
    b->n = want;
    /* new buffers start zeroed (the device error word relies on it) */
    cudaMemsetAsync(b->p, 0, want, ctx->st);
    return b->p;
}

/* --------------------------------------------------------- profiler --- */

static const char *k_names[QW6H_K_COUNT] = {"matvec",   "pack",       "dequant",  "route",       "argmax",
                                             "moe_plan", "moe_gateup", "moe_down", "moe_combine", "lm_head",
                                             "pf_plan",  "pf_gemm1",   "pf_gemm2", "pf_combine",  "ep",
                                             "ep_publish", "ep_dispatch", "ep_wait", "ep_combine", "moe_block", "sample"};

_Static_assert(QW6H_K_COUNT == QW6CU_NKERNELS, "kernel-id table and public QW6CU_NKERNELS disagree");

const char *qw6cu_kernel_name(int kid) { return kid >= 0 && kid < QW6H_K_COUNT ? k_names[kid] : "?"; }

int qw6cu_profile_begin(qw6cu_ctx *ctx, uint32_t max_launches) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    prof_free(ctx);
    if (max_launches == 0 || max_launches > (1u << 22)) {
        qw6h_set_err("qw6cu_profile_begin: capacity %u out of range", max_launches);
        return QW6CU_ERR_ARG;
    }
    ctx->prof = calloc(max_launches, sizeof *ctx->prof);
    if (!ctx->prof) {
        qw6h_set_err("qw6cu_profile_begin: out of host memory");
        return QW6CU_ERR_NOMEM;
    }
    for (uint32_t i = 0; i < max_launches; i++) {
        cudaError_t e1 = cudaEventCreate(&ctx->prof[i].a), e2 = cudaEventCreate(&ctx->prof[i].b);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            ctx->prof_cap = (int)i;
            prof_free(ctx);
            return cuda_fail("cudaEventCreate", e1 != cudaSuccess ? e1 : e2);
        }
        ctx->prof_cap = (int)i + 1;
    }
    ctx->prof_n = 0;
    ctx->prof_on = 1;
    return 0;
}

/* Inside stream capture an event must be recorded as an external node so
 * that the graph replay timestamps it. */
static void prof_record(cudaEvent_t ev, cudaStream_t st) {
    enum cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
    else
        cudaEventRecord(ev, st);
}

int qw6h_prof_a(qw6cu_ctx *ctx, int kid) {
    if (!ctx->prof_on || ctx->prof_n >= ctx->prof_cap) return -1;
    qw6h_prof_rec *r = &ctx->prof[ctx->prof_n];
    r->kid = kid;
    prof_record(r->a, ctx->st);
    return ctx->prof_n++;
}

void qw6h_prof_b(qw6cu_ctx *ctx, int rec) {
    if (rec >= 0) prof_record(ctx->prof[rec].b, ctx->st);
}

int qw6cu_profile_end(qw6cu_ctx *ctx, double *ms_total, uint32_t *launches) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    for (int k = 0; k < QW6H_K_COUNT; k++) {
        if (ms_total) ms_total[k] = 0.0;
        if (launches) launches[k] = 0;
    }
    cudaError_t e = cudaStreamSynchronize(ctx->st);
    if (e != cudaSuccess) return cuda_fail("cudaStreamSynchronize", e);
    for (int i = 0; i < ctx->prof_n; i++) {
        float ms = 0.f;
        if ((e = cudaEventElapsedTime(&ms, ctx->prof[i].a, ctx->prof[i].b)) != cudaSuccess) {
            prof_free(ctx);
            return cuda_fail("cudaEventElapsedTime", e);
        }
        if (ms_total) ms_total[ctx->prof[i].kid] += ms;
        if (launches) launches[ctx->prof[i].kid]++;
    }
    prof_free(ctx);
    return 0;
}

/* ------------------------------------------------------- device API --- */

size_t qw6cu_packed_bytes(uint32_t quant, uint32_t rows, uint32_t cols) { return qw6k_packed_bytes(quant, rows, cols); }

int qw6cu_pack(qw6cu_ctx *ctx, uint32_t quant, const void *raw, void *packed, uint32_t rows, uint32_t cols,
               uint32_t count, size_t raw_stride, size_t packed_stride) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const size_t rb = qw6_row_bytes(quant, cols) * rows, pb = qw6k_packed_bytes(quant, rows, cols);
    if (!pb || (count > 1 && (raw_stride < rb || packed_stride < pb))) {
        qw6h_set_err("qw6cu_pack: bad shape/strides (quant %u, %u x %u)", quant, rows, cols);
        return QW6CU_ERR_ARG;
    }
    const int rec = qw6h_prof_a(ctx, QW6H_K_PACK);
    rc = qw6h_rc(qw6k_pack(quant, raw, packed, rows, cols, count, raw_stride, packed_stride, ctx->st), "pack");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_dequantize(qw6cu_ctx *ctx, uint32_t quant, const void *raw, float *out, uint32_t rows, uint32_t cols) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_dequant(quant, raw, out, rows, cols, ctx->st), "dequantize");
}

int qw6cu_matvec(qw6cu_ctx *ctx, uint32_t quant, const void *packed, const float *x, float *y, uint32_t rows,
                 uint32_t cols, uint32_t ntok) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_MATVEC);
    rc = qw6h_rc(qw6k_matvec(quant, packed, x, y, rows, cols, ntok, cols, rows, ctx->st), "matvec");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_matvec_f32(qw6cu_ctx *ctx, const float *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_matvec_f32(w, x, y, rows, cols, ctx->st), "matvec_f32");
}

int qw6cu_moe_route(qw6cu_ctx *ctx, const float *logits, uint32_t ntok, uint32_t n_experts, uint32_t top_k,
                    int32_t *idx, float *w) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_moe_route(logits, ntok, n_experts, top_k, idx, w, ctx->st), "moe_route");
}

int qw6cu_silu_mul(qw6cu_ctx *ctx, const float *gate, const float *up, float *out, uint32_t n) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_silu_mul(gate, up, out, n, ctx->st), "silu_mul");
}

int qw6cu_moe_gather(qw6cu_ctx *ctx, const float *expert_out, const float *w, const float *shared_out,
                     float shared_weight, float *out, uint32_t dim, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_moe_gather(expert_out, w, shared_out, shared_weight, out, dim, top_k, ctx->st), "moe_gather");
}

int qw6cu_argmax(qw6cu_ctx *ctx, const float *x, uint32_t n, uint32_t *idx, float *val) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    unsigned long long *key = qw6h_buf(ctx, QW6H_BUF_KEY, 64);
    if (!key) return QW6CU_ERR_NOMEM;
    return qw6h_rc(qw6k_argmax(x, n, key, idx, val, ctx->st), "argmax");
}

int qw6cu_lm_head_argmax(qw6cu_ctx *ctx, uint32_t quant, const void *packed, const float *x, uint32_t ntok,
                         uint32_t rows, uint32_t cols, uint32_t row_offset, unsigned long long *keys, float *logits) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_LM_HEAD);
    rc = qw6h_rc(qw6k_matvec_argmax(quant, packed, x, logits, keys, rows, cols, ntok, cols, rows, row_offset, ctx->st),
                 "lm_head_argmax");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_sample(qw6cu_ctx *ctx, const float *logits, uint32_t n, uint32_t nrows, float temp, float top_p, int top_k,
                 const float *u, uint32_t *token) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!logits || !u || !token || !n || !nrows) {
        qw6h_set_err("qw6cu_sample: invalid arguments");
        return QW6CU_ERR_ARG;
    }
    const size_t wb = qw6k_sample_ws_bytes(nrows);
    void *ws = qw6h_buf(ctx, QW6H_BUF_SAMPLE, wb);
    if (!ws) return QW6CU_ERR_NOMEM;
    const int rec = qw6h_prof_a(ctx, QW6H_K_SAMPLE);
    rc = qw6h_rc(qw6k_sample(logits, n, n, nrows, temp, top_p, top_k, u, token, ws, wb, ctx->st), "sample");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_argmax_keys_reduce(qw6cu_ctx *ctx, const unsigned long long *keys, uint32_t nshards, uint32_t ntok,
                             uint32_t *idx, float *val) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    return qw6h_rc(qw6k_argmax_keys_reduce(keys, nshards, ntok, idx, val, ctx->st), "argmax_keys_reduce");
}

/* Device error word of the context (bounded waits record timeouts here). */
int *qw6h_dev_err(qw6cu_ctx *ctx) {
    uint8_t *k = qw6h_buf(ctx, QW6H_BUF_KEY, 64);
    return k ? (int *)(k + 32) : NULL;
}

int qw6cu_gemm_bf16_nt(qw6cu_ctx *ctx, const void *A, const void *B, float *D, uint32_t M, uint32_t N, uint32_t K) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    int *err = qw6h_dev_err(ctx);
    if (!err) return QW6CU_ERR_NOMEM;
    return qw6h_rc(qw6k_gemm_bf16_nt(A, B, D, M, N, K, err, ctx->st), "gemm_bf16_nt");
}

int qw6cu_check_device_errors(qw6cu_ctx *ctx) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    int *err = qw6h_dev_err(ctx);
    if (!err) return QW6CU_ERR_NOMEM;
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, err, sizeof h, cudaMemcpyDeviceToHost, ctx->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
    if (e != cudaSuccess) return cuda_fail("qw6cu_check_device_errors", e);
    if (h) {
        cudaMemsetAsync(err, 0, sizeof h, ctx->st);
        cudaStreamSynchronize(ctx->st);
        qw6h_set_err("a device-side bounded wait timed out (code %d); the kernel returned without its result", h);
        return QW6CU_ERR_TIMEOUT;
    }
    return 0;
}

/* ------------------------------------------ per-call host entry points --- */

static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
static qw6cu_ctx *g_default;

/* Process-wide context of the qw6_vk_*_host calls (created on first use). */
qw6cu_ctx *qw6h_default_locked(void) {
    if (!g_default && qw6cu_create(&g_default, -1) != 0) g_default = NULL;
    return g_default;
}

static int h2d(qw6cu_ctx *c, void *dst, const void *src, size_t n) {
    cudaError_t e = cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, c->st);
    return e == cudaSuccess ? 0 : cuda_fail("cudaMemcpyAsync H2D", e);
}
static int d2h(qw6cu_ctx *c, void *dst, const void *src, size_t n) {
    cudaError_t e = cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, c->st);
    return e == cudaSuccess ? 0 : cuda_fail("cudaMemcpyAsync D2H", e);
}
static int finish(qw6cu_ctx *c, int rc) {
    cudaError_t e = cudaStreamSynchronize(c->st);
    if (rc == 0 && e != cudaSuccess) rc = cuda_fail("cudaStreamSynchronize", e);
    return rc;
}

static int host_matmul(uint32_t quant, const void *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                       const char *name) {
    if (!w || !x || !y || rows == 0 || cols == 0 || cols % 256) {
        qw6h_set_err("%s: invalid arguments (rows %u, cols %u; cols must be a multiple of 256)", name, rows, cols);
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    const size_t rb = qw6_row_bytes(quant, cols) * (size_t)rows, pb = qw6k_packed_bytes(quant, rows, cols);
    void *draw = NULL, *dpk = NULL;
    float *dx = NULL, *dy = NULL;
    if (!rc) {
        draw = qw6h_buf(c, QW6H_BUF_RAW, rb);
        dpk = qw6h_buf(c, QW6H_BUF_PACKED, pb);
        dx = qw6h_buf(c, QW6H_BUF_X, (size_t)cols * 4);
        dy = qw6h_buf(c, QW6H_BUF_Y, (size_t)rows * 4);
        if (!draw || !dpk || !dx || !dy) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, draw, w, rb);
    if (!rc) rc = h2d(c, dx, x, (size_t)cols * 4);
    if (!rc) rc = qw6h_rc(qw6k_pack(quant, draw, dpk, rows, cols, 1, rb, pb, c->st), name);
    if (!rc) rc = qw6h_rc(qw6k_matvec(quant, dpk, dx, dy, rows, cols, 1, cols, rows, c->st), name);
    if (!rc) rc = d2h(c, y, dy, (size_t)rows * 4);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    return rc ? -1 : 0;
}

int qw6_vk_matmul_q4k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_Q4_K_M, w, x, y, rows, cols, "qw6_vk_matmul_q4k_host");
}
int qw6_vk_matmul_q5k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_Q5_K, w, x, y, rows, cols, "qw6_vk_matmul_q5k_host");
}
int qw6_vk_matmul_q6k_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_Q6_K, w, x, y, rows, cols, "qw6_vk_matmul_q6k_host");
}
int qw6_vk_matmul_iq2xxs_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_IQ2_XXS, w, x, y, rows, cols, "qw6_vk_matmul_iq2xxs_host");
}
int qw6_vk_matmul_iq2s_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_IQ2_S, w, x, y, rows, cols, "qw6_vk_matmul_iq2s_host");
}
int qw6_vk_matmul_iq3s_host(const void *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    return host_matmul(QW6F_IQ3_S, w, x, y, rows, cols, "qw6_vk_matmul_iq3s_host");
}

int qw6_vk_matvec_f32_host(const float *w, const float *x, float *y, uint32_t rows, uint32_t cols) {
    if (!w || !x || !y || rows == 0 || cols == 0) {
        qw6h_set_err("qw6_vk_matvec_f32_host: invalid arguments");
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    const size_t wb = (size_t)rows * cols * 4;
    float *dw = NULL, *dx = NULL, *dy = NULL;
    if (!rc) {
        dw = qw6h_buf(c, QW6H_BUF_RAW, wb);
        dx = qw6h_buf(c, QW6H_BUF_X, (size_t)cols * 4);
        dy = qw6h_buf(c, QW6H_BUF_Y, (size_t)rows * 4);
        if (!dw || !dx || !dy) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, dw, w, wb);
    if (!rc) rc = h2d(c, dx, x, (size_t)cols * 4);
    if (!rc) rc = qw6h_rc(qw6k_matvec_f32(dw, dx, dy, rows, cols, c->st), "qw6_vk_matvec_f32_host");
    if (!rc) rc = d2h(c, y, dy, (size_t)rows * 4);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    return rc ? -1 : 0;
}

int qw6_vk_silu_mul_host(const float *gate, const float *up, float *out, uint32_t n) {
    if (!gate || !up || !out || n == 0) {
        qw6h_set_err("qw6_vk_silu_mul_host: invalid arguments");
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    float *dg = NULL, *du = NULL, *dout = NULL;
    if (!rc) {
        dg = qw6h_buf(c, QW6H_BUF_RAW, (size_t)n * 4);
        du = qw6h_buf(c, QW6H_BUF_X, (size_t)n * 4);
        dout = qw6h_buf(c, QW6H_BUF_Y, (size_t)n * 4);
        if (!dg || !du || !dout) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, dg, gate, (size_t)n * 4);
    if (!rc) rc = h2d(c, du, up, (size_t)n * 4);
    if (!rc) rc = qw6h_rc(qw6k_silu_mul(dg, du, dout, n, c->st), "qw6_vk_silu_mul_host");
    if (!rc) rc = d2h(c, out, dout, (size_t)n * 4);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    return rc ? -1 : 0;
}

static int host_argmax(const float *x, uint32_t n, uint32_t *out_idx, float *out_val, const char *name) {
    if (!x || n == 0 || !out_idx) {
        qw6h_set_err("%s: invalid arguments", name);
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    float *dx = NULL;
    uint32_t *dres = NULL;
    unsigned long long *key = NULL;
    if (!rc) {
        dx = qw6h_buf(c, QW6H_BUF_X, (size_t)n * 4);
        dres = qw6h_buf(c, QW6H_BUF_Y, 64);
        key = qw6h_buf(c, QW6H_BUF_KEY, 64);
        if (!dx || !dres || !key) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, dx, x, (size_t)n * 4);
    if (!rc) rc = qw6h_rc(qw6k_argmax(dx, n, key, dres, (float *)(dres + 1), c->st), name);
    uint32_t res[2] = {0, 0};
    if (!rc) rc = d2h(c, res, dres, sizeof res);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    if (rc) return -1;
    *out_idx = res[0];
    if (out_val) memcpy(out_val, &res[1], 4);
    return 0;
}

int qw6_vk_argmax_host(const float *x, uint32_t n, uint32_t *out_idx, float *out_val) {
    return host_argmax(x, n, out_idx, out_val, "qw6_vk_argmax_host");
}

int qw6_vk_sampling_greedy_host(const float *logits, uint32_t n, uint32_t *token) {
    return host_argmax(logits, n, token, NULL, "qw6_vk_sampling_greedy_host");
}

int qw6_vk_moe_route_host(const float *logits, uint32_t *indices, float *weights, uint32_t n_experts,
                          uint32_t top_k) {
    /* same limits as qw6_vk_moe_route (qw6_vk.c:906) */
    if (!logits || !indices || !weights || n_experts == 0 || n_experts > 256 || top_k == 0 || top_k > n_experts ||
        top_k > 8) {
        qw6h_set_err("qw6_vk_moe_route_host: invalid arguments (n_experts %u, top_k %u)", n_experts, top_k);
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    float *dl = NULL;
    int32_t *di = NULL;
    if (!rc) {
        dl = qw6h_buf(c, QW6H_BUF_X, (size_t)n_experts * 4);
        di = qw6h_buf(c, QW6H_BUF_Y, 2 * 8 * 4);
        if (!dl || !di) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, dl, logits, (size_t)n_experts * 4);
    if (!rc) rc = qw6h_rc(qw6k_moe_route(dl, 1, n_experts, top_k, di, (float *)(di + 8), c->st), "moe_route");
    int32_t res[16];
    if (!rc) rc = d2h(c, res, di, sizeof res);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    if (rc) return -1;
    for (uint32_t k = 0; k < top_k; k++) indices[k] = (uint32_t)res[k];
    memcpy(weights, res + 8, top_k * 4);
    return 0;
}

int qw6_vk_moe_gather_host(const float *expert_out, const float *expert_weights, const float *shared_out,
                           float shared_weight, float *out, uint32_t dim, uint32_t top_k) {
    /* same limits as qw6_vk_moe_gather (qw6_vk.c:933) */
    if (!expert_out || !expert_weights || !out || dim == 0 || top_k == 0 || top_k > 8) {
        qw6h_set_err("qw6_vk_moe_gather_host: invalid arguments (dim %u, top_k %u)", dim, top_k);
        return -1;
    }
    pthread_mutex_lock(&g_lock);
    qw6cu_ctx *c = qw6h_default_locked();
    int rc = c ? qw6h_use(c) : -1;
    float *de = NULL, *dw = NULL, *ds = NULL, *dout = NULL;
    if (!rc) {
        de = qw6h_buf(c, QW6H_BUF_RAW, (size_t)top_k * dim * 4);
        dw = qw6h_buf(c, QW6H_BUF_KEY, 64);
        ds = qw6h_buf(c, QW6H_BUF_X, (size_t)dim * 4);
        dout = qw6h_buf(c, QW6H_BUF_Y, (size_t)dim * 4);
        if (!de || !dw || !ds || !dout) rc = QW6CU_ERR_NOMEM;
    }
    if (!rc) rc = h2d(c, de, expert_out, (size_t)top_k * dim * 4);
    if (!rc) rc = h2d(c, dw, expert_weights, (size_t)top_k * 4);
    if (!rc && shared_out) rc = h2d(c, ds, shared_out, (size_t)dim * 4);
    if (!rc)
        rc = qw6h_rc(qw6k_moe_gather(de, dw, shared_out ? ds : NULL, shared_weight, dout, dim, top_k, c->st),
                     "moe_gather");
    if (!rc) rc = d2h(c, out, dout, (size_t)dim * 4);
    if (c) rc = finish(c, rc);
    pthread_mutex_unlock(&g_lock);
    return rc ? -1 : 0;
}

/* ---- entry points of qw6_vk.h outside this library's path ---- */

static int not_provided(const char *name) {
    qw6h_set_err("%s: not provided by libqw6cuda (outside the quantized matvec / MoE path)", name);
    return -1;
}

int qw6_vk_rmsnorm_host(const float *x, const float *w, float *y, uint32_t n, float eps) {
    (void)x; (void)w; (void)y; (void)n; (void)eps;
    return not_provided("qw6_vk_rmsnorm_host");
}
int qw6_vk_rmsnorm_chunked_host(const float *x, const float *w, float *y, uint32_t n, float eps, uint32_t g) {
    (void)x; (void)w; (void)y; (void)n; (void)eps; (void)g;
    return not_provided("qw6_vk_rmsnorm_chunked_host");
}
int qw6_vk_attention_gqa_host(const float *q, const float *k, const float *v, float *o, uint32_t s, uint32_t a,
                              uint32_t b, uint32_t d) {
    (void)q; (void)k; (void)v; (void)o; (void)s; (void)a; (void)b; (void)d;
    return not_provided("qw6_vk_attention_gqa_host");
}
int qw6_vk_deltanet_conv1d_host(const float *x, const uint16_t *w, float *o, uint32_t d, uint32_t k) {
    (void)x; (void)w; (void)o; (void)d; (void)k;
    return not_provided("qw6_vk_deltanet_conv1d_host");
}
int qw6_vk_deltanet_retrieve_host(const float *s, const float *q, float *o, uint32_t a, uint32_t b, uint32_t c,
                                  uint32_t d) {
    (void)s; (void)q; (void)o; (void)a; (void)b; (void)c; (void)d;
    return not_provided("qw6_vk_deltanet_retrieve_host");
}
int qw6_vk_deltanet_update_host(float *s, const float *k, const float *v, const float *q, const float *be,
                                uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    (void)s; (void)k; (void)v; (void)q; (void)be; (void)a; (void)b; (void)c; (void)d;
    return not_provided("qw6_vk_deltanet_update_host");
}
int qw6_vk_mrope_host(float *q, float *k, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t p, uint32_t r) {
    (void)q; (void)k; (void)a; (void)b; (void)c; (void)d; (void)p; (void)r;
    return not_provided("qw6_vk_mrope_host");
}
int qw6_vk_mtp_draft_host(const float *w, const float *h, float *l, uint32_t v, uint32_t hs) {
    (void)w; (void)h; (void)l; (void)v; (void)hs;
    return not_provided("qw6_vk_mtp_draft_host");
}

