/* qw6_moe_host.c -- host side of the routed-MoE entry points (C11). */
#define _POSIX_C_SOURCE 200809L

#include <stddef.h>
#include <string.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"

size_t qw6cu_moe_workspace_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts,
                                 uint32_t top_k) {
    return qw6k_moe_ws_bytes(ntok, hidden, inter, n_experts, top_k);
}

static int moe_desc(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                    const qw6cu_expert_pack *down, uint32_t ntok, uint32_t hidden, uint32_t inter,
                    uint32_t n_experts, uint32_t top_k, qw6k_moe_desc *d) {
    if (!gate || !up || !down || gate->quant != up->quant) {
        qw6h_set_err("qw6cu_moe_decode: gate and up packs must be given and share one quant type");
        return QW6CU_ERR_ARG;
    }
    d->gq = gate->quant;
    d->dq = down->quant;
    d->gate = gate->base;
    d->up = up->base;
    d->down = down->base;
    d->gstride = gate->stride;
    d->ustride = up->stride;
    d->dstride = down->stride;
    d->ntok = ntok;
    d->hidden = hidden;
    d->inter = inter;
    d->ne = n_experts;
    d->topk = top_k;
    d->ws_bytes = qw6k_moe_ws_bytes(ntok, hidden, inter, n_experts, top_k);
    d->ws = qw6h_buf(ctx, QW6H_BUF_WS, d->ws_bytes);
    return d->ws ? 0 : QW6CU_ERR_NOMEM;
}

static int moe_run(qw6cu_ctx *ctx, const qw6k_moe_desc *d) {
    int rc = qw6h_rc(qw6k_moe_check(d), "moe_decode");
    static const int kid[4] = {QW6H_K_MOE_PLAN, QW6H_K_MOE_GATEUP, QW6H_K_MOE_DOWN, QW6H_K_MOE_COMBINE};
    const int n = rc ? 0 : qw6k_moe_nphases(d);
    for (int ph = 0; ph < n && !rc; ph++) {
        const int rec = qw6h_prof_a(ctx, kid[qw6k_moe_phase_kind(d, ph)]);
        rc = qw6h_rc(qw6k_moe_phase(d, ph, ctx->st), "moe_decode");
        qw6h_prof_b(ctx, rec);
    }
    return rc;
}

int qw6cu_moe_decode(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                     const qw6cu_expert_pack *down, const float *logits, const float *x, float *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    if ((rc = moe_desc(ctx, gate, up, down, ntok, hidden, inter, n_experts, top_k, &d))) return rc;
    d.logits = logits;
    d.x = x;
    d.out = out;
    return moe_run(ctx, &d);
}

int qw6cu_moe_decode_hostio(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                            const qw6cu_expert_pack *down, const float *logits, const float *x, float *out,
                            uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!logits || !x || !out) {
        qw6h_set_err("qw6cu_moe_decode_hostio: null host buffer");
        return QW6CU_ERR_ARG;
    }
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    if ((rc = moe_desc(ctx, gate, up, down, ntok, hidden, inter, n_experts, top_k, &d))) return rc;
    const size_t lb = (size_t)ntok * n_experts * 4, xb = (size_t)ntok * hidden * 4;
    uint8_t *in = qw6h_buf(ctx, QW6H_BUF_X, ((lb + 255) & ~(size_t)255) + xb);
    float *dout = qw6h_buf(ctx, QW6H_BUF_Y, xb);
    if (!in || !dout) return QW6CU_ERR_NOMEM;
    d.logits = (const float *)in;
    d.x = (const float *)(in + ((lb + 255) & ~(size_t)255));
    d.out = dout;
    cudaError_t e = cudaMemcpyAsync((void *)d.logits, logits, lb, cudaMemcpyHostToDevice, ctx->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync((void *)d.x, x, xb, cudaMemcpyHostToDevice, ctx->st);
    if (e != cudaSuccess) {
        qw6h_set_err("qw6cu_moe_decode_hostio: H2D copy failed: %s", cudaGetErrorString(e));
        return QW6CU_ERR_CUDA;
    }
    rc = moe_run(ctx, &d);
    if (!rc && (e = cudaMemcpyAsync(out, dout, xb, cudaMemcpyDeviceToHost, ctx->st)) != cudaSuccess) {
        qw6h_set_err("qw6cu_moe_decode_hostio: D2H copy failed: %s", cudaGetErrorString(e));
        rc = QW6CU_ERR_CUDA;
    }
    e = cudaStreamSynchronize(ctx->st);
    if (!rc && e != cudaSuccess) {
        qw6h_set_err("qw6cu_moe_decode_hostio: %s", cudaGetErrorString(e));
        rc = QW6CU_ERR_CUDA;
    }
    return rc;
}

/* Allocation-free variant: the workspace is the library's fixed 1 MiB device
 * array (k_static.cu) instead of a context buffer, and work goes on the
 * caller's stream on the calling thread's current device. */
int qw6cu_moe_decode_noalloc(const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                             const qw6cu_expert_pack *down, const float *logits, const float *x, float *out,
                             uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k,
                             void *stream) {
    if (!gate || !up || !down || gate->quant != up->quant) {
        qw6h_set_err("qw6cu_moe_decode_noalloc: gate and up packs must be given and share one quant type");
        return QW6CU_ERR_ARG;
    }
    void *scratch = NULL;
    size_t cap = 0;
    if (qw6k_static_scratch(&scratch, &cap)) {
        qw6h_set_err("qw6cu_moe_decode_noalloc: first-call set-up on this device failed (cudaGetSymbolAddress of "
                     "the fixed scratch, or configuring the decode kernels)");
        return QW6CU_ERR_CUDA;
    }
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    d.gq = gate->quant;
    d.dq = down->quant;
    d.gate = gate->base;
    d.up = up->base;
    d.down = down->base;
    d.gstride = gate->stride;
    d.ustride = up->stride;
    d.dstride = down->stride;
    d.logits = logits;
    d.x = x;
    d.out = out;
    d.ntok = ntok;
    d.hidden = hidden;
    d.inter = inter;
    d.ne = n_experts;
    d.topk = top_k;
    d.ws = scratch;
    d.ws_bytes = qw6k_moe_ws_bytes(ntok, hidden, inter, n_experts, top_k);
    if (d.ws_bytes > cap) {
        qw6h_set_err("qw6cu_moe_decode_noalloc: this shape needs %zu bytes of scratch; the fixed scratch holds %zu "
                     "(use fewer tokens or qw6cu_moe_decode)",
                     d.ws_bytes, cap);
        return QW6CU_ERR_ARG;
    }
    int rc = qw6h_rc(qw6k_moe_check(&d), "moe_decode_noalloc");
    const int n = rc ? 0 : qw6k_moe_nphases(&d);
    for (int ph = 0; ph < n && !rc; ph++)
        rc = qw6h_rc(qw6k_moe_phase(&d, ph, (cudaStream_t)stream), "moe_decode_noalloc");
    return rc;
}

size_t qw6cu_moe_prefill_workspace_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts,
                                         uint32_t top_k) {
    return qw6k_moe_prefill_ws_bytes(ntok, hidden, inter, n_experts, top_k);
}

/* The prefill layer on ctx->st; the workspace and the error word must
 * already have their full size when the call is part of a pipeline. */
static int prefill_run(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                       const qw6cu_expert_pack *down, const float *logits, const void *x_bf16, float *out,
                       uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k) {
    int *err = qw6h_dev_err(ctx);
    if (!err) return QW6CU_ERR_NOMEM;
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    d.gq = gate->quant;
    d.dq = down->quant;
    d.gate = gate->base;
    d.up = up->base;
    d.down = down->base;
    d.gstride = gate->stride;
    d.ustride = up->stride;
    d.dstride = down->stride;
    d.logits = logits;
    d.x = (const float *)x_bf16;
    d.out = out;
    d.ntok = ntok;
    d.hidden = hidden;
    d.inter = inter;
    d.ne = n_experts;
    d.topk = top_k;
    d.ws_bytes = qw6k_moe_prefill_ws_bytes(ntok, hidden, inter, n_experts, top_k);
    d.ws = qw6h_buf(ctx, QW6H_BUF_WS, d.ws_bytes);
    if (!d.ws) return QW6CU_ERR_NOMEM;
    int rc = qw6h_rc(qw6k_moe_prefill_check(&d, err), "moe_prefill");
    static const int kid[7] = {QW6H_K_PF_PLAN,  QW6H_K_PF_PLAN,  QW6H_K_PF_PLAN, QW6H_K_PF_PLAN,
                               QW6H_K_PF_GEMM1, QW6H_K_PF_GEMM2, QW6H_K_PF_COMBINE};
    for (int ph = 0; ph < 7 && !rc; ph++) {
        const int rec = qw6h_prof_a(ctx, kid[ph]);
        rc = qw6h_rc(qw6k_moe_prefill_phase(&d, err, ph, ctx->st), "moe_prefill");
        qw6h_prof_b(ctx, rec);
    }
    return rc;
}

int qw6cu_moe_prefill(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                      const qw6cu_expert_pack *down, const float *logits, const void *x_bf16, float *out,
                      uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!gate || !up || !down || gate->quant != up->quant) {
        qw6h_set_err("qw6cu_moe_prefill: gate and up packs must be given and share one quant type");
        return QW6CU_ERR_ARG;
    }
    return prefill_run(ctx, gate, up, down, logits, x_bf16, out, ntok, hidden, inter, n_experts, top_k);
}

static int io_setup(qw6cu_ctx *ctx) {
    if (ctx->io_ready) return 0;
    cudaStream_t s[2];
    cudaError_t e = cudaSuccess;
    int ns = 0, ne = 0;
    for (; ns < 2; ns++)
        if ((e = cudaStreamCreateWithFlags(&s[ns], cudaStreamNonBlocking)) != cudaSuccess) break;
    for (; e == cudaSuccess && ne < 9; ne++)
        if ((e = cudaEventCreateWithFlags(&ctx->io_ev[ne], cudaEventDisableTiming)) != cudaSuccess) break;
    if (e != cudaSuccess) {
        for (int i = 0; i < ne; i++) cudaEventDestroy(ctx->io_ev[i]);
        for (int i = 0; i < ns; i++) cudaStreamDestroy(s[i]);
        qw6h_set_err("qw6cu_moe_prefill_hostio: creating copy streams/events: %s", cudaGetErrorString(e));
        return QW6CU_ERR_CUDA;
    }
    ctx->io_in = s[0];
    ctx->io_out = s[1];
    ctx->io_ready = 1;
    return 0;
}

/* The two-slot host-buffer pipeline shared by qw6cu_moe_prefill_hostio and
 * qw6cu_ep_layer_hostio: batch b's logits/x are copied in on io_in, run(b)
 * enqueues the layer on the context stream, and its output is read back on
 * io_out; slot b % 2 is reused only once batch b-2's experts consumed its
 * inputs and its output was read.  Drains all three streams before it
 * returns, also after an error. */
int qw6h_hostio_run(qw6cu_ctx *ctx, const char *what, const float *const *logits, const void *const *x_bf16,
                    float *const *out, uint32_t n_batches, size_t lg_bytes, size_t x_bytes, size_t out_bytes,
                    qw6h_hostio_fn run, void *arg) {
    if (!n_batches) return 0;
    if (!logits || !x_bf16 || !out) {
        qw6h_set_err("%s: null host pointer array", what);
        return QW6CU_ERR_ARG;
    }
    for (uint32_t b = 0; b < n_batches; b++)
        if (!logits[b] || !x_bf16[b] || !out[b]) {
            qw6h_set_err("%s: null host buffer of batch %u", what, b);
            return QW6CU_ERR_ARG;
        }
    int rc = io_setup(ctx);
    if (rc) return rc;
    const size_t lb = (lg_bytes + 255) & ~(size_t)255, xb = (x_bytes + 255) & ~(size_t)255;
    const size_t slot = lb + xb + ((out_bytes + 255) & ~(size_t)255);
    uint8_t *io = qw6h_buf(ctx, QW6H_BUF_IO, 2 * slot);
    if (!io) return QW6CU_ERR_NOMEM;
    cudaEvent_t *ev = ctx->io_ev;
    cudaStream_t cs = ctx->st;
    /* the copies start after the work already queued on the context stream
     * (including the zero-fill of freshly grown buffers) */
    cudaError_t e = cudaEventRecord(ev[0], cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->io_in, ev[0], 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->io_out, ev[0], 0);
    for (uint32_t b = 0; b < n_batches && e == cudaSuccess && !rc; b++) {
        const int s = (int)(b & 1);
        uint8_t *base = io + (size_t)s * slot;
        float *dl = (float *)base, *dout = (float *)(base + lb + xb);
        void *dx = base + lb;
        /* copy in once batch b-2 (same slot) has consumed its inputs */
        if ((e = cudaStreamWaitEvent(ctx->io_in, ev[3 + s], 0)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(dl, logits[b], lg_bytes, cudaMemcpyHostToDevice, ctx->io_in)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(dx, x_bf16[b], x_bytes, cudaMemcpyHostToDevice, ctx->io_in)) != cudaSuccess) break;
        if ((e = cudaEventRecord(ev[1 + s], ctx->io_in)) != cudaSuccess) break;
        /* run once the inputs landed and batch b-2's output has been read */
        if ((e = cudaStreamWaitEvent(cs, ev[1 + s], 0)) != cudaSuccess) break;
        if ((e = cudaStreamWaitEvent(cs, ev[7 + s], 0)) != cudaSuccess) break;
        if ((rc = run(arg, dl, dx, dout))) break;
        if ((e = cudaEventRecord(ev[3 + s], cs)) != cudaSuccess) break;
        if ((e = cudaEventRecord(ev[5 + s], cs)) != cudaSuccess) break;
        /* read back once the layer wrote it */
        if ((e = cudaStreamWaitEvent(ctx->io_out, ev[5 + s], 0)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(out[b], dout, out_bytes, cudaMemcpyDeviceToHost, ctx->io_out)) != cudaSuccess) break;
        if ((e = cudaEventRecord(ev[7 + s], ctx->io_out)) != cudaSuccess) break;
    }
    cudaError_t e2 = cudaStreamSynchronize(ctx->io_in);
    cudaError_t e3 = cudaStreamSynchronize(cs);
    cudaError_t e4 = cudaStreamSynchronize(ctx->io_out);
    if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3 != cudaSuccess ? e3 : e4;
    if (!rc && e != cudaSuccess) {
        qw6h_set_err("%s: %s", what, cudaGetErrorString(e));
        rc = QW6CU_ERR_CUDA;
    }
    return rc;
}

typedef struct {
    qw6cu_ctx *ctx;
    const qw6cu_expert_pack *gate, *up, *down;
    uint32_t ntok, hidden, inter, n_experts, top_k;
} prefill_job;

static int prefill_job_run(void *arg, const float *logits, const void *x_bf16, float *out) {
    const prefill_job *j = (const prefill_job *)arg;
    return prefill_run(j->ctx, j->gate, j->up, j->down, logits, x_bf16, out, j->ntok, j->hidden, j->inter,
                       j->n_experts, j->top_k);
}

int qw6cu_moe_prefill_hostio(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                             const qw6cu_expert_pack *down, const float *const *logits, const void *const *x_bf16,
                             float *const *out, uint32_t n_batches, uint32_t ntok, uint32_t hidden, uint32_t inter,
                             uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!gate || !up || !down || gate->quant != up->quant) {
        qw6h_set_err("qw6cu_moe_prefill_hostio: gate and up packs must be given and share one quant type");
        return QW6CU_ERR_ARG;
    }
    /* the workspace and the error word at their full size before the first
     * copy (growing one later would synchronize inside the pipeline) */
    if (n_batches &&
        (!qw6h_dev_err(ctx) ||
         !qw6h_buf(ctx, QW6H_BUF_WS, qw6k_moe_prefill_ws_bytes(ntok, hidden, inter, n_experts, top_k))))
        return QW6CU_ERR_NOMEM;
    prefill_job j = {ctx, gate, up, down, ntok, hidden, inter, n_experts, top_k};
    return qw6h_hostio_run(ctx, "qw6cu_moe_prefill_hostio", logits, x_bf16, out, n_batches,
                           (size_t)ntok * n_experts * 4, (size_t)ntok * hidden * 2, (size_t)ntok * hidden * 4,
                           prefill_job_run, &j);
}

int qw6cu_moe_expert_rows(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                          const qw6cu_expert_pack *down, const void *x_bf16, const int32_t *row_expert,
                          void *out_bf16, uint32_t nrows, uint32_t hidden, uint32_t inter, uint32_t n_experts) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!gate || !up || !down || gate->quant != up->quant || !row_expert || !out_bf16) {
        qw6h_set_err("qw6cu_moe_expert_rows: packs (gate/up of one quant type), row_expert and out are required");
        return QW6CU_ERR_ARG;
    }
    if (!nrows) return 0;
    int *err = qw6h_dev_err(ctx);
    if (!err) return QW6CU_ERR_NOMEM;
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    d.gq = gate->quant;
    d.dq = down->quant;
    d.gate = gate->base;
    d.up = up->base;
    d.down = down->base;
    d.gstride = gate->stride;
    d.ustride = up->stride;
    d.dstride = down->stride;
    d.x = (const float *)x_bf16;
    d.ntok = nrows;
    d.hidden = hidden;
    d.inter = inter;
    d.ne = n_experts;
    d.topk = 1;
    d.row_expert = row_expert;
    d.dout = out_bf16;
    d.ws_bytes = qw6k_moe_prefill_ws_bytes(nrows, hidden, inter, n_experts, 1);
    d.ws = qw6h_buf(ctx, QW6H_BUF_WS, d.ws_bytes);
    if (!d.ws) return QW6CU_ERR_NOMEM;
    rc = qw6h_rc(qw6k_moe_prefill_check(&d, err), "moe_expert_rows");
    static const int kid[6] = {QW6H_K_PF_PLAN, QW6H_K_PF_PLAN, QW6H_K_PF_PLAN, QW6H_K_PF_PLAN, QW6H_K_PF_GEMM1,
                               QW6H_K_PF_GEMM2};
    for (int ph = 1; ph < 6 && !rc; ph++) {
        const int rec = qw6h_prof_a(ctx, kid[ph]);
        rc = qw6h_rc(qw6k_moe_prefill_phase(&d, err, ph, ctx->st), "moe_expert_rows");
        qw6h_prof_b(ctx, rec);
    }
    return rc;
}

int qw6cu_ep_count(qw6cu_ctx *ctx, const int32_t *idx, uint32_t nassign, uint32_t n_experts, int32_t *expert_count,
                   int32_t *pos) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_EP);
    rc = qw6h_rc(qw6k_ep_count(idx, nassign, n_experts, expert_count, pos, ctx->st), "ep_count");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_ep_pack(qw6cu_ctx *ctx, const int32_t *idx, const int32_t *pos, const int32_t *expert_count,
                  uint32_t nassign, uint32_t top_k, uint32_t n_experts, const void *x_bf16, uint32_t hidden,
                  void *send_x, int32_t *send_pos) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_EP);
    rc = qw6h_rc(qw6k_ep_pack(idx, pos, expert_count, nassign, top_k, n_experts, x_bf16, hidden, send_x, send_pos,
                              ctx->st),
                 "ep_pack");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_ep_expand(qw6cu_ctx *ctx, const int32_t *recv_count, uint32_t world, uint32_t experts_per_rank,
                    int32_t *row_expert) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_EP);
    rc = qw6h_rc(qw6k_ep_expand(recv_count, world, experts_per_rank, row_expert, ctx->st), "ep_expand");
    qw6h_prof_b(ctx, rec);
    return rc;
}

int qw6cu_ep_combine(qw6cu_ctx *ctx, const void *ret_bf16, const float *w, const int32_t *send_pos, uint32_t ntok,
                     uint32_t top_k, uint32_t hidden, float *out) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const int rec = qw6h_prof_a(ctx, QW6H_K_EP);
    rc = qw6h_rc(qw6k_ep_combine(ret_bf16, w, send_pos, ntok, top_k, hidden, out, ctx->st), "ep_combine");
    qw6h_prof_b(ctx, rec);
    return rc;
}

/* ------------------------------------------------------ MoE FFN block -- */

static size_t al256h(size_t n) { return (n + 255) & ~(size_t)255; }

/* y[t] = W . x[t] for ntok tokens in chunks of the matvec's 32 */
static int block_matvec(qw6cu_ctx *ctx, uint32_t quant, const void *w, const float *x, float *y, uint32_t rows,
                        uint32_t cols, uint32_t ntok) {
    int rc = 0;
    for (uint32_t t0 = 0; t0 < ntok && !rc; t0 += 32) {
        const uint32_t n = ntok - t0 < 32 ? ntok - t0 : 32;
        const int rec = qw6h_prof_a(ctx, QW6H_K_MATVEC);
        rc = qw6h_rc(qw6k_matvec(quant, w, x + (size_t)t0 * cols, y + (size_t)t0 * rows, rows, cols, n, cols, rows,
                                 ctx->st),
                     "moe_block shared expert");
        qw6h_prof_b(ctx, rec);
    }
    return rc;
}

int qw6cu_moe_block(qw6cu_ctx *ctx, const float *x, const float *norm_w, const float *router,
                    const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up, const qw6cu_expert_pack *down,
                    const qw6cu_shared_expert *shared, float *out, uint32_t ntok, uint32_t hidden, uint32_t inter,
                    uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!x || !norm_w || !router || !out || !ntok || !hidden || !n_experts || n_experts > 256 ||
        (shared && (!shared->gate || !shared->up || !shared->down || !shared->inter))) {
        qw6h_set_err("qw6cu_moe_block: invalid arguments");
        return QW6CU_ERR_ARG;
    }
    const uint32_t si = shared ? shared->inter : 0;
    const size_t o_norm = 0, o_log = o_norm + al256h((size_t)ntok * hidden * 4),
                 o_sg = o_log + al256h((size_t)ntok * n_experts * 4), o_ffn = o_sg + al256h((size_t)ntok * 4),
                 o_g = o_ffn + al256h((size_t)ntok * hidden * 4), o_u = o_g + al256h((size_t)ntok * si * 4),
                 o_m = o_u + al256h((size_t)ntok * si * 4), o_sh = o_m + al256h((size_t)ntok * si * 4),
                 total = o_sh + (shared ? al256h((size_t)ntok * hidden * 4) : 0);
    uint8_t *b = qw6h_buf(ctx, QW6H_BUF_BLOCK, total);
    if (!b) return QW6CU_ERR_NOMEM;
    float *normed = (float *)(b + o_norm), *logits = (float *)(b + o_log), *sg = (float *)(b + o_sg);
    float *ffn = (float *)(b + o_ffn), *g = (float *)(b + o_g), *u = (float *)(b + o_u), *m = (float *)(b + o_m);
    float *sh = shared ? (float *)(b + o_sh) : NULL;
    qw6k_moe_desc d;
    memset(&d, 0, sizeof d);
    if ((rc = moe_desc(ctx, gate, up, down, ntok, hidden, inter, n_experts, top_k, &d))) return rc;
    d.logits = logits;
    d.x = normed;
    d.out = ffn;
    int rec = qw6h_prof_a(ctx, QW6H_K_MOE_BLOCK);
    rc = qw6h_rc(qw6k_block_pre(x, NULL, NULL, NULL, norm_w, router, shared ? shared->router : NULL, normed, logits,
                                sg, ntok, hidden, n_experts, ctx->st),
                 "moe_block");
    qw6h_prof_b(ctx, rec);
    if (!rc) rc = moe_run(ctx, &d);
    if (!rc && shared) {
        rc = block_matvec(ctx, shared->gate_quant, shared->gate, normed, g, si, hidden, ntok);
        if (!rc) rc = block_matvec(ctx, shared->up_quant, shared->up, normed, u, si, hidden, ntok);
        if (!rc) rc = qw6h_rc(qw6k_silu_mul(g, u, m, ntok * si, ctx->st), "moe_block shared expert");
        if (!rc) rc = block_matvec(ctx, shared->down_quant, shared->down, m, sh, hidden, si, ntok);
    }
    if (!rc) {
        rec = qw6h_prof_a(ctx, QW6H_K_MOE_BLOCK);
        rc = qw6h_rc(qw6k_block_post(x, ffn, sh, sg, out, NULL, ntok, hidden, ctx->st), "moe_block");
        qw6h_prof_b(ctx, rec);
    }
    return rc;
}
