/* qw6_ep_host.c -- expert-parallel MoE layer over peer memory (qw6cu_ep_*).
 *
 * One qw6cu_ep per rank (one process per GPU).  It owns:
 *   - a symmetric region (one cudaMalloc, identical layout on every rank):
 *     signal words, the double-buffered [2][world][ne] count matrix, the
 *     receive rows rx [cap][hidden] bf16 with the destination of each
 *     row's output, and ret [max_tokens * top_k][hidden] bf16, where the
 *     owners' down GEMM writes this rank's expert outputs;
 *     cap = world * max_tokens * top_k;
 *   - private buffers: step epoch, abort and dispatch-counter words, routing,
 *     per-expert counts/positions, send offsets and rows, and the grouped
 *     GEMM workspace.
 * The regions of the other ranks are mapped with CUDA IPC handles that the
 * caller exchanges (qw6cu_ep_handle -> all-gather -> qw6cu_ep_connect).
 * qw6cu_ep_layer then enqueues the whole layer on the context's stream with
 * no host synchronisation (so it can be captured in a CUDA graph):
 *   route -> count -> publish counts / plan -> dispatch rows -> wait rows ->
 *   grouped GEMMs over the received rows (sorted mode; the down GEMM writes
 *   every output row straight into its source's ret) -> signal outputs ->
 *   wait outputs -> local combine.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"

struct qw6cu_ep {
    qw6cu_ctx *ctx;
    uint64_t wait_ns; /* limit of the cross-GPU waits (0: the 2 s default) */
    uint32_t rank, world, ne, epr, topk, hidden, inter, max_tok, cap;
    uint8_t *region;
    size_t region_bytes, o_sig, o_cnt, o_rx, o_smeta, o_ret;
    uint8_t *peer_host[QW6K_EP_MAX_WORLD];
    int opened[QW6K_EP_MAX_WORLD];
    int connected;
    uint8_t *priv;
    uint8_t **peers_dev;
    uint32_t *epoch, *done_ctas;
    int *abort;
    int32_t *idx, *cnt_self, *pos, *sendoff, *local_cnt, *send_row, *ucnt, *upos, *ubase, *eslot;
    float *w;
    void *ws;
    size_t ws_bytes;
};

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

static int ep_fail(const char *what, cudaError_t e) {
    qw6h_set_err("%s: %s", what, cudaGetErrorString(e));
    return QW6CU_ERR_CUDA;
}

size_t qw6cu_ep_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int qw6cu_ep_create(qw6cu_ctx *ctx, uint32_t rank, uint32_t world, uint32_t n_experts, uint32_t top_k,
                    uint32_t hidden, uint32_t inter, uint32_t max_tokens, qw6cu_ep **out) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!out || !world || world > QW6K_EP_MAX_WORLD || rank >= world || !n_experts || n_experts > 256 ||
        n_experts % world || !top_k || top_k > 32 || top_k > n_experts || !hidden || hidden % 256 || !inter ||
        inter % 256 || !max_tokens || (uint64_t)world * max_tokens * top_k > (1u << 22)) {
        qw6h_set_err("qw6cu_ep_create: bad arguments");
        return QW6CU_ERR_ARG;
    }
    *out = NULL;
    qw6cu_ep *ep = (qw6cu_ep *)calloc(1, sizeof *ep);
    if (!ep) return QW6CU_ERR_NOMEM;
    ep->ctx = ctx;
    ep->rank = rank;
    ep->world = world;
    ep->ne = n_experts;
    ep->epr = n_experts / world;
    ep->topk = top_k;
    ep->hidden = hidden;
    ep->inter = inter;
    ep->max_tok = max_tokens;
    ep->cap = world * max_tokens * top_k;
    const size_t n = (size_t)max_tokens * top_k;
    ep->o_sig = 0;
    ep->o_cnt = al256(3 * QW6K_EP_MAX_WORLD * sizeof(uint32_t));
    ep->o_rx = ep->o_cnt + al256((size_t)2 * world * (n_experts + world) * sizeof(int32_t));
    ep->o_smeta = ep->o_rx + al256((size_t)ep->cap * hidden * 2);
    ep->o_ret = ep->o_smeta + al256((size_t)ep->cap * 8);
    ep->region_bytes = ep->o_ret + al256(n * hidden * 2);
    cudaError_t e = cudaMalloc((void **)&ep->region, ep->region_bytes);
    if (e != cudaSuccess) {
        free(ep);
        return ep_fail("qw6cu_ep_create: cudaMalloc(region)", e);
    }
    /* the sorted-mode grouped GEMM over up to cap received rows of epr experts */
    ep->ws_bytes = qw6k_moe_prefill_ws_bytes(ep->cap, hidden, inter, ep->epr, 1);
    size_t off = 0, o_peers, o_epoch, o_idx, o_w, o_cnt, o_pos, o_send, o_local, o_row, o_ucnt, o_upos, o_ubase,
           o_eslot, o_ws;
    o_peers = off; off += al256(QW6K_EP_MAX_WORLD * sizeof(void *));
    o_epoch = off; off += 256; /* epoch, abort, done_ctas */
    o_idx = off; off += al256(n * 4);
    o_w = off; off += al256(n * 4);
    o_cnt = off; off += al256(256 * 4);
    o_pos = off; off += al256(n * 4);
    o_send = off; off += al256(256 * 4);
    o_local = off; off += al256(256 * 4);
    o_row = off; off += al256(n * 4);
    o_ucnt = off; off += al256(QW6K_EP_MAX_WORLD * 4);
    o_upos = off; off += al256(n * 4);
    o_ubase = off; off += al256(QW6K_EP_MAX_WORLD * 4);
    o_eslot = off; off += al256(256 * 4);
    o_ws = off; off += al256(ep->ws_bytes);
    e = cudaMalloc((void **)&ep->priv, off);
    if (e != cudaSuccess) {
        cudaFree(ep->region);
        free(ep);
        return ep_fail("qw6cu_ep_create: cudaMalloc(private)", e);
    }
    ep->peers_dev = (uint8_t **)(ep->priv + o_peers);
    ep->epoch = (uint32_t *)(ep->priv + o_epoch);
    ep->abort = (int *)(ep->priv + o_epoch + 4);
    ep->done_ctas = (uint32_t *)(ep->priv + o_epoch + 8);
    ep->idx = (int32_t *)(ep->priv + o_idx);
    ep->w = (float *)(ep->priv + o_w);
    ep->cnt_self = (int32_t *)(ep->priv + o_cnt);
    ep->pos = (int32_t *)(ep->priv + o_pos);
    ep->sendoff = (int32_t *)(ep->priv + o_send);
    ep->local_cnt = (int32_t *)(ep->priv + o_local);
    ep->send_row = (int32_t *)(ep->priv + o_row);
    ep->ucnt = (int32_t *)(ep->priv + o_ucnt);
    ep->upos = (int32_t *)(ep->priv + o_upos);
    ep->ubase = (int32_t *)(ep->priv + o_ubase);
    ep->eslot = (int32_t *)(ep->priv + o_eslot);
    ep->ws = ep->priv + o_ws;
    /* signals and counts start at zero (epoch 0 = nothing published); rank r
     * owns experts [r*epr, (r+1)*epr) until qw6cu_ep_set_placement */
    int32_t ident[256];
    for (uint32_t g = 0; g < n_experts; g++) ident[g] = (int32_t)g;
    if ((e = cudaMemset(ep->region, 0, ep->o_rx)) != cudaSuccess ||
        (e = cudaMemset(ep->priv, 0, o_ws)) != cudaSuccess ||
        (e = cudaMemcpy(ep->eslot, ident, n_experts * sizeof(int32_t), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaDeviceSynchronize()) != cudaSuccess) {
        qw6cu_ep_destroy(ep);
        return ep_fail("qw6cu_ep_create: cudaMemset", e);
    }
    *out = ep;
    return 0;
}

int qw6cu_ep_handle(qw6cu_ep *ep, void *handle) {
    if (!ep || !handle) {
        qw6h_set_err("qw6cu_ep_handle: null argument");
        return QW6CU_ERR_ARG;
    }
    int rc = qw6h_use(ep->ctx);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, ep->region);
    if (e != cudaSuccess) return ep_fail("cudaIpcGetMemHandle", e);
    memcpy(handle, &h, sizeof h);
    return 0;
}

int qw6cu_ep_connect(qw6cu_ep *ep, const void *handles) {
    if (!ep || !handles || ep->connected) {
        qw6h_set_err("qw6cu_ep_connect: null argument or already connected");
        return QW6CU_ERR_ARG;
    }
    int rc = qw6h_use(ep->ctx);
    if (rc) return rc;
    for (uint32_t p = 0; p < ep->world; p++) {
        if (p == ep->rank) {
            ep->peer_host[p] = ep->region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)handles + (size_t)p * sizeof h, sizeof h);
        void *ptr = NULL;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return ep_fail("cudaIpcOpenMemHandle", e);
        ep->peer_host[p] = (uint8_t *)ptr;
        ep->opened[p] = 1;
    }
    cudaError_t e =
        cudaMemcpyAsync(ep->peers_dev, ep->peer_host, ep->world * sizeof(void *), cudaMemcpyHostToDevice, ep->ctx->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ep->ctx->st);
    if (e != cudaSuccess) return ep_fail("qw6cu_ep_connect: cudaMemcpyAsync", e);
    ep->connected = 1;
    return 0;
}

int qw6cu_ep_set_placement(qw6cu_ep *ep, const uint32_t *experts) {
    if (!ep || !experts) {
        qw6h_set_err("qw6cu_ep_set_placement: null argument");
        return QW6CU_ERR_ARG;
    }
    int32_t slot[256];
    for (uint32_t g = 0; g < ep->ne; g++) slot[g] = -1;
    for (uint32_t i = 0; i < ep->ne; i++) {
        if (experts[i] >= ep->ne || slot[experts[i]] >= 0) {
            qw6h_set_err("qw6cu_ep_set_placement: experts is not a permutation of 0..n_experts-1 (entry %u)", i);
            return QW6CU_ERR_ARG;
        }
        slot[experts[i]] = (int32_t)i;
    }
    int rc = qw6h_use(ep->ctx);
    if (rc) return rc;
    /* ordered on the layer's stream: steps enqueued before keep the old placement */
    cudaError_t e = cudaMemcpyAsync(ep->eslot, slot, ep->ne * sizeof(int32_t), cudaMemcpyHostToDevice, ep->ctx->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ep->ctx->st);
    return e == cudaSuccess ? 0 : ep_fail("qw6cu_ep_set_placement", e);
}

void qw6cu_ep_destroy(qw6cu_ep *ep) {
    if (!ep) return;
    if (qw6h_use(ep->ctx) == 0) cudaDeviceSynchronize();
    for (uint32_t p = 0; p < ep->world; p++)
        if (ep->opened[p]) cudaIpcCloseMemHandle(ep->peer_host[p]);
    cudaFree(ep->priv);
    cudaFree(ep->region);
    free(ep);
}

int qw6cu_ep_set_wait_limit(qw6cu_ep *ep, uint32_t ms) {
    if (!ep || !ms) {
        qw6h_set_err("qw6cu_ep_set_wait_limit: invalid arguments");
        return QW6CU_ERR_ARG;
    }
    ep->wait_ns = (uint64_t)ms * 1000000ull;
    return 0;
}

int qw6cu_ep_layer(qw6cu_ep *ep, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                   const qw6cu_expert_pack *down, const float *logits, const void *x_bf16, float *out,
                   uint32_t ntok) {
    if (!ep || !ep->connected || !gate || !up || !down || gate->quant != up->quant || !logits || !x_bf16 || !out ||
        !ntok || ntok > ep->max_tok) {
        qw6h_set_err("qw6cu_ep_layer: not connected, bad packs or ntok outside 1..max_tokens");
        return QW6CU_ERR_ARG;
    }
    qw6cu_ctx *ctx = ep->ctx;
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    int *err = qw6h_dev_err(ctx);
    if (!err) return QW6CU_ERR_NOMEM;
    int r = qw6h_prof_a(ctx, QW6H_K_ROUTE);
    rc = qw6h_rc(qw6k_moe_route(logits, ntok, ep->ne, ep->topk, ep->idx, ep->w, ctx->st), "ep route");
    qw6h_prof_b(ctx, r);
    if (rc) return rc;

    qw6k_ep_desc d;
    memset(&d, 0, sizeof d);
    d.peers = (uint8_t *const *)ep->peers_dev;
    d.o_sig = ep->o_sig;
    d.o_cnt = ep->o_cnt;
    d.o_rx = ep->o_rx;
    d.o_smeta = ep->o_smeta;
    d.o_ret = ep->o_ret;
    d.nmax = (uint32_t)(ep->max_tok * ep->topk);
    d.rank = ep->rank;
    d.world = ep->world;
    d.ne = ep->ne;
    d.topk = ep->topk;
    d.hidden = ep->hidden;
    d.ntok = ntok;
    d.cap = ep->cap;
    d.epoch = ep->epoch;
    d.abort = ep->abort;
    d.done_ctas = ep->done_ctas;
    d.err = err;
    d.wait_ns = ep->wait_ns;
    d.idx = ep->idx;
    d.w = ep->w;
    d.eslot = ep->eslot;
    d.cnt_self = ep->cnt_self;
    d.pos = ep->pos;
    d.ucnt = ep->ucnt;
    d.upos = ep->upos;
    d.ubase = ep->ubase;
    d.sendoff = ep->sendoff;
    d.local_cnt = ep->local_cnt;
    d.send_row = ep->send_row;
    d.x = x_bf16;
    d.out = out;

    qw6k_moe_desc m;
    memset(&m, 0, sizeof m);
    m.gq = gate->quant;
    m.dq = down->quant;
    m.gate = gate->base;
    m.up = up->base;
    m.down = down->base;
    m.gstride = gate->stride;
    m.ustride = up->stride;
    m.dstride = down->stride;
    m.x = (const float *)(ep->region + ep->o_rx);
    m.ntok = ep->cap;
    m.hidden = ep->hidden;
    m.inter = ep->inter;
    m.ne = ep->epr;
    m.topk = 1;
    m.out_peers = (uint8_t *const *)ep->peers_dev;
    m.out_off = ep->o_ret;
    m.slot_dst = (const int32_t *)(ep->region + ep->o_smeta) + 1;
    m.out_rows = ep->max_tok * ep->topk;
    m.expert_counts = ep->local_cnt;
    m.slot_row = (const int32_t *)(ep->region + ep->o_smeta);
    m.slot_stride = 2;
    m.ws = ep->ws;
    m.ws_bytes = ep->ws_bytes;
    rc = qw6h_rc(qw6k_moe_prefill_check(&m, err), "ep grouped GEMM");
    if (rc) return rc;

    /* publish/plan, dispatch, wait rows | GEMMs | signal, wait outputs, combine */
    static const int ep_kid[6] = {QW6H_K_EP_PUBLISH, QW6H_K_EP_DISPATCH, QW6H_K_EP_WAIT,
                                  QW6H_K_EP,         QW6H_K_EP_WAIT,     QW6H_K_EP_COMBINE};
    r = qw6h_prof_a(ctx, QW6H_K_EP);
    rc = qw6h_rc(qw6k_ep_p2p_phase(&d, 6, ctx->st), "ep count");
    qw6h_prof_b(ctx, r);
    for (int ph = 0; ph < 3 && !rc; ph++) {
        r = qw6h_prof_a(ctx, ep_kid[ph]);
        rc = qw6h_rc(qw6k_ep_p2p_phase(&d, ph, ctx->st), "ep phase");
        qw6h_prof_b(ctx, r);
    }
    static const int pf_phase[3] = {2, 4, 5};
    static const int pf_kid[3] = {QW6H_K_PF_PLAN, QW6H_K_PF_GEMM1, QW6H_K_PF_GEMM2};
    for (int i = 0; i < 3 && !rc; i++) {
        r = qw6h_prof_a(ctx, pf_kid[i]);
        rc = qw6h_rc(qw6k_moe_prefill_phase(&m, err, pf_phase[i], ctx->st), "ep grouped GEMM");
        qw6h_prof_b(ctx, r);
    }
    for (int ph = 3; ph < 6 && !rc; ph++) {
        r = qw6h_prof_a(ctx, ep_kid[ph]);
        rc = qw6h_rc(qw6k_ep_p2p_phase(&d, ph, ctx->st), "ep phase");
        qw6h_prof_b(ctx, r);
    }
    return rc;
}

typedef struct {
    qw6cu_ep *ep;
    const qw6cu_expert_pack *gate, *up, *down;
    uint32_t ntok;
} ep_job;

static int ep_job_run(void *arg, const float *logits, const void *x_bf16, float *out) {
    const ep_job *j = (const ep_job *)arg;
    return qw6cu_ep_layer(j->ep, j->gate, j->up, j->down, logits, x_bf16, out, j->ntok);
}

int qw6cu_ep_layer_hostio(qw6cu_ep *ep, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                          const qw6cu_expert_pack *down, const float *const *logits, const void *const *x_bf16,
                          float *const *out, uint32_t n_batches, uint32_t ntok) {
    if (!ep || !ep->connected || !ntok || ntok > ep->max_tok) {
        qw6h_set_err("qw6cu_ep_layer_hostio: not connected or ntok outside 1..max_tokens");
        return QW6CU_ERR_ARG;
    }
    int rc = qw6h_use(ep->ctx);
    if (rc) return rc;
    if (n_batches && !qw6h_dev_err(ep->ctx)) return QW6CU_ERR_NOMEM;
    ep_job j = {ep, gate, up, down, ntok};
    return qw6h_hostio_run(ep->ctx, "qw6cu_ep_layer_hostio", logits, x_bf16, out, n_batches,
                           (size_t)ntok * ep->ne * 4, (size_t)ntok * ep->hidden * 2, (size_t)ntok * ep->hidden * 4,
                           ep_job_run, &j);
}

int qw6cu_ep_last_rows(qw6cu_ep *ep, uint32_t *rows) {
    if (!ep || !rows) {
        qw6h_set_err("qw6cu_ep_last_rows: null argument");
        return QW6CU_ERR_ARG;
    }
    int rc = qw6h_use(ep->ctx);
    if (rc) return rc;
    int32_t c[256];
    cudaError_t e = cudaMemcpyAsync(c, ep->local_cnt, ep->epr * sizeof(int32_t), cudaMemcpyDeviceToHost, ep->ctx->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ep->ctx->st);
    if (e != cudaSuccess) return ep_fail("qw6cu_ep_last_rows", e);
    uint64_t s = 0;
    for (uint32_t i = 0; i < ep->epr; i++) s += (uint32_t)c[i];
    *rows = (uint32_t)s;
    return 0;
}
