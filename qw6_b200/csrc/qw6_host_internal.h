/* qw6_host_internal.h -- context struct and helpers shared by the host C
 * files of libqw6cuda (not installed). */
#ifndef QW6_HOST_INTERNAL_H
#define QW6_HOST_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"

enum {
    QW6H_BUF_RAW = 0, /* raw weights / first operand of a host call */
    QW6H_BUF_PACKED,  /* packed weights of a host call */
    QW6H_BUF_X,       /* activations */
    QW6H_BUF_Y,       /* outputs */
    QW6H_BUF_KEY,     /* small scratch (argmax key, routing weights) */
    QW6H_BUF_WS,      /* workspace of the fused MoE / LM-head calls */
    QW6H_BUF_BLOCK,   /* intermediates of the MoE FFN block */
    QW6H_BUF_SAMPLE,  /* per-row histograms of the sampler */
    QW6H_BUF_IO,      /* the two input/output slots of the pipelined host-buffer prefill */
    QW6H_NBUF
};

typedef struct {
    void *p;
    size_t n;
} qw6h_buf_t;

/* Kernel ids of the profiler (names in qw6cu_kernel_name). */
enum {
    QW6H_K_MATVEC = 0,
    QW6H_K_PACK,
    QW6H_K_DEQUANT,
    QW6H_K_ROUTE,
    QW6H_K_ARGMAX,
    QW6H_K_MOE_PLAN,
    QW6H_K_MOE_GATEUP,
    QW6H_K_MOE_DOWN,
    QW6H_K_MOE_COMBINE,
    QW6H_K_LM_HEAD,
    QW6H_K_PF_PLAN,
    QW6H_K_PF_GEMM1,
    QW6H_K_PF_GEMM2,
    QW6H_K_PF_COMBINE,
    QW6H_K_EP,
    QW6H_K_EP_PUBLISH,
    QW6H_K_EP_DISPATCH,
    QW6H_K_EP_WAIT,
    QW6H_K_EP_COMBINE,
    QW6H_K_MOE_BLOCK,
    QW6H_K_SAMPLE,
    QW6H_K_COUNT
};

typedef struct {
    int kid;
    cudaEvent_t a, b;
} qw6h_prof_rec;

struct qw6cu_ctx {
    int device;
    int num_sms;
    cudaStream_t own; /* stream created with the context */
    cudaStream_t st;  /* stream work is enqueued on */
    qw6h_buf_t buf[QW6H_NBUF];
    void *pinned;     /* pinned host staging (unused unless requested) */
    /* per-launch event profiler (qw6cu_profile_begin/end) */
    int prof_on, prof_cap, prof_n;
    qw6h_prof_rec *prof;
    /* copy streams and events of the pipelined host-buffer prefill, created
     * on its first call: ev[0] start; per slot s: ev[1+s] inputs landed,
     * ev[3+s] inputs consumed, ev[5+s] output ready, ev[7+s] output read */
    int io_ready;
    cudaStream_t io_in, io_out;
    cudaEvent_t io_ev[9];
};

void qw6h_set_err(const char *fmt, ...);
int qw6h_rc(int rc, const char *what);
int qw6h_use(qw6cu_ctx *ctx);
void *qw6h_buf(qw6cu_ctx *ctx, int i, size_t bytes);
qw6cu_ctx *qw6h_default_locked(void);
/* Profiler hooks around one launch: rec = qw6h_prof_a(ctx, kid); launch;
 * qw6h_prof_b(ctx, rec).  No-ops unless profiling is on. */
int qw6h_prof_a(qw6cu_ctx *ctx, int kid);
int *qw6h_dev_err(qw6cu_ctx *ctx);
void qw6h_prof_b(qw6cu_ctx *ctx, int rec);
/* Pipelined host-buffer batches (two device slots, the context's copy
 * streams): run(arg, logits, x, out) enqueues one batch's layer on ctx->st
 * with device pointers into the current slot. */
typedef int (*qw6h_hostio_fn)(void *arg, const float *logits, const void *x_bf16, float *out);
int qw6h_hostio_run(qw6cu_ctx *ctx, const char *what, const float *const *logits, const void *const *x_bf16,
                    float *const *out, uint32_t n_batches, size_t lg_bytes, size_t x_bytes, size_t out_bytes,
                    qw6h_hostio_fn run, void *arg);

#endif /* QW6_HOST_INTERNAL_H */
