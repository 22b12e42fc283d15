/* qw6_moe_host.c -- host side of the routed-MoE entry points (C11). */
#define _POSIX_C_SOURCE 200809L

#include <stddef.h>

#include "qw6_cuda.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"

size_t qw6cu_moe_workspace_bytes(uint32_t ntok, uint32_t hidden, uint32_t inter, uint32_t n_experts,
                                 uint32_t top_k) {
    return qw6k_moe_ws_bytes(ntok, hidden, inter, n_experts, top_k);
}

int qw6cu_moe_decode(qw6cu_ctx *ctx, const qw6cu_expert_pack *gate, const qw6cu_expert_pack *up,
                     const qw6cu_expert_pack *down, const float *logits, const float *x, float *out, uint32_t ntok,
                     uint32_t hidden, uint32_t inter, uint32_t n_experts, uint32_t top_k) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!gate || !up || !down || gate->quant != up->quant) {
        qw6h_set_err("qw6cu_moe_decode: gate and up packs must be given and share one quant type");
        return QW6CU_ERR_ARG;
    }
    const size_t need = qw6k_moe_ws_bytes(ntok, hidden, inter, n_experts, top_k);
    void *ws = qw6h_buf(ctx, QW6H_BUF_WS, need);
    if (!ws) return QW6CU_ERR_NOMEM;
    return qw6h_rc(qw6k_moe_decode(gate->quant, gate->base, gate->stride, up->base, up->stride, down->quant,
                                   down->base, down->stride, logits, x, out, ntok, hidden, inter, n_experts, top_k,
                                   ws, need, ctx->st),
                   "moe_decode");
}
