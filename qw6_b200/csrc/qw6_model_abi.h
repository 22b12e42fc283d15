/* qw6_model_abi.h -- the memory layout of qw6's qw6_model_t as qw6.c built
 * with QW6_VULKAN passes it to qw6_vk_pipe_init / qw6_vk_pipe_forward
 * (qw6.h:94-205: qw6_tensor_t, then the model struct with its per-layer
 * tensors).  The drop-in pipeline reads the tensors out of the caller's
 * model through this mirror; the field order and types follow qw6.h so that
 * every offset matches (checked against qw6.h itself by
 * tests/test_abi.py::test_model_layout_matches_qw6).  Only what the pipeline
 * reads is named; nothing here is written. */
#ifndef QW6_MODEL_ABI_H
#define QW6_MODEL_ABI_H

#include <stddef.h>
#include <stdint.h>

#define QW6ABI_LAYERS 40
#define QW6ABI_EXPERTS 256

typedef struct {
    char name[128];
    uint32_t rows, cols;
    uint32_t ne[4];
    uint32_t n_dims;
    int quant;            /* qw6_quant_t */
    void *data;           /* raw GGUF rows in host memory */
    size_t data_size;
    uint64_t file_offset;
    size_t vk_offset;     /* present when qw6 is built with QW6_VULKAN */
} qw6abi_tensor;

typedef struct {
    int type;
    qw6abi_tensor norm, post_norm;
    qw6abi_tensor attn_q, attn_k, attn_v, attn_o, attn_q_norm, attn_k_norm, attn_gate;
    qw6abi_tensor conv1d, dn_key, dn_value, dn_query, dn_out, dn_gate, dn_norm, dn_alpha, dn_beta, dn_dt, dn_a;
    qw6abi_tensor moe_router, shared_router;
    qw6abi_tensor expert_gate[QW6ABI_EXPERTS], expert_up[QW6ABI_EXPERTS], expert_down[QW6ABI_EXPERTS];
    qw6abi_tensor shared_gate, shared_up, shared_down;
} qw6abi_layer;

typedef struct {
    qw6abi_tensor tok_embeddings, output, output_norm;
    qw6abi_layer layers[QW6ABI_LAYERS];
    struct {
        qw6abi_tensor norm, embed;
    } mtp;
    float *deltanet_state[QW6ABI_LAYERS];
    float *k_cache[QW6ABI_LAYERS];
    float *v_cache[QW6ABI_LAYERS];
    uint32_t max_context;
    uint32_t current_context;
} qw6abi_model;

#endif /* QW6_MODEL_ABI_H */
