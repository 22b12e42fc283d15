/* qw6_gguf.c -- GGUF file reading and device upload (host C11).
 *
 * qw6 reads its model from one GGUF file (qw6_gguf_parse, qw6.c:871-1060;
 * qw6_gguf_read_file, qw6.c:1097-1240): a little-endian header (magic
 * "GGUF", version 3, tensor and metadata counts), metadata key/value pairs,
 * a tensor table (name, dims, ggml type, offset), then the tensor data from
 * an aligned offset.  Expert packs are 3-D tensors [cols, rows, n_experts]
 * whose expert e starts at e * rows * row_bytes (bind_expert_pack,
 * qw6.c:542-597).  This file parses that layout itself (the file is
 * memory-mapped, nothing is read twice), maps the ggml types to qw6's quant
 * codes as qw6_gguf_to_quant does (qw6.c:1079-1094), and uploads tensors to
 * the GPU: block formats into the packed tile layout (qw6cu_pack), expert
 * packs with a fixed packed stride per expert, and the MoE tensors of every
 * layer into one device allocation described by a table the kernels can read
 * (qw6cu_gguf_upload_moe).
 */
#define _POSIX_C_SOURCE 200809L

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_runtime_api.h>

#include "qw6_cuda.h"
#include "qw6_formats.h"
#include "qw6_host_internal.h"
#include "qw6_launch.h"

#define GGUF_MAGIC 0x46554747u /* "GGUF" */
#define GGUF_MAX_DIMS 4

typedef struct {
    char *name;
    uint32_t n_dims;
    uint64_t dims[GGUF_MAX_DIMS];
    uint32_t ggml_type;
    uint64_t offset; /* from the data section */
} gguf_tensor;

struct qw6cu_gguf {
    int fd;
    const uint8_t *map;
    size_t size;
    uint32_t version, alignment;
    uint64_t n_tensors, n_kv, data_offset;
    gguf_tensor *t;
};

/* ---- bounded little-endian reader over the mapping ---- */
typedef struct {
    const uint8_t *p, *end;
    int bad;
} rd_t;

static int rd_take(rd_t *r, void *dst, size_t n) {
    if (r->bad || (size_t)(r->end - r->p) < n) {
        r->bad = 1;
        return -1;
    }
    if (dst) memcpy(dst, r->p, n);
    r->p += n;
    return 0;
}
static uint32_t rd_u32(rd_t *r) {
    uint32_t v = 0;
    rd_take(r, &v, 4);
    return v;
}
static uint64_t rd_u64(rd_t *r) {
    uint64_t v = 0;
    rd_take(r, &v, 8);
    return v;
}
/* string: u64 length + bytes (not NUL-terminated); *out malloc'd if given */
static int rd_str(rd_t *r, char **out) {
    const uint64_t n = rd_u64(r);
    if (r->bad || n > (uint64_t)(r->end - r->p) || n > (1u << 20)) {
        r->bad = 1;
        return -1;
    }
    if (out) {
        *out = malloc((size_t)n + 1);
        if (!*out) {
            r->bad = 1;
            return -1;
        }
        memcpy(*out, r->p, (size_t)n);
        (*out)[n] = 0;
    }
    r->p += n;
    return 0;
}

/* bytes of one scalar of a GGUF metadata type (0: string/array/unknown) */
static size_t kv_scalar_bytes(uint32_t type) {
    switch (type) {
    case 0: case 1: case 7: return 1;  /* u8, i8, bool */
    case 2: case 3: return 2;          /* u16, i16 */
    case 4: case 5: case 6: return 4;  /* u32, i32, f32 */
    case 10: case 11: case 12: return 8; /* u64, i64, f64 */
    default: return 0;
    }
}

static int skip_value(rd_t *r, uint32_t type, int depth) {
    if (type == 8) return rd_str(r, NULL);
    if (type == 9) {
        if (depth > 2) return -1;
        const uint32_t et = rd_u32(r);
        const uint64_t n = rd_u64(r);
        if (r->bad) return -1;
        const size_t sb = kv_scalar_bytes(et);
        if (sb) return (n > (uint64_t)(r->end - r->p) / sb) ? (r->bad = 1, -1) : rd_take(r, NULL, (size_t)n * sb);
        for (uint64_t i = 0; i < n && !r->bad; i++) skip_value(r, et, depth + 1);
        return r->bad ? -1 : 0;
    }
    const size_t sb = kv_scalar_bytes(type);
    if (!sb) {
        r->bad = 1;
        return -1;
    }
    return rd_take(r, NULL, sb);
}

/* ggml type -> qw6_quant_t (qw6.c:1079-1094); -1 if qw6 has no such type */
static int ggml_to_quant(uint32_t t) {
    switch (t) {
    case 0: return QW6F_FP32;
    case 1: return QW6F_FP16;
    case 30: return QW6F_BF16;
    case 8: return QW6F_Q8_0;
    case 12: return QW6F_Q4_K_M;
    case 13: return QW6F_Q5_K;
    case 14: return QW6F_Q6_K;
    case 16: return QW6F_IQ2_XXS;
    case 21: return QW6F_IQ3_S;
    case 22: return QW6F_IQ2_S;
    default: return -1;
    }
}

/* bytes of one row of `cols` elements (0: unknown type or ragged blocks) */
static size_t row_bytes_of(int quant, uint64_t cols) {
    if (quant == QW6F_Q8_0) return cols % 32 ? 0 : (size_t)(cols / 32) * 34;
    return qw6_row_bytes((uint32_t)quant, (uint32_t)cols);
}

static uint64_t tensor_rows(const gguf_tensor *t) {
    uint64_t r = 1;
    for (uint32_t d = 1; d < t->n_dims; d++) r *= t->dims[d];
    return r;
}

void qw6cu_gguf_close(qw6cu_gguf *g) {
    if (!g) return;
    if (g->t)
        for (uint64_t i = 0; i < g->n_tensors; i++) free(g->t[i].name);
    free(g->t);
    if (g->map) munmap((void *)g->map, g->size);
    if (g->fd >= 0) close(g->fd);
    free(g);
}

int qw6cu_gguf_open(const char *path, qw6cu_gguf **out) {
    if (!path || !out) {
        qw6h_set_err("qw6cu_gguf_open: invalid arguments");
        return QW6CU_ERR_ARG;
    }
    *out = NULL;
    qw6cu_gguf *g = calloc(1, sizeof *g);
    if (!g) return QW6CU_ERR_NOMEM;
    g->fd = open(path, O_RDONLY);
    struct stat st;
    if (g->fd < 0 || fstat(g->fd, &st) != 0 || st.st_size < 24) {
        qw6h_set_err("qw6cu_gguf_open: cannot open or stat %s", path);
        qw6cu_gguf_close(g);
        return QW6CU_ERR_ARG;
    }
    g->size = (size_t)st.st_size;
    g->map = mmap(NULL, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (g->map == MAP_FAILED) {
        g->map = NULL;
        qw6h_set_err("qw6cu_gguf_open: mmap failed");
        qw6cu_gguf_close(g);
        return QW6CU_ERR_ARG;
    }
    rd_t r = {g->map, g->map + g->size, 0};
    const uint32_t magic = rd_u32(&r);
    g->version = rd_u32(&r);
    g->n_tensors = rd_u64(&r);
    g->n_kv = rd_u64(&r);
    g->alignment = 32; /* the GGUF default */
    if (magic != GGUF_MAGIC || g->version != 3 || g->n_tensors > (1u << 20) || g->n_kv > (1u << 20)) {
        qw6h_set_err("qw6cu_gguf_open: not a GGUF v3 file (magic 0x%08x, version %u)", magic, g->version);
        qw6cu_gguf_close(g);
        return QW6CU_ERR_ARG;
    }
    for (uint64_t i = 0; i < g->n_kv && !r.bad; i++) {
        char *key = NULL;
        if (rd_str(&r, &key)) break;
        const uint32_t type = rd_u32(&r);
        if (!r.bad && type == 4 && strcmp(key, "general.alignment") == 0) {
            g->alignment = rd_u32(&r);
        } else {
            skip_value(&r, type, 0);
        }
        free(key);
    }
    g->t = calloc(g->n_tensors ? g->n_tensors : 1, sizeof *g->t);
    if (!g->t) {
        qw6cu_gguf_close(g);
        return QW6CU_ERR_NOMEM;
    }
    for (uint64_t i = 0; i < g->n_tensors && !r.bad; i++) {
        gguf_tensor *t = &g->t[i];
        if (rd_str(&r, &t->name)) break;
        t->n_dims = rd_u32(&r);
        if (t->n_dims == 0 || t->n_dims > GGUF_MAX_DIMS) {
            r.bad = 1;
            break;
        }
        for (uint32_t d = 0; d < t->n_dims; d++) t->dims[d] = rd_u64(&r);
        t->ggml_type = rd_u32(&r);
        t->offset = rd_u64(&r);
    }
    if (r.bad || g->alignment == 0 || (g->alignment & (g->alignment - 1))) {
        qw6h_set_err("qw6cu_gguf_open: truncated or malformed header / tensor table");
        qw6cu_gguf_close(g);
        return QW6CU_ERR_ARG;
    }
    const uint64_t pos = (uint64_t)(r.p - g->map);
    g->data_offset = (pos + g->alignment - 1) / g->alignment * g->alignment;
    /* every tensor of a known type must lie inside the file */
    for (uint64_t i = 0; i < g->n_tensors; i++) {
        const gguf_tensor *t = &g->t[i];
        const int q = ggml_to_quant(t->ggml_type);
        if (q < 0) continue;
        const size_t rb = row_bytes_of(q, t->dims[0]);
        const uint64_t bytes = (uint64_t)rb * tensor_rows(t);
        if (!rb || g->data_offset + t->offset + bytes > g->size || t->offset % g->alignment) {
            qw6h_set_err("qw6cu_gguf_open: tensor %s does not fit the file", t->name);
            qw6cu_gguf_close(g);
            return QW6CU_ERR_ARG;
        }
    }
    *out = g;
    return 0;
}

uint32_t qw6cu_gguf_tensor_count(const qw6cu_gguf *g) { return g ? (uint32_t)g->n_tensors : 0; }

int qw6cu_gguf_find(const qw6cu_gguf *g, const char *name) {
    if (!g || !name) return -1;
    for (uint64_t i = 0; i < g->n_tensors; i++)
        if (strcmp(g->t[i].name, name) == 0) return (int)i;
    return -1;
}

int qw6cu_gguf_tensor_info(const qw6cu_gguf *g, uint32_t i, qw6cu_gguf_tensor *info) {
    if (!g || !info || i >= g->n_tensors) return QW6CU_ERR_ARG;
    const gguf_tensor *t = &g->t[i];
    memset(info, 0, sizeof *info);
    info->name = t->name;
    info->n_dims = t->n_dims;
    for (uint32_t d = 0; d < t->n_dims; d++) info->dims[d] = t->dims[d];
    info->ggml_type = t->ggml_type;
    info->quant = ggml_to_quant(t->ggml_type);
    info->file_offset = g->data_offset + t->offset;
    info->bytes = info->quant < 0 ? 0 : (uint64_t)row_bytes_of(info->quant, t->dims[0]) * tensor_rows(t);
    info->data = g->map + info->file_offset;
    return 0;
}

/* device bytes a 2-D matrix of quant q takes when uploaded */
static size_t up_bytes(int q, uint32_t rows, uint32_t cols) {
    if (q == QW6F_FP32) return (size_t)rows * cols * 4;
    return qw6k_packed_bytes((uint32_t)q, rows, cols);
}

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

/* copy `count` raw matrices of one tensor to the device and pack them at
 * dst + i * dst_stride (FP32 rows are copied as they are) */
static int upload_mats(qw6cu_ctx *ctx, int q, const uint8_t *src, uint32_t rows, uint32_t cols, uint32_t count,
                       void *dst, size_t dst_stride) {
    const size_t rb = row_bytes_of(q, cols) * rows, total = rb * count;
    if (q == QW6F_FP32) {
        cudaError_t e = cudaMemcpy2DAsync(dst, dst_stride, src, rb, rb, count, cudaMemcpyHostToDevice, ctx->st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->st);
        return e == cudaSuccess ? 0 : QW6CU_ERR_CUDA;
    }
    void *raw = qw6h_buf(ctx, QW6H_BUF_RAW, total);
    if (!raw) return QW6CU_ERR_NOMEM;
    cudaError_t e = cudaMemcpyAsync(raw, src, total, cudaMemcpyHostToDevice, ctx->st);
    if (e != cudaSuccess) return QW6CU_ERR_CUDA;
    int rc = qw6h_rc(qw6k_pack((uint32_t)q, raw, dst, rows, cols, count, rb, dst_stride, ctx->st), "gguf upload");
    if (!rc && cudaStreamSynchronize(ctx->st) != cudaSuccess) rc = QW6CU_ERR_CUDA;
    return rc;
}

size_t qw6cu_gguf_upload_bytes(const qw6cu_gguf *g, uint32_t i) {
    if (!g || i >= g->n_tensors) return 0;
    const gguf_tensor *t = &g->t[i];
    const int q = ggml_to_quant(t->ggml_type);
    if (q < 0 || t->n_dims > 3 || t->dims[0] > 0xffffffffull || t->dims[1] > 0xffffffffull) return 0;
    const uint32_t cols = (uint32_t)t->dims[0], rows = t->n_dims > 1 ? (uint32_t)t->dims[1] : 1;
    const uint64_t count = t->n_dims > 2 ? t->dims[2] : 1;
    const size_t one = up_bytes(q, rows, cols);
    return one ? (count > 1 ? al256(one) * count : one) : 0;
}

int qw6cu_gguf_upload(qw6cu_ctx *ctx, const qw6cu_gguf *g, uint32_t i, void *dst, size_t dst_bytes,
                      qw6cu_expert_pack *out) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    const size_t need = qw6cu_gguf_upload_bytes(g, i);
    if (!need || !dst || dst_bytes < need || !out || ((uintptr_t)dst & 255u)) {
        qw6h_set_err("qw6cu_gguf_upload: tensor %u not uploadable (unsupported type or shape) or too small/unaligned "
                     "destination (%zu bytes needed, 256-byte aligned)", i, need);
        return QW6CU_ERR_ARG;
    }
    const gguf_tensor *t = &g->t[i];
    const int q = ggml_to_quant(t->ggml_type);
    const uint32_t cols = (uint32_t)t->dims[0], rows = t->n_dims > 1 ? (uint32_t)t->dims[1] : 1;
    const uint32_t count = t->n_dims > 2 ? (uint32_t)t->dims[2] : 1;
    const size_t stride = count > 1 ? al256(up_bytes(q, rows, cols)) : up_bytes(q, rows, cols);
    rc = upload_mats(ctx, q, g->map + g->data_offset + t->offset, rows, cols, count, dst, stride);
    if (rc) return rc;
    out->quant = (uint32_t)q;
    out->base = dst;
    out->stride = stride;
    return 0;
}

int qw6cu_gguf_upload_moe(qw6cu_ctx *ctx, const qw6cu_gguf *g, uint32_t n_layers, qw6cu_moe_table *tab) {
    int rc = qw6h_use(ctx);
    if (rc) return rc;
    if (!g || !tab || !n_layers || n_layers > 4096) return QW6CU_ERR_ARG;
    memset(tab, 0, sizeof *tab);
    static const char *kind[3] = {"ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"};
    uint32_t *idx = calloc((size_t)n_layers * 3, sizeof *idx);
    size_t *off = calloc((size_t)n_layers * 3, sizeof *off);
    qw6cu_expert_pack *packs = calloc((size_t)n_layers * 3, sizeof *packs);
    if (!idx || !off || !packs) {
        free(idx);
        free(off);
        free(packs);
        return QW6CU_ERR_NOMEM;
    }
    size_t total = 0;
    for (uint32_t l = 0; l < n_layers && !rc; l++)
        for (int k = 0; k < 3 && !rc; k++) {
            char name[96];
            snprintf(name, sizeof name, "blk.%u.%s.weight", l, kind[k]);
            const int i = qw6cu_gguf_find(g, name);
            const size_t b = i < 0 ? 0 : qw6cu_gguf_upload_bytes(g, (uint32_t)i);
            if (i < 0 || !b || g->t[i].n_dims != 3) {
                qw6h_set_err("qw6cu_gguf_upload_moe: %s missing or not a 3-D expert pack of a supported type", name);
                rc = QW6CU_ERR_ARG;
                break;
            }
            idx[l * 3 + k] = (uint32_t)i;
            off[l * 3 + k] = total;
            total += al256(b);
        }
    void *dev = NULL, *tdev = NULL;
    if (!rc && cudaMalloc(&dev, total) != cudaSuccess) rc = QW6CU_ERR_NOMEM;
    for (uint32_t j = 0; j < n_layers * 3 && !rc; j++)
        rc = qw6cu_gguf_upload(ctx, g, idx[j], (uint8_t *)dev + off[j], total - off[j], &packs[j]);
    if (!rc && cudaMalloc(&tdev, sizeof *packs * n_layers * 3) != cudaSuccess) rc = QW6CU_ERR_NOMEM;
    if (!rc && (cudaMemcpyAsync(tdev, packs, sizeof *packs * n_layers * 3, cudaMemcpyHostToDevice, ctx->st) !=
                    cudaSuccess ||
                cudaStreamSynchronize(ctx->st) != cudaSuccess))
        rc = QW6CU_ERR_CUDA;
    if (rc) {
        cudaFree(dev);
        cudaFree(tdev);
        free(packs);
    } else {
        tab->n_layers = n_layers;
        tab->packs = packs;
        tab->packs_dev = tdev;
        tab->weights = dev;
        tab->bytes = total;
    }
    free(idx);
    free(off);
    return rc;
}

void qw6cu_moe_table_free(qw6cu_moe_table *tab) {
    if (!tab) return;
    cudaFree(tab->weights);
    cudaFree(tab->packs_dev);
    free(tab->packs);
    memset(tab, 0, sizeof *tab);
}
