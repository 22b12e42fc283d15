/* qw6_formats.h -- GGUF super-block formats handled by libqw6cuda.
 *
 * Shared by the C host code, the CUDA kernels and the test oracle.  The
 * quant codes are the values of qw6's qw6_quant_t (qw6.h:77-92) so that a
 * caller holding a qw6_tensor_t can pass t->quant unchanged.
 *
 * Byte layouts (QK_K = 256 weights per super-block), as declared in
 * qw6.c:1406-1446:
 *   Q4_K    144 B  {u16 d, u16 dmin, u8 scales[12], u8 qs[128]}
 *   Q5_K    176 B  {u16 d, u16 dmin, u8 scales[12], u8 qh[32], u8 qs[128]}
 *   Q6_K    210 B  {u8 ql[128], u8 qh[64], i8 scales[16], u16 d}   (d LAST)
 *   IQ2_XXS  66 B  {u16 d, u16 qs[32]}
 *   IQ2_S    82 B  {u16 d, u8 qs[64], u8 qh[8], u8 scales[8]}
 *   IQ3_S   110 B  {u16 d, u8 qs[64], u8 qh[8], u8 signs[32], u8 scales[4]}
 * A matrix is row-major: row r starts at r * (cols/256) * block_bytes
 * (qw6.c:1711-1712).  All multi-byte fields are little-endian.
 */
#ifndef QW6_FORMATS_H
#define QW6_FORMATS_H

#include <stdint.h>
#include <stddef.h>

#define QW6_QK 256u

#ifdef __CUDACC__
#define QW6_HD __host__ __device__
#else
#define QW6_HD
#endif

enum {
    QW6F_FP32 = 0,
    QW6F_FP16 = 1,
    QW6F_BF16 = 2,
    QW6F_Q8_0 = 3,
    QW6F_Q4_K_M = 4,
    QW6F_Q4_K_S = 5,
    QW6F_Q5_K = 6,
    QW6F_Q6_K = 7,
    QW6F_Q3_K_M = 8,
    QW6F_IQ3_S = 9,
    QW6F_IQ3_XXS = 10,
    QW6F_IQ2_S = 11,
    QW6F_IQ2_M = 12,
    QW6F_IQ2_XXS = 13
};

#define QW6_BLOCK_Q4_K 144u
#define QW6_BLOCK_Q5_K 176u
#define QW6_BLOCK_Q6_K 210u
#define QW6_BLOCK_IQ2_XXS 66u
#define QW6_BLOCK_IQ2_S 82u
#define QW6_BLOCK_IQ3_S 110u

/* Super-block byte size of a 256-weight block format, 0 for anything the
 * block kernels do not handle.  Q4_K_M and Q4_K_S share the Q4_K block
 * (qw6.c:1693-1694).  IQ2_M and Q8_0 return 0: qw6's CPU dequantizer
 * rejects both (qw6.c:1706-1707). */
static inline QW6_HD uint32_t qw6_block_bytes(uint32_t quant) {
    switch (quant) {
    case QW6F_Q4_K_M:
    case QW6F_Q4_K_S: return QW6_BLOCK_Q4_K;
    case QW6F_Q5_K: return QW6_BLOCK_Q5_K;
    case QW6F_Q6_K: return QW6_BLOCK_Q6_K;
    case QW6F_IQ2_XXS: return QW6_BLOCK_IQ2_XXS;
    case QW6F_IQ2_S: return QW6_BLOCK_IQ2_S;
    case QW6F_IQ3_S: return QW6_BLOCK_IQ3_S;
    default: return 0;
    }
}

/* Bytes of one matrix row: 256-blocks for the K/IQ formats, elements for
 * the plain float formats, 0 when the format/shape is not representable. */
static inline QW6_HD size_t qw6_row_bytes(uint32_t quant, uint32_t cols) {
    uint32_t bb = qw6_block_bytes(quant);
    if (bb) return (cols % QW6_QK) ? 0 : (size_t)(cols / QW6_QK) * bb;
    if (quant == QW6F_FP32) return (size_t)cols * 4u;
    if (quant == QW6F_FP16 || quant == QW6F_BF16) return (size_t)cols * 2u;
    return 0;
}

/* IQ2 sign table entry i: 7 explicit sign bits plus bit 7 chosen so the
 * byte has even parity -- the closed form of qw6's ksigns_iq2xs
 * (qw6_iq_tables.h:11-20).  Bit j of the result negates weight j. */
static inline QW6_HD uint8_t qw6_ksigns(uint32_t i) {
    uint32_t p = i & 127u;
    p ^= p >> 4;
    p ^= p >> 2;
    p ^= p >> 1;
    return (uint8_t)((i & 127u) | ((p & 1u) << 7));
}

#endif /* QW6_FORMATS_H */
