/* qw6_selftest.c -- qw6_vk_selftest(): closed-form known-answer tests of
 * the GPU entry points, the same patterns qw6's own Vulkan self-test uses
 * (qw6_vk.c:1609-1954), run through the drop-in host API.
 *
 * Returns 0 when every check passes, 1 otherwise (the reference's
 * convention, qw6.c:3540).  Expected values are computed in closed form
 * from the synthetic block contents.
 */
#define _POSIX_C_SOURCE 200809L

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "qw6_vk.h"

static void put16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xffu);
    p[1] = (uint8_t)(v >> 8);
}

static int check(const char *what, const float *got, const double *want, int n, double tol) {
    for (int i = 0; i < n; i++)
        if (!(fabs((double)got[i] - want[i]) <= tol)) {
            fprintf(stderr, "qw6cuda selftest: %s[%d] = %.6f, expected %.6f\n", what, i, got[i], want[i]);
            return 1;
        }
    return 0;
}

/* Q4_K: d=1, dmin=0, all 8 sub-block scales 1, q = (3r + 5c + 7) & 15
 * (qw6_vk.c:1609-1649). */
static int kat_q4k(void) {
    uint8_t w[3 * 144];
    float x[256], y[3];
    double want[3] = {0, 0, 0};
    memset(w, 0, sizeof w);
    for (int c = 0; c < 256; c++) x[c] = sinf((float)c * 0.031f);
    for (int r = 0; r < 3; r++) {
        uint8_t *b = w + 144 * r;
        put16(b, 0x3c00);
        for (int j = 0; j < 4; j++) b[4 + j] = 1;  /* scales 0..3 */
        for (int j = 8; j < 12; j++) b[4 + j] = 1; /* low nibbles of scales 4..7 */
        for (int c = 0; c < 256; c++) {
            const int chunk = c / 64, hi = (c / 32) & 1, l = c % 32;
            const uint8_t q = (uint8_t)((r * 3 + c * 5 + 7) & 15);
            uint8_t *p = b + 16 + 32 * chunk + l;
            *p = hi ? (uint8_t)((*p & 0x0f) | (q << 4)) : (uint8_t)((*p & 0xf0) | q);
            want[r] += (double)q * x[c];
        }
    }
    if (qw6_vk_matmul_q4k_host(w, x, y, 3, 256)) return 1;
    return check("matmul_q4k", y, want, 3, 1e-2);
}

/* Q5_K: as Q4_K with 5-bit q = (7r + 3c + 5) & 31 (qw6_vk.c:1651-1704). */
static int kat_q5k(void) {
    uint8_t w[3 * 176];
    float x[256], y[3];
    double want[3] = {0, 0, 0};
    memset(w, 0, sizeof w);
    for (int c = 0; c < 256; c++) x[c] = cosf((float)c * 0.027f);
    for (int r = 0; r < 3; r++) {
        uint8_t *b = w + 176 * r;
        put16(b, 0x3c00);
        for (int j = 0; j < 4; j++) b[4 + j] = 1;
        for (int j = 8; j < 12; j++) b[4 + j] = 1;
        for (int c = 0; c < 256; c++) {
            const int chunk = c / 64, hi = (c / 32) & 1, l = c % 32;
            const uint8_t q = (uint8_t)((r * 7 + c * 3 + 5) & 31);
            uint8_t *p = b + 48 + 32 * chunk + l;
            *p = hi ? (uint8_t)((*p & 0x0f) | ((q & 15) << 4)) : (uint8_t)((*p & 0xf0) | (q & 15));
            if (q & 16) b[16 + l] |= (uint8_t)(1u << (2 * chunk + hi));
            want[r] += (double)q * x[c];
        }
    }
    if (qw6_vk_matmul_q5k_host(w, x, y, 3, 256)) return 1;
    return check("matmul_q5k", y, want, 3, 1e-2);
}

/* Q6_K: d=1, all scales 1, q = ((11r + 7c + 9) & 63) - 32 (qw6_vk.c:1706-1742). */
static int kat_q6k(void) {
    uint8_t w[3 * 210];
    float x[256], y[3];
    double want[3] = {0, 0, 0};
    memset(w, 0, sizeof w);
    for (int c = 0; c < 256; c++) x[c] = sinf((float)c * 0.019f) + 0.2f * cosf((float)c * 0.013f);
    for (int r = 0; r < 3; r++) {
        uint8_t *b = w + 210 * r;
        put16(b + 208, 0x3c00);
        for (int i = 0; i < 16; i++) b[192 + i] = 1;
        for (int c = 0; c < 256; c++) {
            const int half = c / 128, in = c % 128, l = in % 32, quad = in / 32;
            const int qv = ((r * 11 + c * 7 + 9) & 63) - 32;
            const unsigned u = (unsigned)(qv + 32);
            uint8_t *ql = b + 64 * half + l + ((quad & 1) ? 32 : 0);
            *ql = quad < 2 ? (uint8_t)((*ql & 0xf0) | (u & 15)) : (uint8_t)((*ql & 0x0f) | ((u & 15) << 4));
            b[128 + 32 * half + l] |= (uint8_t)(((u >> 4) & 3) << (2 * quad));
            want[r] += (double)qv * x[c];
        }
    }
    if (qw6_vk_matmul_q6k_host(w, x, y, 3, 256)) return 1;
    return check("matmul_q6k", y, want, 3, 1e-2);
}

/* IQ2_XXS: all-zero qs (grid entry 0 = all 8s, no signs, scale nibble 0)
 * so every weight is d * 0.125 * 8 = d (qw6_vk.c:1744-1787). */
static int kat_iq2xxs(void) {
    uint8_t w[3 * 66];
    float x[256], y[3];
    double want[3] = {0, 0, 0};
    const uint16_t dh[3] = {0x3c00, 0x3e00, 0x4000};
    const double dv[3] = {1.0, 1.5, 2.0};
    memset(w, 0, sizeof w);
    for (int c = 0; c < 256; c++) x[c] = sinf((float)c * 0.029f) + 0.15f * cosf((float)c * 0.017f);
    for (int r = 0; r < 3; r++) {
        put16(w + 66 * r, dh[r]);
        for (int c = 0; c < 256; c++) want[r] += dv[r] * x[c];
    }
    if (qw6_vk_matmul_iq2xxs_host(w, x, y, 3, 256)) return 1;
    return check("matmul_iq2xxs", y, want, 3, 2e-2);
}

static int kat_silu_argmax_route_gather(void) {
    int fail = 0;
    enum { SN = 513, AN = 4097, GN = 1029, EN = 256, GD = 257 };
    static float g[SN], u[SN], o[SN], ax[AN], gx[GN], lg[EN], ge[8 * GD], gs[GD], go[GD];
    double want[GD];
    for (int i = 0; i < SN; i++) {
        g[i] = ((float)(i % 31) - 15.0f) * 0.125f;
        u[i] = cosf((float)i * 0.031f);
    }
    if (qw6_vk_silu_mul_host(g, u, o, SN)) return 1;
    for (int i = 0; i < SN && !fail; i++) {
        const double e = ((double)g[i] / (1.0 + exp(-(double)g[i]))) * u[i];
        if (fabs(o[i] - e) > 2e-5) {
            fprintf(stderr, "qw6cuda selftest: silu_mul[%d] = %.6f, expected %.6f\n", i, o[i], e);
            fail = 1;
        }
    }
    for (int i = 0; i < AN; i++) ax[i] = sinf((float)i * 0.019f) - (float)(i % 7) * 0.01f;
    ax[3079] = 42.0f;
    uint32_t idx = 0;
    float val = 0;
    if (qw6_vk_argmax_host(ax, AN, &idx, &val) || idx != 3079 || val != 42.0f) {
        fprintf(stderr, "qw6cuda selftest: argmax got %u (%.3f), expected 3079\n", idx, val);
        fail = 1;
    }
    for (int i = 0; i < GN; i++) gx[i] = cosf((float)i * 0.023f) - 0.001f * (float)i;
    gx[877] = 11.0f;
    uint32_t tok = 0;
    if (qw6_vk_sampling_greedy_host(gx, GN, &tok) || tok != 877) {
        fprintf(stderr, "qw6cuda selftest: sampling_greedy got %u, expected 877\n", tok);
        fail = 1;
    }
    for (int i = 0; i < EN; i++) lg[i] = sinf((float)i * 0.17f) + cosf((float)i * 0.031f);
    lg[7] = 5.0f;
    lg[149] = 4.5f;
    uint32_t ri[8];
    float rw[8];
    if (qw6_vk_moe_route_host(lg, ri, rw, EN, 8)) return 1;
    double ws = 0;
    for (int k = 0; k < 8; k++) ws += rw[k];
    if (ri[0] != 7 || ri[1] != 149 || fabs(ws - 1.0) > 1e-5) {
        fprintf(stderr, "qw6cuda selftest: moe_route got %u,%u sum %.6f\n", ri[0], ri[1], ws);
        fail = 1;
    }
    for (int k = 1; k < 8; k++)
        if (rw[k] > rw[k - 1] || lg[ri[k]] > lg[ri[k - 1]]) fail = 1;
    float gw[8];
    double wsum = 0;
    for (int e = 0; e < 8; e++) {
        gw[e] = 0.1f + 0.03f * (float)e;
        wsum += gw[e];
        for (int i = 0; i < GD; i++) ge[e * GD + i] = sinf((float)(e * 17 + i) * 0.021f);
    }
    for (int e = 0; e < 8; e++) gw[e] = (float)(gw[e] / wsum);
    for (int i = 0; i < GD; i++) {
        gs[i] = cosf((float)i * 0.019f);
        want[i] = 0.25 * gs[i];
        for (int e = 0; e < 8; e++) want[i] += (double)gw[e] * ge[e * GD + i];
    }
    if (qw6_vk_moe_gather_host(ge, gw, gs, 0.25f, go, GD, 8)) return 1;
    fail |= check("moe_gather", go, want, GD, 2e-5);
    return fail;
}

int qw6_vk_selftest(void) {
    int fail = 0;
    fail |= kat_q4k();
    fail |= kat_q5k();
    fail |= kat_q6k();
    fail |= kat_iq2xxs();
    fail |= kat_silu_argmax_route_gather();
    fprintf(stderr, "qw6cuda selftest: %s\n", fail ? "FAILED" : "passed");
    return fail ? 1 : 0;
}
