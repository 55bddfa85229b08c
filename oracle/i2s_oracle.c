/*
 * i2s_oracle.c -- scalar CPU restatement of the ternary i2_s mul_mat path (TEST INFRASTRUCTURE).
 *
 * Only tests/, the smoke check and bench.py's CPU-baseline leg use this file; the product library
 * never links it. The algorithm statement, its provenance and the byte layout are in i2s_oracle.h.
 * Build flags must keep IEEE fp32 semantics: -fno-fast-math -ffp-contract=off (no FMA contraction).
 */
#include "i2s_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QK 128 /* weights per interleave block (x86 QK_I2_S of the BitNet fork) */

static int64_t roundup128(int64_t k) { return (k + QK - 1) / QK * QK; }

size_t orc_i2s_nbytes(int64_t nrow, int64_t n_per_row) {
    return (size_t)(nrow * n_per_row / 4) + 32;
}

size_t orc_i2s_r_nbytes(int64_t nrow, int64_t n_per_row) {
    return (size_t)(nrow * roundup128(n_per_row) / 4) + 32;
}

/* Position of flat weight g in the flattened layout. */
static inline void i2s_pos(int64_t g, int64_t *byte, int *shift) {
    int64_t b = g / QK;
    int j = (int)(g % QK);
    *byte = 32 * b + (j % 32);
    *shift = 6 - 2 * (j / 32);
}

static void put_scale(uint8_t *dst, size_t code_bytes, float scale) {
    memset(dst + code_bytes, 0, 32);
    memcpy(dst + code_bytes, &scale, sizeof(float));
}

/* quantize_i2_s restated: scale = max|w| over the tensor, code from the sign, |w| < 1e-6 -> 0. */
size_t orc_i2s_quantize(const float *src, uint8_t *dst, int64_t nrow, int64_t n_per_row) {
    const int64_t n = nrow * n_per_row;
    if (n % QK != 0) return 0; /* the flattened interleave needs whole 128-weight blocks */
    double amax = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double a = fabs((double)src[i]);
        if (a > amax) amax = a;
    }
    memset(dst, 0, (size_t)(n / 4));
    for (int64_t g = 0; g < n; ++g) {
        int code;
        if (fabs((double)src[g]) < 1e-6) code = 1;
        else code = ((double)src[g] * amax > 0) ? 2 : 0;
        int64_t byte; int shift;
        i2s_pos(g, &byte, &shift);
        dst[byte] |= (uint8_t)(code << shift);
    }
    put_scale(dst, (size_t)(n / 4), (float)amax);
    return orc_i2s_nbytes(nrow, n_per_row);
}

size_t orc_i2s_pack_ternary(const int8_t *t, float scale, uint8_t *dst, int64_t nrow, int64_t n_per_row) {
    const int64_t n = nrow * n_per_row;
    if (n % QK != 0) return 0;
    memset(dst, 0, (size_t)(n / 4));
    for (int64_t g = 0; g < n; ++g) {
        int code = (int)t[g] + 1;
        int64_t byte; int shift;
        i2s_pos(g, &byte, &shift);
        dst[byte] |= (uint8_t)((code & 3) << shift);
    }
    put_scale(dst, (size_t)(n / 4), scale);
    return orc_i2s_nbytes(nrow, n_per_row);
}

float orc_i2s_unpack_ternary(const uint8_t *src, int8_t *t, int64_t nrow, int64_t n_per_row) {
    const int64_t n = nrow * n_per_row;
    for (int64_t g = 0; g < n; ++g) {
        int64_t byte; int shift;
        i2s_pos(g, &byte, &shift);
        t[g] = (int8_t)(((src[byte] >> shift) & 3) - 1);
    }
    float scale;
    memcpy(&scale, src + n / 4, sizeof(float));
    return scale;
}

void orc_i2s_dequantize(const uint8_t *src, float *dst, int64_t nrow, int64_t n_per_row) {
    const int64_t n = nrow * n_per_row;
    int8_t *t = (int8_t *)malloc((size_t)n);
    float scale = orc_i2s_unpack_ternary(src, t, nrow, n_per_row);
    for (int64_t g = 0; g < n; ++g) dst[g] = (float)t[g] * scale;
    free(t);
}

size_t orc_i2s_to_rowpadded(const uint8_t *src, uint8_t *dst, int64_t nrow, int64_t n_per_row) {
    const int64_t K = n_per_row, Kp = roundup128(K);
    const size_t code_bytes = (size_t)(nrow * Kp / 4);
    memset(dst, 0x55, code_bytes); /* code 1 in all four slots = zero weight */
    for (int64_t r = 0; r < nrow; ++r) {
        for (int64_t k = 0; k < K; ++k) {
            int64_t sb; int ss;
            i2s_pos(r * K + k, &sb, &ss);
            int code = (src[sb] >> ss) & 3;
            int64_t db; int ds;
            i2s_pos(k, &db, &ds);
            db += r * (Kp / 4);
            dst[db] = (uint8_t)((dst[db] & ~(3 << ds)) | (code << ds));
        }
    }
    float scale;
    memcpy(&scale, src + nrow * K / 4, sizeof(float));
    put_scale(dst, code_bytes, scale);
    return code_bytes + 32;
}

/* quantize_row_i8_s restated (per token). */
void orc_act_quant(const float *x, int64_t M, int64_t K, int8_t *q, float *s, int32_t *sums) {
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * K;
        double amax = 0.00001;
        for (int64_t k = 0; k < K; ++k) {
            double a = fabs((double)xr[k]);
            if (a > amax) amax = a;
        }
        const float sc = (float)(127.0 / amax);
        int32_t sum = 0;
        for (int64_t k = 0; k < K; ++k) {
            const float prod = xr[k] * sc; /* fp32 product */
            double r = round((double)prod);
            if (r > 127) r = 127;
            if (r < -128) r = -128;
            const int8_t v = (int8_t)r;
            q[m * K + k] = v;
            sum += v;
        }
        s[m] = sc;
        if (sums) sums[m] = sum;
    }
}

void orc_gemm_i32(const int8_t *t, const int8_t *q, int64_t M, int64_t N, int64_t K, int32_t *acc) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            int32_t a = 0;
            const int8_t *tr = t + n * K, *qr = q + m * K;
            for (int64_t k = 0; k < K; ++k) a += (int32_t)tr[k] * (int32_t)qr[k];
            acc[m * N + n] = a;
        }
}

void orc_rescale(const int32_t *acc, const float *s, float w_scale, int64_t M, int64_t N, float *y) {
    for (int64_t m = 0; m < M; ++m) {
        const float r = w_scale / s[m];
        for (int64_t n = 0; n < N; ++n) y[m * N + n] = (float)acc[m * N + n] * r;
    }
}

void orc_mul_mat_i2s(const uint8_t *W, const float *X, int64_t M, int64_t N, int64_t K, float *Y) {
    int8_t *t = (int8_t *)malloc((size_t)(N * K));
    int8_t *q = (int8_t *)malloc((size_t)(M * K));
    float *s = (float *)malloc(sizeof(float) * (size_t)M);
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)(M * N));
    const float ws = orc_i2s_unpack_ternary(W, t, N, K);
    orc_act_quant(X, M, K, q, s, NULL);
    orc_gemm_i32(t, q, M, N, K, acc);
    orc_rescale(acc, s, ws, M, N, Y);
    free(t); free(q); free(s); free(acc);
}

void orc_rms_norm(const float *x, const float *g, int64_t M, int64_t K, float eps, float *y) {
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * K;
        double sum = 0.0;
        for (int64_t k = 0; k < K; ++k) sum += (double)(xr[k] * xr[k]);
        const float mean = (float)(sum / (double)K);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t k = 0; k < K; ++k) {
            float v = xr[k] * scale;
            if (g) v = v * g[k];
            y[m * K + k] = v;
        }
    }
}

void orc_sqrelu_mul(const float *g, const float *u, int64_t n, float *p) {
    for (int64_t i = 0; i < n; ++i) {
        const float r = g[i] > 0.0f ? g[i] : 0.0f;
        const float r2 = r * r;
        p[i] = r2 * u[i];
    }
}

/* exp by Cody-Waite range reduction (x = n ln2 + r, ln2 split into a 16-bit head and a tail) and the
 * degree-7 Taylor polynomial of e^r in Horner form with fused multiply-adds, scaled by 2^n; inputs below
 * -86 give 0, above 88 saturate. The same IEEE operation sequence as the device's det_expf. */
float orc_det_expf(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    if (x > 88.0f) x = 88.0f;
    const float n = rintf(x * 1.44269502162933349609375f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.428606765330187045e-06f, r);
    float p = 1.98412698412698412698e-04f;
    p = fmaf(p, r, 1.38888888888888888889e-03f);
    p = fmaf(p, r, 8.33333333333333333333e-03f);
    p = fmaf(p, r, 4.16666666666666666667e-02f);
    p = fmaf(p, r, 1.66666666666666666667e-01f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const uint32_t bits = (uint32_t)((int)n + 127) << 23;
    float two_n;
    memcpy(&two_n, &bits, sizeof two_n);
    return p * two_n;
}

/* 1 / d for a normal d > 0 (the device's det_recipf): the bit-pattern seed 0x7EF311C3 - bits(d) (within
 * 12.5%) and three Newton-Raphson steps y <- y + y (1 - d y), each two fused multiply-adds; relative error
 * below 2^-22. */
float orc_det_recipf(float d) {
    uint32_t bits;
    memcpy(&bits, &d, sizeof bits);
    bits = 0x7EF311C3u - bits;
    float y;
    memcpy(&y, &bits, sizeof y);
    for (int i = 0; i < 3; ++i) y = fmaf(y, fmaf(-d, y, 1.0f), y);
    return y;
}

/* tanh(u) = sign(u) (1 - 2 / (e^{2|u|} + 1)) with the reciprocal of orc_det_recipf, |u| > 9 -> +-1 (the
 * device's det_tanhf). */
float orc_det_tanhf(float u) {
    const float a = fabsf(u);
    const float t = (a > 9.0f) ? 1.0f : 1.0f - 2.0f * orc_det_recipf(orc_det_expf(2.0f * a) + 1.0f);
    return copysignf(t, u);
}

/* Sum of e[0..n) in the device's warp order: lane l adds e[j], j = l mod 32, for increasing j; then
 * an xor butterfly over the 32 lane sums (offsets 16, 8, 4, 2, 1); the result is lane 0's value. */
float orc_warp_order_sum(const float *e, int64_t n) {
    float lanes[32], nxt[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t j = l; j < n; j += 32) acc = acc + e[j];
        lanes[l] = acc;
    }
    for (int off = 16; off > 0; off >>= 1) {
        for (int l = 0; l < 32; ++l) nxt[l] = lanes[l] + lanes[l ^ off];
        memcpy(lanes, nxt, sizeof lanes);
    }
    return lanes[0];
}

void orc_soft_max_ext(const float *x, const float *mask, int64_t mask_rows, int64_t M, int64_t N,
                      float scale, float *y) {
    float *w = (float *)malloc(sizeof(float) * (size_t)N);
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * N;
        const float *mr = mask ? mask + (m % mask_rows) * N : NULL;
        float mx = -INFINITY;
        for (int64_t n = 0; n < N; ++n) {
            float v = xr[n] * scale;
            if (mr) v = v + mr[n];
            w[n] = v;
            if (v > mx) mx = v;
        }
        for (int64_t n = 0; n < N; ++n) w[n] = (w[n] == -INFINITY) ? 0.0f : orc_det_expf(w[n] - mx);
        const float sum = orc_warp_order_sum(w, N);
        const float inv = (sum > 0.0f) ? 1.0f / sum : 0.0f;
        for (int64_t n = 0; n < N; ++n) y[m * N + n] = w[n] * inv;
    }
    free(w);
}

void orc_ffn_block(const float *X, int64_t M, int64_t H, int64_t F,
                   const float *g_norm1, const float *g_norm2, float eps,
                   const uint8_t *W_gate, const uint8_t *W_up, const uint8_t *W_down,
                   float *Y, float *P_dbg) {
    float *xn = (float *)malloc(sizeof(float) * (size_t)(M * H));
    float *gt = (float *)malloc(sizeof(float) * (size_t)(M * F));
    float *up = (float *)malloc(sizeof(float) * (size_t)(M * F));
    float *p = (float *)malloc(sizeof(float) * (size_t)(M * F));
    orc_rms_norm(X, g_norm1, M, H, eps, xn);
    orc_mul_mat_i2s(W_gate, xn, M, F, H, gt);
    orc_mul_mat_i2s(W_up, xn, M, F, H, up);
    orc_sqrelu_mul(gt, up, M * F, p);
    if (P_dbg) memcpy(P_dbg, p, sizeof(float) * (size_t)(M * F));
    orc_rms_norm(p, g_norm2, M, F, eps, p);
    orc_mul_mat_i2s(W_down, p, M, H, F, Y);
    free(xn); free(gt); free(up); free(p);
}
