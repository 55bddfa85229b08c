/*
 * i2s_cpu_fast.c -- threaded SIMD i2_s mul_mat on the host cores (TEST INFRASTRUCTURE).
 *
 * The timed CPU baseline for bench.py. The reference's own CPU i2_s kernel lives in microsoft/BitNet's
 * ggml fork (ggml_vec_dot_i2_i8_s), which is absent from the reference tree, so this file restates
 * that kernel's method: decode the 2-bit codes {0,1,2} of one 32-byte block into four 32-byte vectors
 * with shift+mask, multiply them as unsigned bytes against the signed int8 activations
 * (AVX512-VNNI vpdpbusd, or AVX2 vpmaddubsw+vpmaddwd), and subtract the per-token activation sum,
 * since sum_k (t_k+1) q_k - sum_k q_k = sum_k t_k q_k.
 * Integer results are exact, and the fp32 steps call the scalar oracle's per-row functions, so the
 * output is bit-identical to i2s_oracle.c.
 */
#include "i2s_oracle.h"

#include <immintrin.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QK 128

/* Minimal static parallel-for over [0, n) on nthreads pthreads (no OpenMP runtime needed). */
typedef void (*range_fn)(void *ctx, int64_t begin, int64_t end);
typedef struct { range_fn fn; void *ctx; int64_t begin, end; } range_job;
static void *range_thunk(void *p) { range_job *j = (range_job *)p; j->fn(j->ctx, j->begin, j->end); return NULL; }
void orc_parallel_for(int64_t n, int nthreads, range_fn fn, void *ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (n < nthreads) nthreads = (int)(n > 0 ? n : 1);
    pthread_t th[256];
    range_job jobs[256];
    for (int i = 0; i < nthreads; ++i) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].begin = n * i / nthreads; jobs[i].end = n * (i + 1) / nthreads;
    }
    for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, range_thunk, &jobs[i]);
    range_thunk(&jobs[0]);
    for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
}

static int64_t rup128(int64_t k) { return (k + QK - 1) / QK * QK; }

int orc_fast_isa(void) {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl") &&
        __builtin_cpu_supports("avx512bw"))
        return 2;
    if (__builtin_cpu_supports("avx2")) return 1;
    return 0;
}

/* Decode one row-padded row (Kp/4 bytes) into Kp code bytes in {0,1,2}. */
static void decode_row_scalar(const uint8_t *src, uint8_t *codes, int64_t Kp) {
    for (int64_t b = 0; b < Kp / QK; ++b)
        for (int j = 0; j < QK; ++j) codes[b * QK + j] = (src[b * 32 + (j % 32)] >> (6 - 2 * (j / 32))) & 3;
}

__attribute__((target("avx2"))) static void decode_row_avx2(const uint8_t *src, uint8_t *codes, int64_t Kp) {
    const __m256i m3 = _mm256_set1_epi8(3);
    for (int64_t b = 0; b < Kp / QK; ++b) {
        __m256i v = _mm256_loadu_si256((const __m256i *)(src + 32 * b));
        _mm256_storeu_si256((__m256i *)(codes + b * QK + 0), _mm256_and_si256(_mm256_srli_epi16(v, 6), m3));
        _mm256_storeu_si256((__m256i *)(codes + b * QK + 32), _mm256_and_si256(_mm256_srli_epi16(v, 4), m3));
        _mm256_storeu_si256((__m256i *)(codes + b * QK + 64), _mm256_and_si256(_mm256_srli_epi16(v, 2), m3));
        _mm256_storeu_si256((__m256i *)(codes + b * QK + 96), _mm256_and_si256(v, m3));
    }
}

__attribute__((target("avx2"))) static inline int32_t hsum8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

#define RB 4 /* rows per register block */
#define TB 4 /* tokens per register block */

/* codes: RB x Kp (u8), q: M x Kp (s8, zero padded). raw[t*RB + r] = sum_k codes[r][k]*q[t][k]. */
__attribute__((target("avx2,avx512vl,avx512bw,avx512vnni"))) static void
block_dot_vnni(const uint8_t *codes, int nr, const int8_t *q, int nt, int64_t Kp, int32_t *raw) {
    __m256i acc[RB][TB];
    for (int r = 0; r < RB; ++r)
        for (int t = 0; t < TB; ++t) acc[r][t] = _mm256_setzero_si256();
    for (int64_t k = 0; k < Kp; k += 32) {
        __m256i c[RB], x[TB];
        for (int r = 0; r < RB; ++r) c[r] = _mm256_loadu_si256((const __m256i *)(codes + (r < nr ? r : 0) * Kp + k));
        for (int t = 0; t < TB; ++t) x[t] = _mm256_loadu_si256((const __m256i *)(q + (t < nt ? t : 0) * Kp + k));
        for (int r = 0; r < RB; ++r)
            for (int t = 0; t < TB; ++t) acc[r][t] = _mm256_dpbusd_epi32(acc[r][t], c[r], x[t]);
    }
    for (int r = 0; r < RB; ++r)
        for (int t = 0; t < TB; ++t) raw[t * RB + r] = hsum8(acc[r][t]);
}

__attribute__((target("avx2"))) static void
block_dot_avx2(const uint8_t *codes, int nr, const int8_t *q, int nt, int64_t Kp, int32_t *raw) {
    __m256i acc[RB][TB];
    const __m256i ones = _mm256_set1_epi16(1);
    for (int r = 0; r < RB; ++r)
        for (int t = 0; t < TB; ++t) acc[r][t] = _mm256_setzero_si256();
    for (int64_t k = 0; k < Kp; k += 32) {
        __m256i c[RB], x[TB];
        for (int r = 0; r < RB; ++r) c[r] = _mm256_loadu_si256((const __m256i *)(codes + (r < nr ? r : 0) * Kp + k));
        for (int t = 0; t < TB; ++t) x[t] = _mm256_loadu_si256((const __m256i *)(q + (t < nt ? t : 0) * Kp + k));
        for (int r = 0; r < RB; ++r)
            for (int t = 0; t < TB; ++t)
                acc[r][t] = _mm256_add_epi32(acc[r][t], _mm256_madd_epi16(_mm256_maddubs_epi16(c[r], x[t]), ones));
    }
    for (int r = 0; r < RB; ++r)
        for (int t = 0; t < TB; ++t) raw[t * RB + r] = hsum8(acc[r][t]);
}

static void block_dot_scalar(const uint8_t *codes, int nr, const int8_t *q, int nt, int64_t Kp, int32_t *raw) {
    for (int t = 0; t < TB; ++t)
        for (int r = 0; r < RB; ++r) {
            int32_t a = 0;
            if (r < nr && t < nt)
                for (int64_t k = 0; k < Kp; ++k) a += (int32_t)codes[r * Kp + k] * (int32_t)q[t * Kp + k];
            raw[t * RB + r] = a;
        }
}

/* Y[M,N] from row-padded weights Wr (Kp per row) and zero-padded activations q (M x Kp). */
typedef struct {
    const uint8_t *Wr; int64_t N, Kp; const int8_t *q; const float *s; const int32_t *sums;
    float ws; int64_t M; float *Y; int isa;
    const float *tile_scales; int64_t ldy; /* NULL: ws for every row; else row n uses tile_scales[n/128] */
} gemm_ctx;

static void gemm_range(void *p, int64_t g0, int64_t g1) {
    const gemm_ctx *c = (const gemm_ctx *)p;
    const int64_t Kp = c->Kp, N = c->N, M = c->M;
    uint8_t *codes = (uint8_t *)aligned_alloc(64, (size_t)(RB * Kp));
    memset(codes, 0, (size_t)(RB * Kp));
    int32_t raw[RB * TB];
    for (int64_t gi = g0; gi < g1; ++gi) {
        const int64_t n0 = gi * RB;
        const int nr = (int)((N - n0) < RB ? (N - n0) : RB);
        for (int r = 0; r < nr; ++r) {
            if (c->isa >= 1) decode_row_avx2(c->Wr + (n0 + r) * (Kp / 4), codes + r * Kp, Kp);
            else decode_row_scalar(c->Wr + (n0 + r) * (Kp / 4), codes + r * Kp, Kp);
        }
        for (int64_t m0 = 0; m0 < M; m0 += TB) {
            const int nt = (int)((M - m0) < TB ? (M - m0) : TB);
            if (c->isa == 2) block_dot_vnni(codes, nr, c->q + m0 * Kp, nt, Kp, raw);
            else if (c->isa == 1) block_dot_avx2(codes, nr, c->q + m0 * Kp, nt, Kp, raw);
            else block_dot_scalar(codes, nr, c->q + m0 * Kp, nt, Kp, raw);
            const float ws = c->tile_scales ? c->tile_scales[n0 / QK] : c->ws;
            for (int t = 0; t < nt; ++t) {
                const float rs = ws / c->s[m0 + t];
                for (int r = 0; r < nr; ++r)
                    c->Y[(m0 + t) * c->ldy + n0 + r] = (float)(raw[t * RB + r] - c->sums[m0 + t]) * rs;
            }
        }
    }
    free(codes);
}

typedef struct { const float *X; int64_t K, Kp; int8_t *q; float *s; int32_t *sums; } actq_ctx;

static void actq_range(void *p, int64_t m0, int64_t m1) {
    const actq_ctx *c = (const actq_ctx *)p;
    for (int64_t m = m0; m < m1; ++m) {
        orc_act_quant(c->X + m * c->K, 1, c->K, c->q + m * c->Kp, c->s + m, c->sums + m);
        memset(c->q + m * c->Kp + c->K, 0, (size_t)(c->Kp - c->K));
    }
}

void orc_fast_mul_mat_i2s(const uint8_t *W, const float *X, int64_t M, int64_t N, int64_t K, float *Y,
                          int nthreads) {
    const int isa = orc_fast_isa();
    const int64_t Kp = rup128(K);
    const uint8_t *Wr = W;
    uint8_t *tmp = NULL;
    if (Kp != K) {
        tmp = (uint8_t *)malloc(orc_i2s_r_nbytes(N, K));
        orc_i2s_to_rowpadded(W, tmp, N, K);
        Wr = tmp;
    }
    float ws;
    memcpy(&ws, Wr + N * Kp / 4, sizeof(float));
    int8_t *q = (int8_t *)aligned_alloc(64, (size_t)((M * Kp + 63) / 64 * 64));
    float *s = (float *)malloc(sizeof(float) * (size_t)M);
    int32_t *sums = (int32_t *)malloc(sizeof(int32_t) * (size_t)M);
    actq_ctx ac = {X, K, Kp, q, s, sums};
    orc_parallel_for(M, nthreads, actq_range, &ac);
    gemm_ctx gc = {Wr, N, Kp, q, s, sums, ws, M, Y, isa, NULL, N};
    orc_parallel_for((N + RB - 1) / RB, nthreads, gemm_range, &gc);
    free(q); free(s); free(sums); free(tmp);
}

void orc_fast_gemm_q8_rp(const uint8_t *Wr, const float *tile_scales, int64_t N, int64_t K, const int8_t *q,
                         const float *s, const int32_t *sums, int64_t M, float *Y, int64_t ldy, int nthreads) {
    gemm_ctx gc = {Wr, N, rup128(K), q, s, sums, 0.0f, M, Y, orc_fast_isa(), tile_scales, ldy};
    orc_parallel_for((N + RB - 1) / RB, nthreads, gemm_range, &gc);
}

void orc_fast_act_quant_padded(const float *X, int64_t M, int64_t K, int8_t *q, float *s, int32_t *sums,
                               int nthreads) {
    actq_ctx ac = {X, K, rup128(K), q, s, sums};
    orc_parallel_for(M, nthreads, actq_range, &ac);
}

typedef struct { const float *x; const float *g; int64_t K; float eps; float *y; } rms_ctx;

static void rms_range(void *p, int64_t m0, int64_t m1) {
    const rms_ctx *c = (const rms_ctx *)p;
    for (int64_t m = m0; m < m1; ++m) orc_rms_norm(c->x + m * c->K, c->g, 1, c->K, c->eps, c->y + m * c->K);
}

typedef struct { const float *g; const float *u; int64_t F; float *p; } sq_ctx;

static void sq_range(void *p, int64_t m0, int64_t m1) {
    const sq_ctx *c = (const sq_ctx *)p;
    for (int64_t m = m0; m < m1; ++m) orc_sqrelu_mul(c->g + m * c->F, c->u + m * c->F, c->F, c->p + m * c->F);
}

void orc_fast_ffn_block(const float *X, int64_t M, int64_t H, int64_t F,
                        const float *g_norm1, const float *g_norm2, float eps,
                        const uint8_t *W_gate, const uint8_t *W_up, const uint8_t *W_down,
                        float *Y, int nthreads) {
    float *xn = (float *)malloc(sizeof(float) * (size_t)(M * H));
    float *gt = (float *)malloc(sizeof(float) * (size_t)(M * F));
    float *up = (float *)malloc(sizeof(float) * (size_t)(M * F));
    rms_ctx r1 = {X, g_norm1, H, eps, xn};
    orc_parallel_for(M, nthreads, rms_range, &r1);
    orc_fast_mul_mat_i2s(W_gate, xn, M, F, H, gt, nthreads);
    orc_fast_mul_mat_i2s(W_up, xn, M, F, H, up, nthreads);
    sq_ctx sq = {gt, up, F, gt};
    orc_parallel_for(M, nthreads, sq_range, &sq);
    rms_ctx r2 = {gt, g_norm2, F, eps, gt};
    orc_parallel_for(M, nthreads, rms_range, &r2);
    orc_fast_mul_mat_i2s(W_down, gt, M, H, F, Y, nthreads);
    free(xn); free(gt); free(up);
}
