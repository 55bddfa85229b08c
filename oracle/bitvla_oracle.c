/*
 * bitvla_oracle.c -- CPU restatement of the random-init BitVLA-shape forward (TEST INFRASTRUCTURE).
 *
 * Only tests/ (and the CPU-baseline leg of bench.py) call this; the product library never does.
 * It regenerates the model from the seed with the documented parameter generator and runs the same
 * layer sequence as the device engine, one operator at a time on fp32 host arrays:
 *   ViT block (src/models/smolvla/vision.cpp:305-345 structure): LayerNorm -> act-quant -> q/k/v (+bias)
 *     -> softmax attention -> act-quant -> o (+bias) + residual -> LayerNorm -> act-quant -> fc1 (+bias)
 *     -> GELU(tanh) -> act-quant -> fc2 (+bias) + residual;
 *   connector: post-LayerNorm -> act-quant -> ternary 1152->2560 (+bias) -> GELU -> act-quant ->
 *     ternary 2560->2560 (+bias);
 *   decoder layer (src/models/pi0/vlm.cpp:196-246 structure, BitNet b1.58 sub-norms): RMSNorm ->
 *     act-quant -> q/k/v -> NEOX RoPE -> causal GQA attention -> RMSNorm(attn_sub) -> act-quant -> o +
 *     residual -> RMSNorm -> act-quant -> gate/up -> relu(g)^2 * u -> RMSNorm(ffn_sub) -> act-quant ->
 *     down + residual; final RMSNorm; action head on the last token.
 * Every step is the same IEEE operation sequence as the device kernels (fused multiply-adds where the
 * device uses them, exp/tanh from orc_det_expf/orc_det_tanhf, sums in the device's order), so the whole
 * forward agrees bit for bit; the one unpinned order is the double-precision sum inside the norms
 * (sequential here, a tree on the device), whose rounding to fp32 agrees except with probability
 * ~2^-29 per row.
 *
 * Parameter generator (shared definition with include/b2s_bitvla.h):
 *   bits(seed, tensor, idx) = mix(mix(seed ^ mix(tensor * 0x9E3779B1 + 0x7F4A7C15)) ^ (idx * 0x85EBCA77 +
 *   0x165667B1)) with mix the murmur3 32-bit finalizer; u = bits >> 8 (24 bits).
 *   ternary weight (row r, column k of a K-wide tensor): idx = r*K + k; u < 5033165 -> -1,
 *   u < 11744051 -> 0, else +1; tensor scale = (0.5 + 1.5 u') / sqrt(0.6 K), u' from idx 0xFFFFFFFF.
 *   fp32 parameter: lo + (hi - lo) * (u * 2^-24); text embedding row of token t: tensor 0x80000000 | t.
 *   Tensor ids: patch_w 1, patch_b 2, pos 3, post_w 4, post_b 5, conn1 6, conn1_b 7, conn2 8, conn2_b 9,
 *   final_norm 10, act_w 11, act_b 12; ViT layer l: 0x100 + 16 l + slot (ln1_w, ln1_b, q, k, v, q_b, k_b,
 *   v_b, o, o_b, ln2_w, ln2_b, fc1, fc1_b, fc2, fc2_b); decoder layer l: 0x10000 + 16 l + slot
 *   (attn_norm, q, k, v, attn_sub_norm, o, ffn_norm, gate, up, ffn_sub_norm, down).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "../include/b2s_bitvla.h"
#include "i2s_oracle.h"

#define QK 128

static uint32_t pmix(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

uint32_t orc_bv_param_bits(uint32_t seed, uint32_t tensor, uint32_t idx) {
    const uint32_t t = pmix(seed ^ pmix(tensor * 0x9E3779B1u + 0x7F4A7C15u));
    return pmix(t ^ (idx * 0x85EBCA77u + 0x165667B1u));
}

static float unit24(uint32_t bits) { return (float)(bits >> 8) * (1.0f / 16777216.0f); }

float orc_bv_ternary_scale(uint32_t seed, uint32_t tensor, int64_t K) {
    const float u = unit24(orc_bv_param_bits(seed, tensor, 0xFFFFFFFFu));
    const float a = 0.5f + 1.5f * u;
    const float r = sqrtf(0.6f * (float)K);
    return a / r;
}

static int64_t rup(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

/* ---------------------------------------------------------------- parameter generation */
typedef struct { uint8_t *dst; int64_t K, Kp; uint32_t seed, id; } tern_ctx;

static void tern_range(void *p, int64_t r0, int64_t r1) {
    const tern_ctx *c = (const tern_ctx *)p;
    const int64_t rb = c->Kp / 4;
    for (int64_t r = r0; r < r1; ++r)
        for (int64_t j = 0; j < rb; ++j) {
            const int64_t b = j / 32, i = j % 32;
            uint32_t out = 0;
            for (int g = 0; g < 4; ++g) {
                const int64_t k = QK * b + 32 * g + i;
                uint32_t code = 1;
                if (k < c->K) {
                    const uint32_t u = orc_bv_param_bits(c->seed, c->id, (uint32_t)(r * c->K + k)) >> 8;
                    code = u < 5033165u ? 0u : (u < 11744051u ? 1u : 2u);
                }
                out |= code << (6 - 2 * g);
            }
            c->dst[r * rb + j] = (uint8_t)out;
        }
}

/* Row-padded codes of `rows` rows of tensor `id` (K inputs) written at dst. */
void orc_bv_gen_ternary(uint8_t *dst, int64_t rows, int64_t K, uint32_t seed, uint32_t id, int nthreads) {
    tern_ctx c = {dst, K, rup(K, QK), seed, id};
    orc_parallel_for(rows, nthreads, tern_range, &c);
}

void orc_bv_gen_uniform(float *dst, int64_t n, uint32_t seed, uint32_t id, float lo, float hi) {
    const float width = hi - lo;
    for (int64_t i = 0; i < n; ++i) dst[i] = lo + width * unit24(orc_bv_param_bits(seed, id, (uint32_t)i));
}

/* Stacked ternary weight: parts of rows n[i] from tensors id[i], tile scales per 128 rows. */
typedef struct { uint8_t *codes; float *tiles; int64_t N, K; } tern_w;

static tern_w make_tern(int nparts, const int64_t *rows, const uint32_t *ids, int64_t K, uint32_t seed, int nth) {
    tern_w w;
    w.N = 0;
    for (int i = 0; i < nparts; ++i) w.N += rows[i];
    w.K = K;
    const int64_t rb = rup(K, QK) / 4;
    w.codes = (uint8_t *)malloc((size_t)(w.N * rb));
    w.tiles = (float *)malloc(sizeof(float) * (size_t)((w.N + QK - 1) / QK));
    int64_t r0 = 0;
    for (int i = 0; i < nparts; ++i) {
        orc_bv_gen_ternary(w.codes + r0 * rb, rows[i], K, seed, ids[i], nth);
        const float sc = orc_bv_ternary_scale(seed, ids[i], K);
        for (int64_t r = r0; r < r0 + rows[i]; r += QK) w.tiles[r / QK] = sc;
        r0 += rows[i];
    }
    return w;
}
static tern_w make_tern1(int64_t N, uint32_t id, int64_t K, uint32_t seed, int nth) {
    return make_tern(1, &N, &id, K, seed, nth);
}
static void free_tern(tern_w *w) { free(w->codes); free(w->tiles); }

static float *uniform_new(int64_t n, uint32_t seed, uint32_t id, float lo, float hi) {
    float *p = (float *)malloc(sizeof(float) * (size_t)n);
    orc_bv_gen_uniform(p, n, seed, id, lo, hi);
    return p;
}

/* ---------------------------------------------------------------- operators */
/* LayerNorm as ggml_norm + ggml_mul + ggml_add: mean = (float)(sum x / K) (double sum), v = x - mean,
 * var = (float)(sum v^2 / K), y = ((v * (1/sqrtf(var + eps))) * g) + b. In place allowed. */
void orc_layer_norm(const float *x, const float *g, const float *b, int64_t M, int64_t K, float eps, float *y) {
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * K;
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) acc += (double)xr[k];
        const float mean = (float)(acc / (double)K);
        double acc2 = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const float v = xr[k] - mean;
            acc2 += (double)(v * v);
        }
        const float var = (float)(acc2 / (double)K);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int64_t k = 0; k < K; ++k) {
            float v = (xr[k] - mean) * scale;
            if (g) v = v * g[k];
            if (b) v = v + b[k];
            y[m * K + k] = v;
        }
    }
}

/* GELU, tanh approximation, in the device's operation order (tanh = orc_det_tanhf). */
float orc_gelu_tanh(float x) {
    const float inner = (0.79788456080286535588f * x) * (1.0f + (0.044715f * x) * x);
    return (0.5f * x) * (1.0f + orc_det_tanhf(inner));
}

/* (cos, sin) of theta = pos * base^(-2i/d), evaluated in double and rounded to fp32. */
void orc_rope_table(float base, int hd, int n_pos, float *cs /* [n_pos][hd/2][2] */) {
    const int half = hd / 2;
    for (int p = 0; p < n_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const double inv = pow((double)base, -2.0 * (double)i / (double)hd);
            const double th = (double)p * inv;
            cs[2 * (p * half + i)] = (float)cos(th);
            cs[2 * (p * half + i) + 1] = (float)sin(th);
        }
}

/* NEOX rotation of n_heads heads of M rows (row m at position pos0 + m % period). */
void orc_rope_neox(float *x, int64_t M, int n_heads, int hd, int64_t ld, const float *cs, int period, int pos0) {
    const int half = hd / 2;
    for (int64_t m = 0; m < M; ++m)
        for (int h = 0; h < n_heads; ++h) {
            float *r = x + m * ld + (int64_t)h * hd;
            const int p = pos0 + (int)(period > 0 ? m % period : m);
            for (int i = 0; i < half; ++i) {
                const float c = cs[2 * (p * half + i)], s = cs[2 * (p * half + i) + 1];
                const float x0 = r[i], x1 = r[i + half];
                r[i] = x0 * c - x1 * s;
                r[i + half] = x0 * s + x1 * c;
            }
        }
}

/* Attention of `batch` sequences of T tokens: head h reads q columns [h hd, (h+1) hd) at q_off, its K/V
 * head g = h / (heads / kv_heads) at k_off / v_off. The device kernel's fixed fp32 evaluation, an online
 * softmax over chunks of 64 keys (chunk c = keys [64c, 64c + 64)); for row i with n_i keys (i + 1 if
 * causal, else T):
 *   s_j = fp32(acc * scale), acc = fmaf(q[i][d], k[j][d], acc) over d ascending from +0 (-inf if j >= n_i);
 *   per chunk: m' = max(m, max s_j), alpha = orc_det_expf(m - m'), p_j = orc_det_expf(s_j - m'),
 *   csum = xor butterfly (8, 4, 2, 1) over partials ((p_4t + p_4t+1) + p_4t+2) + p_4t+3, t = 0..15,
 *   l = l * alpha + csum, o[d] = o[d] * alpha then o[d] = fmaf(p_j, v[j][d], o[d]) for j ascending;
 *   out[d] = o[d] * (1 / l). Chunks past the row's last key change nothing, so they are skipped. */
typedef struct {
    const float *qkv; int64_t ld, q_off, k_off, v_off; int batch, heads, kv_heads, hd, T, causal;
    float scale; float *o; int64_t ldo;
} attn_ctx;

static void attn_range(void *p, int64_t i0, int64_t i1) {
    const attn_ctx *c = (const attn_ctx *)p;
    float *acc = (float *)malloc(sizeof(float) * (size_t)c->hd);
    const int group = c->heads / c->kv_heads;
    for (int64_t it = i0; it < i1; ++it) {
        const int b = (int)(it / c->heads), h = (int)(it % c->heads), g = h / group;
        const float *rows = c->qkv + (int64_t)b * c->T * c->ld;
        for (int i = 0; i < c->T; ++i) {
            const float *qi = rows + (int64_t)i * c->ld + c->q_off + (int64_t)h * c->hd;
            const int nk = c->causal ? i + 1 : c->T;
            float m = -INFINITY, l = 0.0f;
            for (int d = 0; d < c->hd; ++d) acc[d] = 0.0f;
            for (int k0 = 0; k0 < nk; k0 += 64) {
                float sc[64], pr[64];
                float cm = -INFINITY;
                for (int jj = 0; jj < 64; ++jj) {
                    const int j = k0 + jj;
                    if (j < nk) {
                        const float *kj = rows + (int64_t)j * c->ld + c->k_off + (int64_t)g * c->hd;
                        float a = 0.0f;
                        for (int d = 0; d < c->hd; ++d) a = fmaf(qi[d], kj[d], a);
                        sc[jj] = a * c->scale;
                    } else {
                        sc[jj] = -INFINITY;
                    }
                    if (sc[jj] > cm) cm = sc[jj];
                }
                const float mn = (m > cm) ? m : cm;
                const float alpha = orc_det_expf(m - mn);
                float part[16], nxt[16];
                for (int jj = 0; jj < 64; ++jj) pr[jj] = orc_det_expf(sc[jj] - mn);
                for (int tq = 0; tq < 16; ++tq) part[tq] = ((pr[4 * tq] + pr[4 * tq + 1]) + pr[4 * tq + 2]) + pr[4 * tq + 3];
                for (int off = 8; off > 0; off >>= 1) {
                    for (int tq = 0; tq < 16; ++tq) nxt[tq] = part[tq] + part[tq ^ off];
                    memcpy(part, nxt, sizeof part);
                }
                l = l * alpha + part[0];
                m = mn;
                const int jn = (nk - k0 < 64) ? nk - k0 : 64;
                for (int d = 0; d < c->hd; ++d) {
                    float a = acc[d] * alpha;
                    for (int jj = 0; jj < jn; ++jj)
                        a = fmaf(pr[jj], rows[(int64_t)(k0 + jj) * c->ld + c->v_off + (int64_t)g * c->hd + d], a);
                    acc[d] = a;
                }
            }
            const float inv = (l > 0.0f) ? 1.0f / l : 0.0f;
            float *oi = c->o + ((int64_t)b * c->T + i) * c->ldo + (int64_t)h * c->hd;
            for (int d = 0; d < c->hd; ++d) oi[d] = acc[d] * inv;
        }
    }
    free(acc);
}

void orc_attention(const float *qkv, int64_t ld, int64_t q_off, int64_t k_off, int64_t v_off, int batch, int heads,
                   int kv_heads, int hd, int T, int causal, float scale, float *o, int64_t ldo, int nthreads) {
    attn_ctx c = {qkv, ld, q_off, k_off, v_off, batch, heads, kv_heads, hd, T, causal, scale, o, ldo};
    orc_parallel_for((int64_t)batch * heads, nthreads, attn_range, &c);
}

/* ---------------------------------------------------------------- linear layers */
typedef struct { int8_t *q; float *s; int32_t *sums; } q8buf;

/* act-quant of x [M][K] into the shared int8 buffer (rows Kp = roundup(K, 128), zero-padded). */
static void quant(const float *x, int64_t M, int64_t K, q8buf *qb, int nth) {
    orc_fast_act_quant_padded(x, M, K, qb->q, qb->s, qb->sums, nth);
}

typedef struct { const float *tmp; int64_t N, ldy; float *y; const float *bias, *res; int act; } epi_ctx;

static void epi_range(void *p, int64_t m0, int64_t m1) {
    const epi_ctx *c = (const epi_ctx *)p;
    for (int64_t m = m0; m < m1; ++m)
        for (int64_t n = 0; n < c->N; ++n) {
            float v = c->tmp[m * c->N + n];
            if (c->bias) v = v + c->bias[n];
            if (c->act == 1) v = orc_gelu_tanh(v);
            if (c->res) v = c->res[m * c->ldy + n] + v;
            c->y[m * c->ldy + n] = v;
        }
}

/* y = W q (+ bias) (GELU if act) (+ residual, res may alias y): the device epilogue order. `tmp` holds
 * M x N floats. */
static void linear(const tern_w *w, const q8buf *qb, int64_t M, float *y, int64_t ldy, const float *bias, int act,
                   const float *res, float *tmp, int nth) {
    orc_fast_gemm_q8_rp(w->codes, w->tiles, w->N, w->K, qb->q, qb->s, qb->sums, M, tmp, w->N, nth);
    epi_ctx c = {tmp, w->N, ldy, y, bias, res, act};
    orc_parallel_for(M, nth, epi_range, &c);
}

/* ---------------------------------------------------------------- the model (weights generated once) */
typedef struct {
    float *ln1_w, *ln1_b, *qkv_b, *o_b, *ln2_w, *ln2_b, *fc1_b, *fc2_b;
    tern_w qkv, wo, fc1, fc2;
} vit_layer;
typedef struct {
    float *attn_norm, *attn_sub, *ffn_norm, *ffn_sub;
    tern_w qkv, wo, gate, up, down;
} dec_layer;
typedef struct orc_bitvla_model orc_bitvla_model;
struct orc_bitvla_model {
    b2s_bitvla_config c;
    uint32_t seed;
    float *patch_w, *patch_b, *pos, *post_w, *post_b, *c1_b, *c2_b, *final_norm, *act_w, *act_b;
    tern_w c1, c2;
    vit_layer *vit;
    dec_layer *dec;
};

orc_bitvla_model *orc_bitvla_create(const b2s_bitvla_config *cfg, uint32_t seed, int nth) {
    orc_bitvla_model *m = (orc_bitvla_model *)calloc(1, sizeof(orc_bitvla_model));
    const b2s_bitvla_config c = *cfg;
    m->c = c;
    m->seed = seed;
    const int P = c.patch, G = c.image_size / P, np = G * G, kdim = 3 * P * P;
    const int D = c.vit_hidden, F = c.vit_ffn, H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim;
    const float pa = 1.0f / sqrtf((float)kdim);
    m->patch_w = uniform_new((int64_t)D * kdim, seed, 1, -pa, pa);
    m->patch_b = uniform_new(D, seed, 2, -0.02f, 0.02f);
    m->pos = uniform_new((int64_t)np * D, seed, 3, -0.02f, 0.02f);
    m->vit = (vit_layer *)calloc((size_t)(c.vit_layers > 0 ? c.vit_layers : 1), sizeof(vit_layer));
    for (int l = 0; l < c.vit_layers; ++l) {
        vit_layer *L = &m->vit[l];
        const uint32_t base = 0x100u + 16u * (uint32_t)l;
        L->ln1_w = uniform_new(D, seed, base + 0, 0.9f, 1.1f);
        L->ln1_b = uniform_new(D, seed, base + 1, -0.02f, 0.02f);
        const int64_t rows3[3] = {D, D, D};
        const uint32_t ids3[3] = {base + 2, base + 3, base + 4};
        L->qkv = make_tern(3, rows3, ids3, D, seed, nth);
        L->qkv_b = (float *)malloc(sizeof(float) * 3 * (size_t)D);
        for (int j = 0; j < 3; ++j) orc_bv_gen_uniform(L->qkv_b + j * D, D, seed, base + 5 + j, -0.02f, 0.02f);
        L->wo = make_tern1(D, base + 8, D, seed, nth);
        L->o_b = uniform_new(D, seed, base + 9, -0.02f, 0.02f);
        L->ln2_w = uniform_new(D, seed, base + 10, 0.9f, 1.1f);
        L->ln2_b = uniform_new(D, seed, base + 11, -0.02f, 0.02f);
        L->fc1 = make_tern1(F, base + 12, D, seed, nth);
        L->fc1_b = uniform_new(F, seed, base + 13, -0.02f, 0.02f);
        L->fc2 = make_tern1(D, base + 14, F, seed, nth);
        L->fc2_b = uniform_new(D, seed, base + 15, -0.02f, 0.02f);
    }
    m->post_w = uniform_new(D, seed, 4, 0.9f, 1.1f);
    m->post_b = uniform_new(D, seed, 5, -0.02f, 0.02f);
    m->c1 = make_tern1(c.conn_hidden, 6, D, seed, nth);
    m->c1_b = uniform_new(c.conn_hidden, seed, 7, -0.02f, 0.02f);
    m->c2 = make_tern1(H, 8, c.conn_hidden, seed, nth);
    m->c2_b = uniform_new(H, seed, 9, -0.02f, 0.02f);
    m->dec = (dec_layer *)calloc((size_t)(c.dec_layers > 0 ? c.dec_layers : 1), sizeof(dec_layer));
    for (int l = 0; l < c.dec_layers; ++l) {
        dec_layer *L = &m->dec[l];
        const uint32_t base = 0x10000u + 16u * (uint32_t)l;
        L->attn_norm = uniform_new(H, seed, base + 0, 0.9f, 1.1f);
        const int64_t rows3[3] = {H, KV, KV};
        const uint32_t ids3[3] = {base + 1, base + 2, base + 3};
        L->qkv = make_tern(3, rows3, ids3, H, seed, nth);
        L->attn_sub = uniform_new(H, seed, base + 4, 0.9f, 1.1f);
        L->wo = make_tern1(H, base + 5, H, seed, nth);
        L->ffn_norm = uniform_new(H, seed, base + 6, 0.9f, 1.1f);
        L->gate = make_tern1(c.dec_ffn, base + 7, H, seed, nth);
        L->up = make_tern1(c.dec_ffn, base + 8, H, seed, nth);
        L->ffn_sub = uniform_new(c.dec_ffn, seed, base + 9, 0.9f, 1.1f);
        L->down = make_tern1(H, base + 10, c.dec_ffn, seed, nth);
    }
    m->final_norm = uniform_new(H, seed, 10, 0.9f, 1.1f);
    const int NA = c.action_chunk * c.action_dim;
    const float aa = 1.0f / sqrtf((float)H);
    m->act_w = uniform_new((int64_t)NA * H, seed, 11, -aa, aa);
    m->act_b = uniform_new(NA, seed, 12, -0.02f, 0.02f);
    return m;
}

void orc_bitvla_free(orc_bitvla_model *m) {
    if (!m) return;
    for (int l = 0; l < m->c.vit_layers; ++l) {
        vit_layer *L = &m->vit[l];
        free(L->ln1_w); free(L->ln1_b); free(L->qkv_b); free(L->o_b); free(L->ln2_w); free(L->ln2_b);
        free(L->fc1_b); free(L->fc2_b);
        free_tern(&L->qkv); free_tern(&L->wo); free_tern(&L->fc1); free_tern(&L->fc2);
    }
    for (int l = 0; l < m->c.dec_layers; ++l) {
        dec_layer *L = &m->dec[l];
        free(L->attn_norm); free(L->attn_sub); free(L->ffn_norm); free(L->ffn_sub);
        free_tern(&L->qkv); free_tern(&L->wo); free_tern(&L->gate); free_tern(&L->up); free_tern(&L->down);
    }
    free(m->vit); free(m->dec);
    free(m->patch_w); free(m->patch_b); free(m->pos); free(m->post_w); free(m->post_b); free(m->c1_b);
    free(m->c2_b); free(m->final_norm); free(m->act_w); free(m->act_b);
    free_tern(&m->c1); free_tern(&m->c2);
    free(m);
}

/* Patch embedding rows: y = (bias + pos) + acc, acc = fmaf(col[k], w[d][k], acc), k ascending. */
typedef struct { const orc_bitvla_model *m; const float *images; float *vx; } patch_ctx;

static void patch_range(void *p, int64_t r0, int64_t r1) {
    const patch_ctx *pc = (const patch_ctx *)p;
    const b2s_bitvla_config *c = &pc->m->c;
    const int P = c->patch, G = c->image_size / P, np = G * G, kdim = 3 * P * P, D = c->vit_hidden;
    float *col = (float *)malloc(sizeof(float) * (size_t)kdim);
    for (int64_t r = r0; r < r1; ++r) {
        const int64_t b = r / np;
        const int p_ = (int)(r % np), py = p_ / G, px = p_ % G;
        for (int k = 0; k < kdim; ++k) {
            const int ch = k / (P * P), ky = (k / P) % P, kx = k % P;
            col[k] = pc->images[((b * 3 + ch) * c->image_size + (py * P + ky)) * c->image_size + (px * P + kx)];
        }
        for (int d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int k = 0; k < kdim; ++k) acc = fmaf(col[k], pc->m->patch_w[(int64_t)d * kdim + k], acc);
            const float pre = pc->m->patch_b[d] + pc->m->pos[(int64_t)p_ * D + d];
            pc->vx[r * D + d] = pre + acc;
        }
    }
    free(col);
}

int orc_bitvla_run(const orc_bitvla_model *m, int batch, const float *images, const int32_t *tokens, float *hidden,
                   float *actions, int nth) {
    const b2s_bitvla_config c = m->c;
    const uint32_t seed = m->seed;
    const int P = c.patch, G = c.image_size / P, np = G * G, seq = np + c.n_text;
    const int D = c.vit_hidden, F = c.vit_ffn, H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim;
    const int64_t Mv = (int64_t)batch * np, Md = (int64_t)batch * seq;
    int kmax = D;
    const int ks[4] = {F, c.conn_hidden, H, c.dec_ffn};
    for (int i = 0; i < 4; ++i) kmax = ks[i] > kmax ? ks[i] : kmax;
    int nmax = 3 * D;
    const int ns[5] = {F, c.conn_hidden, H + 2 * KV, c.dec_ffn, H};
    for (int i = 0; i < 5; ++i) nmax = ns[i] > nmax ? ns[i] : nmax;
    const int64_t Mmax = Md > Mv ? Md : Mv;
    q8buf qb;
    qb.q = (int8_t *)malloc((size_t)(Mmax * rup(kmax, QK)));
    qb.s = (float *)malloc(sizeof(float) * (size_t)Mmax);
    qb.sums = (int32_t *)malloc(sizeof(int32_t) * (size_t)Mmax);
    float *tmp_lin = (float *)malloc(sizeof(float) * (size_t)(Mmax * nmax));

    /* ---- patch embedding ---- */
    float *vx = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    {
        patch_ctx pc = {m, images, vx};
        orc_parallel_for(Mv, nth, patch_range, &pc);
    }

    /* ---- ViT ---- */
    float *vqkv = (float *)malloc(sizeof(float) * (size_t)(Mv * 3 * D));
    float *vattn = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    float *vh = (float *)malloc(sizeof(float) * (size_t)(Mv * F));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    const float vscale = 1.0f / sqrtf((float)(D / c.vit_heads));
    for (int l = 0; l < c.vit_layers; ++l) {
        const vit_layer *L = &m->vit[l];
        orc_layer_norm(vx, L->ln1_w, L->ln1_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&L->qkv, &qb, Mv, vqkv, 3 * D, L->qkv_b, 0, NULL, tmp_lin, nth);
        orc_attention(vqkv, 3 * D, 0, D, 2 * D, batch, c.vit_heads, c.vit_heads, D / c.vit_heads, np, 0, vscale,
                      vattn, D, nth);
        quant(vattn, Mv, D, &qb, nth);
        linear(&L->wo, &qb, Mv, vx, D, L->o_b, 0, vx, tmp_lin, nth);
        orc_layer_norm(vx, L->ln2_w, L->ln2_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&L->fc1, &qb, Mv, vh, F, L->fc1_b, 1, NULL, tmp_lin, nth);
        quant(vh, Mv, F, &qb, nth);
        linear(&L->fc2, &qb, Mv, vx, D, L->fc2_b, 0, vx, tmp_lin, nth);
    }

    /* ---- connector ---- */
    float *dx = (float *)malloc(sizeof(float) * (size_t)(Md * H));
    {
        float *ch = (float *)malloc(sizeof(float) * (size_t)(Mv * c.conn_hidden));
        float *co = (float *)malloc(sizeof(float) * (size_t)(Mv * H));
        orc_layer_norm(vx, m->post_w, m->post_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&m->c1, &qb, Mv, ch, c.conn_hidden, m->c1_b, 1, NULL, tmp_lin, nth);
        quant(ch, Mv, c.conn_hidden, &qb, nth);
        linear(&m->c2, &qb, Mv, co, H, m->c2_b, 0, NULL, tmp_lin, nth);
        for (int b = 0; b < batch; ++b)
            memcpy(dx + (int64_t)b * seq * H, co + (int64_t)b * np * H, sizeof(float) * (size_t)np * H);
        free(ch); free(co);
    }
    free(vqkv); free(vattn); free(vh); free(tmp); free(vx);

    /* ---- text tokens ---- */
    for (int b = 0; b < batch; ++b)
        for (int i = 0; i < c.n_text; ++i) {
            const uint32_t tok = (uint32_t)tokens[(int64_t)b * c.n_text + i];
            float *row = dx + ((int64_t)b * seq + np + i) * H;
            for (int col_i = 0; col_i < H; ++col_i)
                row[col_i] = -0.02f + 0.04f * unit24(orc_bv_param_bits(seed, 0x80000000u | tok, (uint32_t)col_i));
        }

    /* ---- decoder ---- */
    const int ldqkv = H + 2 * KV;
    float *dqkv = (float *)malloc(sizeof(float) * (size_t)(Md * ldqkv));
    float *dattn = (float *)malloc(sizeof(float) * (size_t)(Md * H));
    float *dg = (float *)malloc(sizeof(float) * (size_t)(Md * c.dec_ffn));
    float *du = (float *)malloc(sizeof(float) * (size_t)(Md * c.dec_ffn));
    float *dn = (float *)malloc(sizeof(float) * (size_t)(Md * (H > c.dec_ffn ? H : c.dec_ffn)));
    float *cs = (float *)malloc(sizeof(float) * (size_t)seq * (size_t)c.head_dim);
    orc_rope_table(c.rope_theta, c.head_dim, seq, cs);
    const float dscale = 1.0f / sqrtf((float)c.head_dim);
    for (int l = 0; l < c.dec_layers; ++l) {
        const dec_layer *L = &m->dec[l];
        orc_rms_norm(dx, L->attn_norm, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&L->qkv, &qb, Md, dqkv, ldqkv, NULL, 0, NULL, tmp_lin, nth);
        orc_rope_neox(dqkv, Md, c.dec_heads + c.dec_kv_heads, c.head_dim, ldqkv, cs, seq, 0);
        orc_attention(dqkv, ldqkv, 0, H, H + KV, batch, c.dec_heads, c.dec_kv_heads, c.head_dim, seq, 1, dscale, dattn,
                      H, nth);
        orc_rms_norm(dattn, L->attn_sub, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&L->wo, &qb, Md, dx, H, NULL, 0, dx, tmp_lin, nth);
        orc_rms_norm(dx, L->ffn_norm, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&L->gate, &qb, Md, dg, c.dec_ffn, NULL, 0, NULL, tmp_lin, nth);
        linear(&L->up, &qb, Md, du, c.dec_ffn, NULL, 0, NULL, tmp_lin, nth);
        orc_sqrelu_mul(dg, du, Md * c.dec_ffn, dg);
        orc_rms_norm(dg, L->ffn_sub, Md, c.dec_ffn, c.dec_eps, dn);
        quant(dn, Md, c.dec_ffn, &qb, nth);
        linear(&L->down, &qb, Md, dx, H, NULL, 0, dx, tmp_lin, nth);
    }
    float *hid = hidden ? hidden : (float *)malloc(sizeof(float) * (size_t)(Md * H));
    orc_rms_norm(dx, m->final_norm, Md, H, c.dec_eps, hid);

    /* ---- action head: lane l of a warp sums c = l, l + 32, ...; xor-butterfly; lane 0 + bias ---- */
    if (actions) {
        const int NA = c.action_chunk * c.action_dim;
        for (int b = 0; b < batch; ++b)
            for (int j = 0; j < NA; ++j) {
                const float *hr = hid + ((int64_t)b * seq + seq - 1) * H;
                float lanes[32], nxt[32];
                for (int ln = 0; ln < 32; ++ln) {
                    float acc = 0.0f;
                    for (int cc = ln; cc < H; cc += 32) acc = acc + hr[cc] * m->act_w[(int64_t)j * H + cc];
                    lanes[ln] = acc;
                }
                for (int off = 16; off > 0; off >>= 1) {
                    for (int ln = 0; ln < 32; ++ln) nxt[ln] = lanes[ln] + lanes[ln ^ off];
                    memcpy(lanes, nxt, sizeof(lanes));
                }
                actions[(int64_t)b * NA + j] = lanes[0] + m->act_b[j];
            }
    }
    if (!hidden) free(hid);
    free(cs); free(dqkv); free(dattn); free(dg); free(du); free(dn); free(dx); free(tmp_lin);
    free(qb.q); free(qb.s); free(qb.sums);
    return 0;
}

int orc_bitvla_forward(const b2s_bitvla_config *cfg, uint32_t seed, int batch, const float *images,
                       const int32_t *tokens, float *hidden, float *actions, int nth) {
    orc_bitvla_model *m = orc_bitvla_create(cfg, seed, nth);
    if (!m) return -1;
    const int rc = orc_bitvla_run(m, batch, images, tokens, hidden, actions, nth);
    orc_bitvla_free(m);
    return rc;
}
