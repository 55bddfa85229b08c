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

/* y = W q (+ bias) (GELU if act) (+ residual, res may alias y): the device epilogue order. */
static void linear(const tern_w *w, const q8buf *qb, int64_t M, float *y, int64_t ldy, const float *bias, int act,
                   const float *res, int nth) {
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(M * w->N));
    orc_fast_gemm_q8_rp(w->codes, w->tiles, w->N, w->K, qb->q, qb->s, qb->sums, M, tmp, w->N, nth);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < w->N; ++n) {
            float v = tmp[m * w->N + n];
            if (bias) v = v + bias[n];
            if (act == 1) v = orc_gelu_tanh(v);
            if (res) v = res[m * ldy + n] + v;
            y[m * ldy + n] = v;
        }
    free(tmp);
}

/* ---------------------------------------------------------------- forward */
int orc_bitvla_forward(const b2s_bitvla_config *cfg, uint32_t seed, int batch, const float *images,
                       const int32_t *tokens, float *hidden, float *actions, int nth) {
    const b2s_bitvla_config c = *cfg;
    const int P = c.patch, G = c.image_size / P, np = G * G, seq = np + c.n_text;
    const int D = c.vit_hidden, F = c.vit_ffn, H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim;
    const int64_t Mv = (int64_t)batch * np, Md = (int64_t)batch * seq;
    int kmax = D;
    const int ks[4] = {F, c.conn_hidden, H, c.dec_ffn};
    for (int i = 0; i < 4; ++i) kmax = ks[i] > kmax ? ks[i] : kmax;
    const int64_t Mmax = Md > Mv ? Md : Mv;
    q8buf qb;
    qb.q = (int8_t *)malloc((size_t)(Mmax * rup(kmax, QK)));
    qb.s = (float *)malloc(sizeof(float) * (size_t)Mmax);
    qb.sums = (int32_t *)malloc(sizeof(int32_t) * (size_t)Mmax);

    /* ---- patch embedding: y = (bias + pos) + acc, acc = fmaf(col[k], w[d][k], acc), k ascending ---- */
    const int kdim = 3 * P * P;
    const float pa = 1.0f / sqrtf((float)kdim);
    float *patch_w = uniform_new((int64_t)D * kdim, seed, 1, -pa, pa);
    float *patch_b = uniform_new(D, seed, 2, -0.02f, 0.02f);
    float *pos = uniform_new((int64_t)np * D, seed, 3, -0.02f, 0.02f);
    float *vx = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    float *col = (float *)malloc(sizeof(float) * (size_t)kdim);
    for (int b = 0; b < batch; ++b)
        for (int p = 0; p < np; ++p) {
            const int py = p / G, px = p % G;
            for (int k = 0; k < kdim; ++k) {
                const int ch = k / (P * P), ky = (k / P) % P, kx = k % P;
                col[k] = images[(((int64_t)b * 3 + ch) * c.image_size + (py * P + ky)) * c.image_size + (px * P + kx)];
            }
            for (int d = 0; d < D; ++d) {
                float acc = 0.0f;
                for (int k = 0; k < kdim; ++k) acc = fmaf(col[k], patch_w[(int64_t)d * kdim + k], acc);
                const float pre = patch_b[d] + pos[(int64_t)p * D + d];
                vx[((int64_t)b * np + p) * D + d] = pre + acc;
            }
        }
    free(col); free(patch_w); free(patch_b); free(pos);

    /* ---- ViT ---- */
    float *vqkv = (float *)malloc(sizeof(float) * (size_t)(Mv * 3 * D));
    float *vattn = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    float *vh = (float *)malloc(sizeof(float) * (size_t)(Mv * F));
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(Mv * D));
    const float vscale = 1.0f / sqrtf((float)(D / c.vit_heads));
    for (int l = 0; l < c.vit_layers; ++l) {
        const uint32_t base = 0x100u + 16u * (uint32_t)l;
        float *ln1_w = uniform_new(D, seed, base + 0, 0.9f, 1.1f), *ln1_b = uniform_new(D, seed, base + 1, -0.02f, 0.02f);
        const int64_t rows3[3] = {D, D, D};
        const uint32_t ids3[3] = {base + 2, base + 3, base + 4};
        tern_w qkv = make_tern(3, rows3, ids3, D, seed, nth);
        float *qkv_b = (float *)malloc(sizeof(float) * 3 * (size_t)D);
        for (int j = 0; j < 3; ++j) orc_bv_gen_uniform(qkv_b + j * D, D, seed, base + 5 + j, -0.02f, 0.02f);
        tern_w wo = make_tern1(D, base + 8, D, seed, nth);
        float *o_b = uniform_new(D, seed, base + 9, -0.02f, 0.02f);
        float *ln2_w = uniform_new(D, seed, base + 10, 0.9f, 1.1f), *ln2_b = uniform_new(D, seed, base + 11, -0.02f, 0.02f);
        tern_w fc1 = make_tern1(F, base + 12, D, seed, nth);
        float *fc1_b = uniform_new(F, seed, base + 13, -0.02f, 0.02f);
        tern_w fc2 = make_tern1(D, base + 14, F, seed, nth);
        float *fc2_b = uniform_new(D, seed, base + 15, -0.02f, 0.02f);

        orc_layer_norm(vx, ln1_w, ln1_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&qkv, &qb, Mv, vqkv, 3 * D, qkv_b, 0, NULL, nth);
        orc_attention(vqkv, 3 * D, 0, D, 2 * D, batch, c.vit_heads, c.vit_heads, D / c.vit_heads, np, 0, vscale,
                      vattn, D, nth);
        quant(vattn, Mv, D, &qb, nth);
        linear(&wo, &qb, Mv, vx, D, o_b, 0, vx, nth);
        orc_layer_norm(vx, ln2_w, ln2_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&fc1, &qb, Mv, vh, F, fc1_b, 1, NULL, nth);
        quant(vh, Mv, F, &qb, nth);
        linear(&fc2, &qb, Mv, vx, D, fc2_b, 0, vx, nth);

        free(ln1_w); free(ln1_b); free(qkv_b); free(o_b); free(ln2_w); free(ln2_b); free(fc1_b); free(fc2_b);
        free_tern(&qkv); free_tern(&wo); free_tern(&fc1); free_tern(&fc2);
    }

    /* ---- connector ---- */
    float *dx = (float *)malloc(sizeof(float) * (size_t)(Md * H));
    {
        float *post_w = uniform_new(D, seed, 4, 0.9f, 1.1f), *post_b = uniform_new(D, seed, 5, -0.02f, 0.02f);
        tern_w c1 = make_tern1(c.conn_hidden, 6, D, seed, nth);
        float *c1_b = uniform_new(c.conn_hidden, seed, 7, -0.02f, 0.02f);
        tern_w c2 = make_tern1(H, 8, c.conn_hidden, seed, nth);
        float *c2_b = uniform_new(H, seed, 9, -0.02f, 0.02f);
        float *ch = (float *)malloc(sizeof(float) * (size_t)(Mv * c.conn_hidden));
        float *co = (float *)malloc(sizeof(float) * (size_t)(Mv * H));
        orc_layer_norm(vx, post_w, post_b, Mv, D, c.vit_eps, tmp);
        quant(tmp, Mv, D, &qb, nth);
        linear(&c1, &qb, Mv, ch, c.conn_hidden, c1_b, 1, NULL, nth);
        quant(ch, Mv, c.conn_hidden, &qb, nth);
        linear(&c2, &qb, Mv, co, H, c2_b, 0, NULL, nth);
        for (int b = 0; b < batch; ++b)
            memcpy(dx + (int64_t)b * seq * H, co + (int64_t)b * np * H, sizeof(float) * (size_t)np * H);
        free(post_w); free(post_b); free(c1_b); free(c2_b); free(ch); free(co);
        free_tern(&c1); free_tern(&c2);
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
        const uint32_t base = 0x10000u + 16u * (uint32_t)l;
        float *attn_norm = uniform_new(H, seed, base + 0, 0.9f, 1.1f);
        const int64_t rows3[3] = {H, KV, KV};
        const uint32_t ids3[3] = {base + 1, base + 2, base + 3};
        tern_w qkv = make_tern(3, rows3, ids3, H, seed, nth);
        float *attn_sub = uniform_new(H, seed, base + 4, 0.9f, 1.1f);
        tern_w wo = make_tern1(H, base + 5, H, seed, nth);
        float *ffn_norm = uniform_new(H, seed, base + 6, 0.9f, 1.1f);
        tern_w gate = make_tern1(c.dec_ffn, base + 7, H, seed, nth);
        tern_w up = make_tern1(c.dec_ffn, base + 8, H, seed, nth);
        float *ffn_sub = uniform_new(c.dec_ffn, seed, base + 9, 0.9f, 1.1f);
        tern_w down = make_tern1(H, base + 10, c.dec_ffn, seed, nth);

        orc_rms_norm(dx, attn_norm, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&qkv, &qb, Md, dqkv, ldqkv, NULL, 0, NULL, nth);
        orc_rope_neox(dqkv, Md, c.dec_heads + c.dec_kv_heads, c.head_dim, ldqkv, cs, seq, 0);
        orc_attention(dqkv, ldqkv, 0, H, H + KV, batch, c.dec_heads, c.dec_kv_heads, c.head_dim, seq, 1, dscale, dattn,
                      H, nth);
        orc_rms_norm(dattn, attn_sub, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&wo, &qb, Md, dx, H, NULL, 0, dx, nth);
        orc_rms_norm(dx, ffn_norm, Md, H, c.dec_eps, dn);
        quant(dn, Md, H, &qb, nth);
        linear(&gate, &qb, Md, dg, c.dec_ffn, NULL, 0, NULL, nth);
        linear(&up, &qb, Md, du, c.dec_ffn, NULL, 0, NULL, nth);
        orc_sqrelu_mul(dg, du, Md * c.dec_ffn, dg);
        orc_rms_norm(dg, ffn_sub, Md, c.dec_ffn, c.dec_eps, dn);
        quant(dn, Md, c.dec_ffn, &qb, nth);
        linear(&down, &qb, Md, dx, H, NULL, 0, dx, nth);

        free(attn_norm); free(attn_sub); free(ffn_norm); free(ffn_sub);
        free_tern(&qkv); free_tern(&wo); free_tern(&gate); free_tern(&up); free_tern(&down);
    }
    float *fn = uniform_new(H, seed, 10, 0.9f, 1.1f);
    float *hid = hidden ? hidden : (float *)malloc(sizeof(float) * (size_t)(Md * H));
    orc_rms_norm(dx, fn, Md, H, c.dec_eps, hid);

    /* ---- action head: lane l of a warp sums c = l, l + 32, ...; xor-butterfly; lane 0 + bias ---- */
    if (actions) {
        const int NA = c.action_chunk * c.action_dim;
        const float aa = 1.0f / sqrtf((float)H);
        float *aw = uniform_new((int64_t)NA * H, seed, 11, -aa, aa);
        float *ab = uniform_new(NA, seed, 12, -0.02f, 0.02f);
        for (int b = 0; b < batch; ++b)
            for (int j = 0; j < NA; ++j) {
                const float *hr = hid + ((int64_t)b * seq + seq - 1) * H;
                float lanes[32], nxt[32];
                for (int ln = 0; ln < 32; ++ln) {
                    float acc = 0.0f;
                    for (int cc = ln; cc < H; cc += 32) acc = acc + hr[cc] * aw[(int64_t)j * H + cc];
                    lanes[ln] = acc;
                }
                for (int off = 16; off > 0; off >>= 1) {
                    for (int ln = 0; ln < 32; ++ln) nxt[ln] = lanes[ln] + lanes[ln ^ off];
                    memcpy(lanes, nxt, sizeof(lanes));
                }
                actions[(int64_t)b * NA + j] = lanes[0] + ab[j];
            }
        free(aw); free(ab);
    }
    if (!hidden) free(hid);
    free(fn); free(cs); free(dqkv); free(dattn); free(dg); free(du); free(dn); free(dx);
    free(qb.q); free(qb.s); free(qb.sums);
    return 0;
}
