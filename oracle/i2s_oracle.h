/*
 * i2s_oracle.h -- CPU restatement of the ternary i2_s mul_mat path (TEST INFRASTRUCTURE).
 *
 * This is the oracle: a scalar C restatement used only by tests/, by the smoke check and by the
 * CPU-baseline leg of bench.py. Nothing in the product library links, loads or calls it.
 *
 * What it restates, and from where:
 *   - The op contract of ggml_mul_mat(ctx, W, X): W ne=[K,N] (ne0 = in_features), X f32 ne=[K,M],
 *     Y f32 ne=[N,M], row-major per token. Reference call sites: src/models/smolvla/vision.cpp:314-343,
 *     src/models/pi0/vlm.cpp:217-240, src/models/smolvla/state_proj.cpp:55.
 *   - The i2_s tensor type and its CPU kernels live in microsoft/BitNet's fork of ggml
 *     (src/ggml-bitnet-mad.cpp: quantize_i2_s, quantize_row_i8_s, ggml_vec_dot_i2_i8_s; x86 block
 *     size QK_I2_S = 128). That fork is not vendored in the reference (third_party/llama.cpp is an
 *     empty submodule, .gitmodules:1-3) and no version of it can be pinned, so the published
 *     algorithm is restated here from its description. PARITY UNPINNED: the reference holds no
 *     i2_s golden vectors; the tests pin this restatement with hand-computed known answers.
 *   - RMSNorm follows ggml's CPU rms_norm (double accumulation of float squares, then
 *     scale = 1/sqrtf(mean + eps)) followed by ggml_mul with the norm weight, as used at
 *     src/models/smolvla/action_expert.cpp:731-736 and src/models/pi0/vlm.cpp:216.
 *   - Softmax follows ggml_soft_max_ext(x, mask, scale, 0.0f) as used at
 *     src/models/smolvla/action_expert.cpp:773, with a pinned fp32 evaluation: e = orc_det_expf(l - max)
 *     (Cody-Waite reduction + degree-7 Taylor polynomial, fused multiply-adds), the sum in the device's
 *     warp order (orc_warp_order_sum), p = e * (1/sum).
 *
 * i2_s byte layout ("layout v1", flattened over the whole tensor, n = N*K, n % 128 == 0):
 *   weight g = r*K + k (row r, column k) lives in block b = g/128 at position j = g%128;
 *   it is the 2-bit code in byte 32*b + (j%32) at bit shift 6 - 2*(j/32).
 *   code 0 -> -1, code 1 -> 0, code 2 -> +1 (decode t = code - 1).
 *   After the n/4 code bytes come 32 bytes whose first 4 hold the fp32 tensor scale.
 *   nbytes = n/4 + 32.
 * Row-padded device layout ("i2_s_r"): each row padded to Kp = roundup(K,128) weights with code 1,
 *   row r occupying bytes [r*Kp/4, (r+1)*Kp/4), same in-block interleave, scale at N*Kp/4.
 *   For K % 128 == 0 it is byte-identical to i2_s.
 *
 * Activation quantization (per token, "i8_s"): amax = max(1e-5, max_k |x_k|) in double;
 *   s = (float)(127/amax); q_k = clamp(round((double)(x_k*s)), -128, 127) with round() half away
 *   from zero and x_k*s an fp32 product; sum = sum_k q_k (int32).
 * Accumulator: acc[m,n] = sum_k q[m,k] * t[n,k] (exact int32).
 * Rescale: y[m,n] = (float)acc[m,n] * (w_scale / s[m]), the quotient an fp32 division done once per
 *   token. (The fork's CPU epilogue order is unpinned; any order differs by at most 1-2 ulp.)
 */
#ifndef B2S_I2S_ORACLE_H
#define B2S_I2S_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- i2_s type traits ---- */
size_t orc_i2s_nbytes(int64_t nrow, int64_t n_per_row);
size_t orc_i2s_r_nbytes(int64_t nrow, int64_t n_per_row);
/* Pack float weights (already ternary times a scale) into i2_s; returns bytes written (nbytes),
 * or 0 when nrow*n_per_row is not a multiple of 128 (the layout needs whole blocks). */
size_t orc_i2s_quantize(const float *src, uint8_t *dst, int64_t nrow, int64_t n_per_row);
/* Pack ternary int8 values {-1,0,1} with an explicit scale into i2_s. */
size_t orc_i2s_pack_ternary(const int8_t *t, float scale, uint8_t *dst, int64_t nrow, int64_t n_per_row);
/* Decode i2_s into ternary int8 (row-major N x K) and return the scale. */
float orc_i2s_unpack_ternary(const uint8_t *src, int8_t *t, int64_t nrow, int64_t n_per_row);
/* Dequantize i2_s to float (to_float trait): t * scale. */
void orc_i2s_dequantize(const uint8_t *src, float *dst, int64_t nrow, int64_t n_per_row);
/* Convert flattened i2_s to the row-padded i2_s_r layout. */
size_t orc_i2s_to_rowpadded(const uint8_t *src, uint8_t *dst, int64_t nrow, int64_t n_per_row);

/* ---- activation quantization ---- */
void orc_act_quant(const float *x, int64_t M, int64_t K, int8_t *q, float *s, int32_t *sums);

/* ---- integer GEMM and rescale ---- */
void orc_gemm_i32(const int8_t *t, const int8_t *q, int64_t M, int64_t N, int64_t K, int32_t *acc);
void orc_rescale(const int32_t *acc, const float *s, float w_scale, int64_t M, int64_t N, float *y);

/* Full op: Y[M,N] = i2s_mul_mat(W, X[M,K]) with X per-token quantized. */
void orc_mul_mat_i2s(const uint8_t *W, const float *X, int64_t M, int64_t N, int64_t K, float *Y);

/* ---- neighbours ---- */
/* y[m,k] = (x[m,k] * (1/sqrtf(mean_k x^2 + eps))) * g[k]   (g may be NULL: no weight) */
void orc_rms_norm(const float *x, const float *g, int64_t M, int64_t K, float eps, float *y);
/* p = (max(g,0)*max(g,0)) * u, elementwise */
void orc_sqrelu_mul(const float *g, const float *u, int64_t n, float *p);
/* y[m,:] = softmax(x[m,:]*scale + mask[m % mask_rows, :]) ; mask may be NULL */
void orc_soft_max_ext(const float *x, const float *mask, int64_t mask_rows, int64_t M, int64_t N,
                      float scale, float *y);

/* ---- FFN block: RMSNorm -> gate/up -> sqrelu(gate)*up -> RMSNorm -> down ---- */
void orc_ffn_block(const float *X, int64_t M, int64_t H, int64_t F,
                   const float *g_norm1, const float *g_norm2, float eps,
                   const uint8_t *W_gate, const uint8_t *W_up, const uint8_t *W_down,
                   float *Y, float *P_dbg);

/* ---- deterministic fp32 transcendental functions shared with the device kernels ---- */
float orc_det_expf(float x);
float orc_det_recipf(float d);
float orc_det_tanhf(float u);
float orc_warp_order_sum(const float *e, int64_t n);

/* ---- threaded SIMD variant of the integer path (timed CPU baseline only) ---- */
/* Same results, bit for bit, as orc_act_quant + orc_gemm_i32 + orc_rescale. */
void orc_fast_mul_mat_i2s(const uint8_t *W, const float *X, int64_t M, int64_t N, int64_t K, float *Y,
                          int nthreads);
void orc_fast_ffn_block(const float *X, int64_t M, int64_t H, int64_t F,
                        const float *g_norm1, const float *g_norm2, float eps,
                        const uint8_t *W_gate, const uint8_t *W_up, const uint8_t *W_down,
                        float *Y, int nthreads);
int orc_fast_isa(void); /* 2 = AVX512-VNNI, 1 = AVX2, 0 = scalar */
/* Y[m][n] (row stride ldy) = (float)(acc - sums[m]) * (ws_n / s[m]) from row-padded codes Wr (Kp/4 bytes
 * per row) and pre-quantized activations q [M][Kp] (zero-padded past K); ws_n = tile_scales[n/128]. */
void orc_fast_gemm_q8_rp(const uint8_t *Wr, const float *tile_scales, int64_t N, int64_t K, const int8_t *q,
                         const float *s, const int32_t *sums, int64_t M, float *Y, int64_t ldy, int nthreads);
/* orc_act_quant of M rows of K floats into q [M][Kp] (zero-padded), s [M], sums [M]. */
void orc_fast_act_quant_padded(const float *X, int64_t M, int64_t K, int8_t *q, float *s, int32_t *sums,
                               int nthreads);
/* Static parallel-for over [0, n) on nthreads pthreads. */
void orc_parallel_for(int64_t n, int nthreads, void (*fn)(void *ctx, int64_t begin, int64_t end), void *ctx);

#ifdef __cplusplus
}
#endif
#endif
