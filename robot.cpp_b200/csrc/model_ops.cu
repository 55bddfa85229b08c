// model_ops.cu -- the non-i2_s operators of a BitVLA-shape forward around the i2_s mul_mats.
//
//   * norm_kernel: ggml_norm (LayerNorm) / ggml_rms_norm followed by ggml_mul(weight) and ggml_add(bias),
//     written as fp32 (the ViT post-norm and the decoder's output norm), or as per-token int8 through the
//     act-quant semantics (LayerNorm + act-quant feeding a ternary GEMM). ggml's CPU norms accumulate in
//     double: mean = (float)(sum x / K); v = x - mean; var = (float)(sum v^2 / K);
//     scale = 1/sqrtf(var + eps); y = ((v * scale) * w) + b (src/models/smolvla/vision.cpp:314 pattern).
//   * rope kernels: ggml_rope_ext in NEOX mode (src/models/pi0/vlm.cpp:223-235): for position p and
//     pair (i, i + d/2), theta = p * base^(-2i/d), (x0, x1) -> (x0 cos - x1 sin, x0 sin + x1 cos); the
//     angles in double, either per element or from a per-model table.
//   * attention: one fused fp32 kernel per (query block, head, sequence) -- scores, online softmax, P V -- the
//     ggml graph mul_mat(K, Q) -> soft_max_ext -> mul_mat(V, KQ) of
//     src/models/smolvla/action_expert.cpp:771-774, with grouped K/V heads (GQA) as in
//     src/models/pi0/vlm.cpp:223-235, in a fixed operation order the CPU oracle repeats bit for bit; head
//     dims 128 and 72 use a 128-thread wide-tile form that prefetches the next key chunk, and all forms
//     issue their fma chains as paired fp32 instructions (fma.rn.f32x2: two independent IEEE fmas).
//   * patch embedding (fp32 tile GEMM reading the patches straight from the image, onto bias + position
//     embedding) and a hash-seeded token-embedding gather for random-init vocabularies (the 128256 x 2560
//     table is never materialized).
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

// ------------------------------------------------------------------------------------------------ norms
constexpr int kNormThreads = 256;

__device__ __forceinline__ double block_sum_dbl(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double w = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0.0;
        w = warp_sum_d(w);
        if (lane == 0) red[0] = w;
    }
    __syncthreads();
    return red[0];
}
__device__ __forceinline__ float block_max_f(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float w = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0.0f;
        w = warp_max(w);
        if (lane == 0) red[0] = w;
    }
    __syncthreads();
    return red[0];
}
__device__ __forceinline__ int block_sum_int(int v, int* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_i(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int w = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0;
        w = warp_sum_i(w);
        if (lane == 0) red[0] = w;
    }
    __syncthreads();
    return red[0];
}

// KIND 0: RMSNorm, 1: LayerNorm. QUANT: write int8 codes + scale + sum instead of fp32.
template <int KIND, bool QUANT>
__global__ void __launch_bounds__(kNormThreads)
norm_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ g, const float* __restrict__ b,
            float eps, int K, float* __restrict__ y, int64_t ldy, int8_t* __restrict__ q, int64_t ldq,
            float* __restrict__ s_out, int32_t* __restrict__ sum_out) {
    __shared__ double red[32];
    const int64_t m = blockIdx.x;
    const float* xr = x + m * ldx;
    griddep_wait();
    griddep_launch();
    float mean = 0.0f;
    if (KIND == 1) {
        double acc = 0.0;
        for (int i = threadIdx.x; i < K; i += blockDim.x) acc += (double)xr[i];
        mean = (float)(block_sum_dbl(acc, red) / (double)K);
    }
    double acc2 = 0.0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = (KIND == 1) ? __fsub_rn(xr[i], mean) : xr[i];
        acc2 += (double)__fmul_rn(v, v);
    }
    const float var = (float)(block_sum_dbl(acc2, red) / (double)K);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    auto val = [&](int i) -> float {
        float v = (KIND == 1) ? __fsub_rn(xr[i], mean) : xr[i];
        v = __fmul_rn(v, scale);
        if (g) v = __fmul_rn(v, g[i]);
        if (b) v = __fadd_rn(v, b[i]);
        return v;
    };
    if (!QUANT) {
        for (int i = threadIdx.x; i < K; i += blockDim.x) y[m * ldy + i] = val(i);
        return;
    }
    float amax = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(val(i)));
    amax = block_max_f(amax, reinterpret_cast<float*>(red));
    const float s = actq_scale(amax);
    int sum = 0;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const int a = actq_round(val(i), s);
        q[m * ldq + i] = (int8_t)a;
        sum += a;
    }
    sum = block_sum_int(sum, reinterpret_cast<int*>(red));
    if (threadIdx.x == 0) {
        s_out[m] = s;
        if (sum_out) sum_out[m] = sum;
    }
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

cudaError_t launch_norm(int kind, bool quant, const float* x, int64_t ldx, const float* g, const float* b, float eps,
                        int64_t M, int64_t K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                        cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    if (rowq_eligible(x, ldx, g, b, K, quant ? static_cast<const void*>(q) : static_cast<const void*>(y),
                      quant ? ldq : ldy, quant))
        return launch_rowq(kind, quant, x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st);
    const dim3 grid((unsigned)M), block(kNormThreads);
    const int k = (int)K;
    if (kind == 0) {
        if (quant) return launch_pdl(norm_kernel<0, true>, grid, block, st, x, ldx, g, b, eps, k, y, ldy, q, ldq, s, sums);
        return launch_pdl(norm_kernel<0, false>, grid, block, st, x, ldx, g, b, eps, k, y, ldy, q, ldq, s, sums);
    }
    if (quant) return launch_pdl(norm_kernel<1, true>, grid, block, st, x, ldx, g, b, eps, k, y, ldy, q, ldq, s, sums);
    return launch_pdl(norm_kernel<1, false>, grid, block, st, x, ldx, g, b, eps, k, y, ldy, q, ldq, s, sums);
}

// ------------------------------------------------------------------------------------------------ RoPE
// Angles in double, rounded once to fp32: inv_freq = base^(-2i/d), theta = p * inv_freq,
// (cos, sin) = ((float)cos(theta), (float)sin(theta)); then x0' = x0 c - x1 s, x1' = x0 s + x1 c in fp32.
__device__ __forceinline__ float2 rope_cs(float base, int hd, int pos, int i) {
    const double inv = pow((double)base, -2.0 * (double)i / (double)hd);
    const double th = (double)pos * inv;
    return make_float2((float)cos(th), (float)sin(th));
}
__device__ __forceinline__ void rope_rotate(float* r, int i, int half, float2 cs) {
    const float x0 = r[i], x1 = r[i + half];
    r[i] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    r[i + half] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
}

// One thread per (token, head, pair), angles computed in place.
__global__ void rope_neox_kernel(float* __restrict__ x, int M, int n_heads, int hd, int64_t ld, float base,
                                 int pos0) {
    griddep_wait();
    griddep_launch();
    const int half = hd / 2;
    const int64_t total = (int64_t)M * n_heads * half;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e % half);
        const int h = (int)((e / half) % n_heads);
        const int m = (int)(e / ((int64_t)half * n_heads));
        rope_rotate(x + (int64_t)m * ld + (int64_t)h * hd, i, half, rope_cs(base, hd, pos0 + m, i));
    }
}

cudaError_t launch_rope_neox(float* x, int64_t M, int n_heads, int hd, int64_t ld, float base, int pos0,
                             cudaStream_t st) {
    const int64_t total = M * n_heads * (hd / 2);
    if (total <= 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
    return launch_pdl(rope_neox_kernel, dim3(blocks), dim3(256), st, x, (int)M, n_heads, hd, ld, base, pos0);
}

// The (cos, sin) table [n_pos][hd/2] of the same angles, built once per model.
__global__ void rope_table_kernel(float base, int hd, int n_pos, float2* __restrict__ tab) {
    const int half = hd / 2;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_pos * half; e += gridDim.x * blockDim.x)
        tab[e] = rope_cs(base, hd, e / half, e % half);
}
cudaError_t launch_rope_table(float base, int hd, int n_pos, float2* tab, cudaStream_t st) {
    rope_table_kernel<<<(n_pos * (hd / 2) + 255) / 256, 256, 0, st>>>(base, hd, n_pos, tab);
    return cudaGetLastError();
}

// Rotation from the table; row m is position m % period (sequences of `period` tokens stacked). Grid
// (pair blocks of a row, rows): each thread rotates one (head, i) pair of row blockIdx.y, with 32-bit index
// arithmetic (a grid-stride loop that split a 64-bit element index with three divisions per element was
// bound by those divisions).
__global__ void rope_apply_kernel(float* __restrict__ x, int M, int n_heads, int hd, int64_t ld,
                                  const float2* __restrict__ tab, int period, int m0) {
    griddep_wait();
    griddep_launch();
    const int half = hd / 2;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;  // pair index within the row
    const int m = m0 + (int)blockIdx.y;
    if (j >= n_heads * half || m >= M) return;
    const int h = j / half, i = j - h * half;
    rope_rotate(x + (int64_t)m * ld + (int64_t)h * hd, i, half, tab[(m % period) * half + i]);
}
cudaError_t launch_rope_apply(float* x, int64_t M, int n_heads, int hd, int64_t ld, const float2* tab, int period,
                              cudaStream_t st) {
    const int64_t pairs = (int64_t)n_heads * (hd / 2);
    if (M <= 0 || pairs <= 0) return cudaSuccess;
    for (int64_t m0 = 0; m0 < M; m0 += 65535) {  // grid y is at most 65535 rows per launch
        const int64_t rows = (M - m0) < 65535 ? (M - m0) : 65535;
        cudaError_t e = launch_pdl(rope_apply_kernel, dim3((unsigned)ceil_div(pairs, 256), (unsigned)rows), dim3(256),
                                   st, x, (int)M, n_heads, hd, ld, tab, period, (int)m0);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ------------------------------------------------------------------------------------------------ embeddings
static unsigned grid_for(int64_t total) {
    const int64_t b = (total + 255) / 256;
    return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

// Patch embedding of stacked CHW images ([batch][C][H][W]; patch rows of image b follow those of b - 1):
// Y[r][d] = (bias[d] + pos[r % np][d]) + acc, acc = fma(A[r][k], W[d][k], acc) over k = 0..C*P*P-1 in
// order from +0, with A the non-overlapping patch rows (k = c P^2 + ky P + kx) read straight from the
// image. A 64 x 64 output tile per CTA, 4 x 4 per thread, k staged 32 at a time; the image offset of each
// patch element k comes from a per-CTA table and each thread's patch row base is computed once, so staging
// costs one load per element; the fma chains run as paired fp32 instructions (same results).
constexpr int kPeTile = 64, kPeK = 32, kPeMaxK = 1024;
__global__ void __launch_bounds__(256)
patch_embed_kernel(const float* __restrict__ img, int batch, int C, int H, int W, int P, const float* __restrict__ w,
                   const float* __restrict__ bias, const float* __restrict__ pos, int D, float* __restrict__ y,
                   int64_t ldy) {
    __shared__ __align__(16) float As[kPeK][kPeTile];  // [k][patch row]
    __shared__ __align__(16) float Ws[kPeK][kPeTile];  // [k][output column]
    __shared__ int koff[kPeMaxK];                      // image offset of patch element k (channel, row, column)
    const int gw = W / P, np = (H / P) * gw, kdim = C * P * P, rows = batch * np;
    const int r0 = blockIdx.x * kPeTile, d0 = blockIdx.y * kPeTile;
    const int t = threadIdx.x, ty = t / 16, tx = t % 16;
    for (int k = t; k < kdim; k += 256) koff[k] = ((k / (P * P)) * H + (k / P) % P) * W + k % P;
    // Every staging pass has this thread write column i_s of As and Ws: one patch row, one weight row.
    const int i_s = t % kPeTile, kk0 = t / kPeTile;
    int64_t rbase = -1;
    if (r0 + i_s < rows) {
        const int r = r0 + i_s, bi = r / np, p = r % np, py = p / gw, px = p % gw;
        rbase = ((int64_t)bi * C * H + (int64_t)py * P) * W + (int64_t)px * P;
    }
    const float* wrow = (d0 + i_s < D) ? w + (int64_t)(d0 + i_s) * kdim : nullptr;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    __syncthreads();  // koff written
    for (int k0 = 0; k0 < kdim; k0 += kPeK) {
#pragma unroll
        for (int kk = kk0; kk < kPeK; kk += 256 / kPeTile) {
            const int k = k0 + kk;
            float a = 0.0f, b = 0.0f;
            if (k < kdim) {
                if (rbase >= 0) a = img[rbase + koff[k]];
                if (wrow) b = wrow[k];
            }
            As[kk][i_s] = a;
            Ws[kk][i_s] = b;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kPeK; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&As[kk][4 * ty]);
            const float4 b = *reinterpret_cast<const float4*>(&Ws[kk][4 * tx]);
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // row pairs: the patch load holds them side by side
                ffma2(acc[0][j], acc[1][j], a.x, a.y, bv[j], bv[j]);
                ffma2(acc[2][j], acc[3][j], a.z, a.w, bv[j], bv[j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = r0 + 4 * ty + i;
        if (r >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = d0 + 4 * tx + j;
            if (d >= D) continue;
            float pre = bias ? bias[d] : 0.0f;
            if (pos) pre = __fadd_rn(pre, pos[(int64_t)(r % np) * D + d]);
            y[(int64_t)r * ldy + d] = __fadd_rn(pre, acc[i][j]);
        }
    }
}

cudaError_t launch_patch_embed(const float* img, int batch, int C, int H, int W, int P, const float* w,
                               const float* bias, const float* pos, int D, float* y, int64_t ldy, cudaStream_t st) {
    const int rows = batch * (H / P) * (W / P);
    if (C * P * P > kPeMaxK) return cudaErrorInvalidValue;  // the per-CTA offset table holds 1024 patch elements
    const dim3 grid((unsigned)ceil_div(rows, kPeTile), (unsigned)ceil_div(D, kPeTile));
    patch_embed_kernel<<<grid, 256, 0, st>>>(img, batch, C, H, W, P, w, bias, pos, D, y, ldy);
    return cudaGetLastError();
}

// Random-init embedding row of token t, column c: the parameter generator of the BitVLA engine
// (tensor 0x80000000 | t, element c) mapped to U(-0.02, 0.02) with exact fp32 steps.
__device__ __forceinline__ float hash_embedding(uint32_t seed, uint32_t t, uint32_t c) {
    const float u = (float)(param_bits(seed, 0x80000000u | t, c) >> 8) * (1.0f / 16777216.0f);
    return __fadd_rn(-0.02f, __fmul_rn(0.04f, u));
}
__global__ void embed_tokens_kernel(const int32_t* __restrict__ tokens, int n, int D, uint32_t seed,
                                    float* __restrict__ y, int64_t ldy) {
    const int64_t total = (int64_t)n * D;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e / D), c = (int)(e % D);
        y[(int64_t)i * ldy + c] = hash_embedding(seed, (uint32_t)tokens[i], (uint32_t)c);
    }
}

cudaError_t launch_embed_tokens(const int32_t* tokens, int n, int D, uint32_t seed, float* y, int64_t ldy,
                                cudaStream_t st) {
    embed_tokens_kernel<<<grid_for((int64_t)n * D), 256, 0, st>>>(tokens, n, D, seed, y, ldy);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ attention
// softmax(Q K^T * scale [+ causal mask]) V for `batch` sequences of T tokens (sequence b at rows
// [b T, (b+1) T) of every operand), one CTA per (64-query block, head, sequence), two CTAs per SM.
// Keys are visited in chunks of 64 (chunk c = keys [64c, 64c + 64)) with an online softmax, in a fixed
// fp32 operation order that the CPU oracle repeats exactly. For query row i (n_i = i + 1 keys if causal,
// else T; keys j >= n_i count as masked):
//   s_j  = fp32(acc * scale), acc = fma(q[i][d], k[j][d], acc) over d = 0..hd-1 from +0; masked: -inf
//   per chunk: m' = max(m, max_j s_j);  alpha = det_expf(m - m');  p_j = det_expf(s_j - m')
//              csum = xor-butterfly (offsets 8, 4, 2, 1) over the 16 partial sums
//                     ((p_4t + p_4t+1) + p_4t+2) + p_4t+3, t = 0..15
//              l = l * alpha + csum;  o[d] = o[d] * alpha, then o[d] = fma(p_j, v[j][d], o[d]) for the
//              chunk's keys in ascending order
//   (m starts at -inf, l and o at +0); finally out[d] = o[d] * (1 / l). A chunk where the row has no
// key leaves l and o unchanged (alpha = 1, p = 0), so each row's result depends only on its own keys.
// Query head h reads K/V head h / (heads / kv_heads) (GQA). Shared memory: Q^T [hd][64], one K^T or V
// chunk, the 64 x 64 probability tile and per-row factors; hd % 8 == 0, hd <= 128.
constexpr int kAtQ = 64, kAtThreads = 256, kAtPP = kAtQ + 4;  // P row stride (floats)

size_t attention_smem_bytes(int /*T*/, int hd) {
    return sizeof(float) * ((size_t)hd * kAtQ * 2 + (size_t)kAtQ * kAtPP + 2 * kAtQ);
}

// Rows r0 .. r0 + 63 of one head (hd floats at src + r ldsrc; rows >= T read as zero) into dst[d][64]. With
// a rotation table (rows are positions 0 .. T-1 of their sequence) each (d, d + hd/2) pair is rotated on the
// way in, by the same fp32 operations as rope_rotate, so Q and K arrive exactly as a separate NEOX RoPE pass
// would have left them.
// With src2 the tile holds two half-tiles: columns 0-31 rows r0 .. r0 + 31 of src, columns 32-63 the same
// rows of src2 (another head of the same sequence).
__device__ __forceinline__ void stage_transposed(float* __restrict__ dst, const float* __restrict__ src,
                                                 int64_t ldsrc, int r0, int T, int hd,
                                                 const float2* __restrict__ rope,
                                                 const float* __restrict__ src2 = nullptr) {
    const int half = hd / 2, h4 = half / 4;
    for (int e = threadIdx.x; e < kAtQ * h4; e += blockDim.x) {
        const int i = e % kAtQ, d4 = 4 * (e / kAtQ);
        const int r = r0 + (src2 ? (i & 31) : i);  // position in the sequence
        const float* base = (src2 && i >= 32) ? src2 : src;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (r < T) {
            const float* row = base + (int64_t)r * ldsrc;
            a = *reinterpret_cast<const float4*>(row + d4);
            b = *reinterpret_cast<const float4*>(row + half + d4);
            if (rope) {
                const float4* cs = reinterpret_cast<const float4*>(rope + (int64_t)r * half + d4);
                const float4 c01 = cs[0], c23 = cs[1];  // (cos, sin) of pairs d4 .. d4 + 3
                const float x0[4] = {a.x, a.y, a.z, a.w}, x1[4] = {b.x, b.y, b.z, b.w};
                const float cv[4] = {c01.x, c01.z, c23.x, c23.z}, sv[4] = {c01.y, c01.w, c23.y, c23.w};
                float y0[4], y1[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    y0[c] = __fsub_rn(__fmul_rn(x0[c], cv[c]), __fmul_rn(x1[c], sv[c]));
                    y1[c] = __fadd_rn(__fmul_rn(x0[c], sv[c]), __fmul_rn(x1[c], cv[c]));
                }
                a = make_float4(y0[0], y0[1], y0[2], y0[3]);
                b = make_float4(y1[0], y1[1], y1[2], y1[3]);
            }
        }
        dst[(d4 + 0) * kAtQ + i] = a.x;
        dst[(d4 + 1) * kAtQ + i] = a.y;
        dst[(d4 + 2) * kAtQ + i] = a.z;
        dst[(d4 + 3) * kAtQ + i] = a.w;
        dst[(half + d4 + 0) * kAtQ + i] = b.x;
        dst[(half + d4 + 1) * kAtQ + i] = b.y;
        dst[(half + d4 + 2) * kAtQ + i] = b.z;
        dst[(half + d4 + 3) * kAtQ + i] = b.w;
    }
}

__global__ void __launch_bounds__(kAtThreads, 2)
attention_kernel(const float* __restrict__ q, int64_t ldq, const float* __restrict__ k, int64_t ldk,
                 const float* __restrict__ v, int64_t ldv, float* __restrict__ o, int64_t ldo, int T, int heads,
                 int kv_heads, int hd, float scale, int causal, const float2* __restrict__ rope) {
    extern __shared__ __align__(16) float at_sm[];
    float* Qt = at_sm;                 // [hd][64]
    float* KV = Qt + hd * kAtQ;        // K^T chunk [hd][64] or V chunk [64][hd]
    float* P = KV + hd * kAtQ;         // [64][kAtPP] probabilities of the chunk
    float* alpha_sm = P + kAtQ * kAtPP;   // [64] per-row rescale of the chunk
    float* inv_sm = alpha_sm + kAtQ;      // [64] 1 / l at the end
    // Grid (heads, batch, query blocks) with the last query block first: under a causal mask block b
    // visits b + 1 key chunks, so launching the heaviest blocks first shortens the grid's tail.
    const int h = blockIdx.x, g = h / (heads / kv_heads);
    const int q0 = (int)(gridDim.z - 1u - blockIdx.z) * kAtQ;
    const int64_t row0 = (int64_t)blockIdx.y * T;
    const float* qh = q + row0 * ldq + (int64_t)h * hd;
    const float* kh = k + row0 * ldk + (int64_t)g * hd;
    const float* vh = v + row0 * ldv + (int64_t)g * hd;
    const int t = threadIdx.x;
    const int hd4 = hd / 4;
    griddep_wait();  // q/k/v are written by the preceding kernel
    griddep_launch();

    stage_transposed(Qt, qh, ldq, q0, T, hd, rope);
    const int kend = causal ? min(T, q0 + kAtQ) : T;  // keys any query of this block can see
    const int nchunks = (kend + kAtQ - 1) / kAtQ;

    // score threads: rows 4 ty .. 4 ty + 3, keys 4 tx .. 4 tx + 3 of the chunk (the 16 tx of a row are
    // 16 consecutive lanes of one warp)
    const int ty = t / 16, tx = t % 16;
    float m_r[4], l_r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m_r[i] = -INFINITY;
        l_r[i] = 0.0f;
    }
    // output threads: rows 4 rg .. 4 rg + 3, columns 8 cg .. 8 cg + 7
    const int ncg = hd / 8;
    const bool active = t < 16 * ncg;
    const int rg = active ? t / ncg : 0, cg = active ? t % ncg : 0;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    for (int c = 0; c < nchunks; ++c) {
        const int k0 = c * kAtQ;
        __syncthreads();  // Qt written; the previous chunk's V and P reads are done
        stage_transposed(KV, kh, ldk, k0, T, hd, rope);
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < hd; ++d) {
            const float4 a = *reinterpret_cast<const float4*>(&Qt[d * kAtQ + 4 * ty]);
            const float4 b = *reinterpret_cast<const float4*>(&KV[d * kAtQ + 4 * tx]);
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // row pairs: the Q load holds them side by side
                ffma2(sc[0][j], sc[1][j], a.x, a.y, bv[j], bv[j]);
                ffma2(sc[2][j], sc[3][j], a.z, a.w, bv[j], bv[j]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = 4 * ty + i, qi = q0 + row;
            const int nk = (qi < T) ? (causal ? qi + 1 : T) : 0;
            float cm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = k0 + 4 * tx + j;
                sc[i][j] = (key < nk) ? __fmul_rn(sc[i][j], scale) : -INFINITY;
                cm = fmaxf(cm, sc[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
            const float mn = fmaxf(m_r[i], cm);
            const float alpha = det_expf(__fsub_rn(m_r[i], mn));
            float4 pv;
            pv.x = det_expf(__fsub_rn(sc[i][0], mn));
            pv.y = det_expf(__fsub_rn(sc[i][1], mn));
            pv.z = det_expf(__fsub_rn(sc[i][2], mn));
            pv.w = det_expf(__fsub_rn(sc[i][3], mn));
            float part = __fadd_rn(__fadd_rn(__fadd_rn(pv.x, pv.y), pv.z), pv.w);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
            l_r[i] = __fadd_rn(__fmul_rn(l_r[i], alpha), part);
            m_r[i] = mn;
            *reinterpret_cast<float4*>(&P[row * kAtPP + 4 * tx]) = pv;
            if (tx == 0) alpha_sm[row] = alpha;
        }
        __syncthreads();  // P and alpha written; K^T chunk consumed
        for (int e = t; e < kAtQ * hd4; e += kAtThreads) {
            const int j = e / hd4, d4 = 4 * (e % hd4);
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + j < T) x = *reinterpret_cast<const float4*>(vh + (int64_t)(k0 + j) * ldv + d4);
            *reinterpret_cast<float4*>(&KV[j * hd + d4]) = x;
        }
        __syncthreads();
        if (active) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float al = alpha_sm[4 * rg + i];
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmul_rn(acc[i][j], al);
            }
            const int jn = min(kAtQ, kend - k0);
            // four keys per step: each row's four probabilities are one 16-byte load (the P row stride keeps
            // 4-key groups aligned); keys past jn are skipped, so every output sees the same fma sequence
            for (int j4 = 0; j4 < jn; j4 += 4) {
                float4 p4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) p4[i] = *reinterpret_cast<const float4*>(&P[(4 * rg + i) * kAtPP + j4]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    if (j4 + kk < jn) {
                        const float4 v0 = *reinterpret_cast<const float4*>(&KV[(j4 + kk) * hd + 8 * cg]);
                        const float4 v1 = *reinterpret_cast<const float4*>(&KV[(j4 + kk) * hd + 8 * cg + 4]);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float pr = (kk == 0) ? p4[i].x : (kk == 1) ? p4[i].y : (kk == 2) ? p4[i].z : p4[i].w;
                            ffma2(acc[i][0], acc[i][1], pr, pr, v0.x, v0.y);
                            ffma2(acc[i][2], acc[i][3], pr, pr, v0.z, v0.w);
                            ffma2(acc[i][4], acc[i][5], pr, pr, v1.x, v1.y);
                            ffma2(acc[i][6], acc[i][7], pr, pr, v1.z, v1.w);
                        }
                    }
                }
            }
        }
    }
    if (tx == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) inv_sm[4 * ty + i] = (l_r[i] > 0.0f) ? __fdiv_rn(1.0f, l_r[i]) : 0.0f;
    }
    __syncthreads();
    if (active) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qi = q0 + 4 * rg + i;
            if (qi >= T) continue;
            const float inv = inv_sm[4 * rg + i];
            float* orow = o + (row0 + qi) * ldo + (int64_t)h * hd + 8 * cg;
            *reinterpret_cast<float4*>(orow) = make_float4(__fmul_rn(acc[i][0], inv), __fmul_rn(acc[i][1], inv),
                                                           __fmul_rn(acc[i][2], inv), __fmul_rn(acc[i][3], inv));
            *reinterpret_cast<float4*>(orow + 4) = make_float4(__fmul_rn(acc[i][4], inv), __fmul_rn(acc[i][5], inv),
                                                               __fmul_rn(acc[i][6], inv), __fmul_rn(acc[i][7], inv));
        }
    }
}

// Wider-tile, prefetching form of attention_kernel for head dims 128 and 72 (the BitVLA decoder and ViT): 128
// threads per (64-query block, head, sequence). Every score and output goes through the same fp32 operation
// sequence as in attention_kernel -- ascending-d fma chains, the same 64-key chunks, a row's 64 keys spread
// over 16 consecutive lanes (4 each) with the same max / sum butterflies, ascending-key P.V chains -- so the
// two kernels agree bit for bit. Each thread holds 8 rows x 4 keys of the score tile and 8 rows x 8 columns
// (HD 128) or 4 rows x 9 columns (HD 72) of the output, so each shared-memory load feeds more FMAs; output
// rows are interleaved (rg + 64/OR * i) so the row groups of a warp read different banks of P. Chunk c + 1
// is fetched while chunk c computes: its K rows into registers during the P.V phase (stored transposed,
// RoPE applied, after it), its V rows by cp.async into their own buffer during the next score phase.
// P is a 64 x 64 tile with its 16-byte chunks XOR-swizzled by row (conflict-free row-wise stores and reads).
__device__ __forceinline__ void att_cp_async_16(void* smem_dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

template <int HD>
__global__ void __launch_bounds__(128, HD == 128 ? 2 : 4)
attention_wide_kernel(const float* __restrict__ q, int64_t ldq, const float* __restrict__ k, int64_t ldk,
                      const float* __restrict__ v, int64_t ldv, float* __restrict__ o, int64_t ldo, int T, int heads,
                      int kv_heads, float scale, int causal, const float2* __restrict__ rope) {
    constexpr int OR = HD == 128 ? 8 : 4, OC = HD == 128 ? 8 : 9;  // output rows / columns per thread
    constexpr int NCG = HD / OC;                                   // column groups (16 or 8)
    constexpr int RS = kAtQ / OR;                                  // row stride between a thread's rows
    constexpr int HALF = HD / 2, H4 = HALF / 4;
    constexpr int KITEMS = (kAtQ * H4 + 127) / 128;                // K (row, 4-pair) items per thread
    static_assert(NCG * OC == HD && RS * NCG == 128, "output tiling covers 64 x HD with 128 threads");
    extern __shared__ __align__(16) float at_sm[];
    float* Qt = at_sm;                    // [HD][64]
    float* Kt = Qt + HD * kAtQ;           // K^T chunk [HD][64]
    // Lean form (head dim 72): V shares K^T's buffer and chunks are staged synchronously, so four CTAs fit on
    // an SM and the ViT's 512-CTA grid runs as one wave (three per SM left a 68-CTA second wave).
    constexpr bool kLean = HD == 72;
    float* Vc = kLean ? Kt : Kt + HD * kAtQ;  // V chunk [64][HD]
    float* P = Vc + HD * kAtQ;            // [64][64], chunk q of row r at (q ^ (r & 15))
    float* alpha_sm = P + kAtQ * kAtQ;    // [64] per-row rescale of the chunk
    float* inv_sm = alpha_sm + kAtQ;      // [64] 1 / l at the end
    const int h = blockIdx.x, g = h / (heads / kv_heads);
    const int zi = (int)(gridDim.z - 1u - blockIdx.z);  // heaviest (causal) blocks first
    const int q0 = zi * kAtQ;
    // Paired tail: when the last query block holds at most 32 rows and heads come in pairs within a K/V
    // group, the CTA of even head h takes the tail rows of heads h and h + 1 (tile rows 0-31 and 32-63;
    // same keys, same values) and the CTA of h + 1 has nothing to do. Every row goes through the same
    // operations as in an unpaired tile.
    const bool pair = zi == (int)gridDim.z - 1 && T - q0 <= 32 && (heads / kv_heads) % 2 == 0;
    if (pair && (h & 1)) return;
    const int64_t row0 = (int64_t)blockIdx.y * T;
    const float* qh = q + row0 * ldq + (int64_t)h * HD;
    const float* kh = k + row0 * ldk + (int64_t)g * HD;
    const float* vh = v + row0 * ldv + (int64_t)g * HD;
    const int t = threadIdx.x;
    auto qpos = [&](int row) { return q0 + (pair ? (row & 31) : row); };  // position of a tile row
    griddep_wait();  // q/k/v are written by the preceding kernel
    griddep_launch();

    const int kend = causal ? min(T, q0 + kAtQ) : T;
    const int nchunks = (kend + kAtQ - 1) / kAtQ;
    float4 kpa[KITEMS], kpb[KITEMS];  // K rows of the next chunk: pairs (d4.., HALF + d4..)
    auto load_k = [&](int k0) {
#pragma unroll
        for (int it = 0; it < KITEMS; ++it) {
            const int e = t + 128 * it, i = e % kAtQ, d4 = 4 * (e / kAtQ);
            kpa[it] = kpb[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < kAtQ * H4 && k0 + i < T) {
                const float* row = kh + (int64_t)(k0 + i) * ldk;
                kpa[it] = *reinterpret_cast<const float4*>(row + d4);
                kpb[it] = *reinterpret_cast<const float4*>(row + HALF + d4);
            }
        }
    };
    auto store_k = [&](int k0) {
#pragma unroll
        for (int it = 0; it < KITEMS; ++it) {
            const int e = t + 128 * it, i = e % kAtQ, d4 = 4 * (e / kAtQ);
            if (e >= kAtQ * H4) continue;
            float4 a = kpa[it], b = kpb[it];
            if (rope && k0 + i < T) {
                const float4* cs = reinterpret_cast<const float4*>(rope + (int64_t)(k0 + i) * HALF + d4);
                const float4 c01 = cs[0], c23 = cs[1];
                const float x0[4] = {a.x, a.y, a.z, a.w}, x1[4] = {b.x, b.y, b.z, b.w};
                const float cv[4] = {c01.x, c01.z, c23.x, c23.z}, sv[4] = {c01.y, c01.w, c23.y, c23.w};
                float y0[4], y1[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    y0[c] = __fsub_rn(__fmul_rn(x0[c], cv[c]), __fmul_rn(x1[c], sv[c]));
                    y1[c] = __fadd_rn(__fmul_rn(x0[c], sv[c]), __fmul_rn(x1[c], cv[c]));
                }
                a = make_float4(y0[0], y0[1], y0[2], y0[3]);
                b = make_float4(y1[0], y1[1], y1[2], y1[3]);
            }
            Kt[(d4 + 0) * kAtQ + i] = a.x;
            Kt[(d4 + 1) * kAtQ + i] = a.y;
            Kt[(d4 + 2) * kAtQ + i] = a.z;
            Kt[(d4 + 3) * kAtQ + i] = a.w;
            Kt[(HALF + d4 + 0) * kAtQ + i] = b.x;
            Kt[(HALF + d4 + 1) * kAtQ + i] = b.y;
            Kt[(HALF + d4 + 2) * kAtQ + i] = b.z;
            Kt[(HALF + d4 + 3) * kAtQ + i] = b.w;
        }
    };
    auto issue_v = [&](int k0) {
        for (int e = t; e < kAtQ * (HD / 4); e += 128) {
            const int j = e / (HD / 4), d4 = 4 * (e % (HD / 4));
            const bool in = k0 + j < T;
            att_cp_async_16(&Vc[j * HD + d4], in ? (const void*)(vh + (int64_t)(k0 + j) * ldv + d4) : (const void*)vh,
                            in ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    stage_transposed(Qt, qh, ldq, q0, T, HD, rope, pair ? qh + HD : nullptr);
    load_k(0);
    store_k(0);
    if (!kLean) issue_v(0);
    __syncthreads();  // Qt and K^T of chunk 0 written

    const int ty = t / 16, tx = t % 16;  // score rows 8 ty .. 8 ty + 7, keys 4 tx .. 4 tx + 3
    float m_r[8], l_r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m_r[i] = -INFINITY;
        l_r[i] = 0.0f;
    }
    const int rg = t / NCG, cg = t % NCG;  // output rows rg + RS i, columns OC cg ..
    float acc[OR][OC];
#pragma unroll
    for (int i = 0; i < OR; ++i)
#pragma unroll
        for (int j = 0; j < OC; ++j) acc[i][j] = 0.0f;

    for (int c = 0; c < nchunks; ++c) {
        const int k0 = c * kAtQ;
        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < HD; ++d) {
            const float4 a0 = *reinterpret_cast<const float4*>(&Qt[d * kAtQ + 8 * ty]);
            const float4 a1 = *reinterpret_cast<const float4*>(&Qt[d * kAtQ + 8 * ty + 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Kt[d * kAtQ + 4 * tx]);
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // row pairs: the Q loads hold them side by side
                ffma2(sc[0][j], sc[1][j], a0.x, a0.y, bv[j], bv[j]);
                ffma2(sc[2][j], sc[3][j], a0.z, a0.w, bv[j], bv[j]);
                ffma2(sc[4][j], sc[5][j], a1.x, a1.y, bv[j], bv[j]);
                ffma2(sc[6][j], sc[7][j], a1.z, a1.w, bv[j], bv[j]);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = 8 * ty + i, qi = qpos(row);
            const int nk = (qi < T) ? (causal ? qi + 1 : T) : 0;
            float cm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = k0 + 4 * tx + j;
                sc[i][j] = (key < nk) ? __fmul_rn(sc[i][j], scale) : -INFINITY;
                cm = fmaxf(cm, sc[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
            const float mn = fmaxf(m_r[i], cm);
            const float alpha = det_expf(__fsub_rn(m_r[i], mn));
            float4 pv;
            pv.x = det_expf(__fsub_rn(sc[i][0], mn));
            pv.y = det_expf(__fsub_rn(sc[i][1], mn));
            pv.z = det_expf(__fsub_rn(sc[i][2], mn));
            pv.w = det_expf(__fsub_rn(sc[i][3], mn));
            float part = __fadd_rn(__fadd_rn(__fadd_rn(pv.x, pv.y), pv.z), pv.w);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
            l_r[i] = __fadd_rn(__fmul_rn(l_r[i], alpha), part);
            m_r[i] = mn;
            *reinterpret_cast<float4*>(&P[row * kAtQ + 4 * (tx ^ (row & 15))]) = pv;
            if (tx == 0) alpha_sm[row] = alpha;
        }
        const bool more = c + 1 < nchunks;
        if (kLean) {
            __syncthreads();  // K^T consumed: its buffer takes this chunk's V
            issue_v(k0);
        } else if (more) {
            load_k(k0 + kAtQ);  // in flight during P.V
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // V of this chunk landed, P and alpha written, K^T consumed
#pragma unroll
        for (int i = 0; i < OR; ++i) {
            const float al = alpha_sm[rg + RS * i];
#pragma unroll
            for (int j = 0; j < OC; ++j) acc[i][j] = __fmul_rn(acc[i][j], al);
        }
        const int jn = min(kAtQ, kend - k0);
        for (int j4 = 0; j4 < jn; j4 += 4) {
            float4 p4[OR];
#pragma unroll
            for (int i = 0; i < OR; ++i) {
                const int row = rg + RS * i;
                p4[i] = *reinterpret_cast<const float4*>(&P[row * kAtQ + 4 * ((j4 >> 2) ^ (row & 15))]);
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                if (j4 + kk < jn) {
                    float vv[OC];
                    const float* vr = &Vc[(j4 + kk) * HD + OC * cg];
                    if constexpr (OC == 8) {
                        const float4 v0 = *reinterpret_cast<const float4*>(vr);
                        const float4 v1 = *reinterpret_cast<const float4*>(vr + 4);
                        vv[0] = v0.x; vv[1] = v0.y; vv[2] = v0.z; vv[3] = v0.w;
                        vv[4] = v1.x; vv[5] = v1.y; vv[6] = v1.z; vv[7] = v1.w;
                    } else {
#pragma unroll
                        for (int j = 0; j < OC; ++j) vv[j] = vr[j];
                    }
#pragma unroll
                    for (int i = 0; i < OR; ++i) {
                        const float pr = (kk == 0) ? p4[i].x : (kk == 1) ? p4[i].y : (kk == 2) ? p4[i].z : p4[i].w;
#pragma unroll
                        for (int j = 0; j + 1 < OC; j += 2) ffma2(acc[i][j], acc[i][j + 1], pr, pr, vv[j], vv[j + 1]);
                        if constexpr (OC % 2) acc[i][OC - 1] = __fmaf_rn(pr, vv[OC - 1], acc[i][OC - 1]);
                    }
                }
            }
        }
        if (more) {
            __syncthreads();  // V and P of this chunk consumed
            if (kLean) load_k(k0 + kAtQ);
            store_k(k0 + kAtQ);
            if (!kLean) issue_v(k0 + kAtQ);  // lands during the next score phase
            __syncthreads();                 // K^T of the next chunk written
        }
    }
    if (tx == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) inv_sm[8 * ty + i] = (l_r[i] > 0.0f) ? __fdiv_rn(1.0f, l_r[i]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < OR; ++i) {
        const int row = rg + RS * i, qi = qpos(row);
        if (qi >= T) continue;
        const float inv = inv_sm[row];
        const int ho = h + ((pair && row >= 32) ? 1 : 0);
        float* orow = o + (row0 + qi) * ldo + (int64_t)ho * HD + OC * cg;
        if constexpr (OC == 8) {
            *reinterpret_cast<float4*>(orow) = make_float4(__fmul_rn(acc[i][0], inv), __fmul_rn(acc[i][1], inv),
                                                           __fmul_rn(acc[i][2], inv), __fmul_rn(acc[i][3], inv));
            *reinterpret_cast<float4*>(orow + 4) = make_float4(__fmul_rn(acc[i][4], inv), __fmul_rn(acc[i][5], inv),
                                                               __fmul_rn(acc[i][6], inv), __fmul_rn(acc[i][7], inv));
        } else {
#pragma unroll
            for (int j = 0; j < OC; ++j) orow[j] = __fmul_rn(acc[i][j], inv);
        }
    }
}

// Shared memory of attention_wide_kernel<HD>.
static size_t attention_wide_smem(int hd) {
    return sizeof(float) * ((size_t)(hd == 72 ? 2 : 3) * hd * kAtQ + (size_t)kAtQ * kAtQ + 2 * kAtQ);
}

bool attention_supported(int T, int hd, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo, const void* q,
                         const void* k, const void* v, const void* o) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return T > 0 && hd > 0 && hd % 8 == 0 && hd <= 128 && ldq % 4 == 0 && ldk % 4 == 0 && ldv % 4 == 0 &&
           ldo % 4 == 0 && a16(q) && a16(k) && a16(v) && a16(o) && attention_smem_bytes(T, hd) <= 227 * 1024;
}

cudaError_t launch_attention(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                             int batch, int T, int heads, int kv_heads, int hd, float scale, bool causal, float* o,
                             int64_t ldo, cudaStream_t st, const float2* rope) {
    if (batch <= 0 || T <= 0) return cudaSuccess;
    const size_t smem = (hd == 128 || hd == 72) ? attention_wide_smem(hd) : attention_smem_bytes(T, hd);
    // head dims 128 and 72 take the wider-tile kernel (same results bit for bit)
    const void* kfn = hd == 128 ? reinterpret_cast<const void*>(attention_wide_kernel<128>)
                    : hd == 72  ? reinterpret_cast<const void*>(attention_wide_kernel<72>)
                                : reinterpret_cast<const void*>(attention_kernel);
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_dynamic_smem(kfn, smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)heads, (unsigned)batch, (unsigned)ceil_div(T, kAtQ));
    cfg.blockDim = dim3(hd == 128 || hd == 72 ? 128 : kAtThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (hd == 128)
        return cudaLaunchKernelEx(&cfg, attention_wide_kernel<128>, q, ldq, k, ldk, v, ldv, o, ldo, T, heads, kv_heads,
                                  scale, causal ? 1 : 0, rope);
    if (hd == 72)
        return cudaLaunchKernelEx(&cfg, attention_wide_kernel<72>, q, ldq, k, ldk, v, ldv, o, ldo, T, heads, kv_heads,
                                  scale, causal ? 1 : 0, rope);
    return cudaLaunchKernelEx(&cfg, attention_kernel, q, ldq, k, ldk, v, ldv, o, ldo, T, heads, kv_heads, hd, scale,
                              causal ? 1 : 0, rope);
}

}  // namespace b2s
