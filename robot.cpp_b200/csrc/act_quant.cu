// act_quant.cu -- per-token absmax int8 activation quantization, alone and fused behind RMSNorm.
//
// Semantics (restated from the BitNet fork's quantize_row_i8_s, see oracle/i2s_oracle.h):
//   s = 127 / max(1e-5, max_k |x_k|);  q_k = clamp(round_half_away(fp32(x_k * s)), -128, 127);
//   sum = sum_k q_k (the correction term of the unsigned-code dot product).
// The fused variant first applies ggml's rms_norm + ggml_mul(weight)
// (src/models/smolvla/action_expert.cpp:731-736, src/models/pi0/vlm.cpp:216): the sum of fp32 squares
// is accumulated in double, mean = (float)(sum/K), scale = 1/sqrtf(mean + eps), y = (x*scale)*g;
// the normalized row is never written to HBM, only its int8 codes.
//
// One CTA per token row; the row is read with 16-byte vector loads when K % 4 == 0 and the row
// pointer is 16-byte aligned (the common case), otherwise with scalar loads. HBM-bound: bytes per
// row = 4K (read, once from DRAM; the second pass hits L1/L2) + K (int8 write) + 8.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

constexpr int kActThreads = 256;

__device__ __forceinline__ float block_max(float v, float* red) {
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

__device__ __forceinline__ int block_sum_i(int v, int* red) {
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

__device__ __forceinline__ double block_sum_d(double v, double* red) {
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

// NORM = false: plain act-quant of x. NORM = true: act-quant of (x * rms_scale) * g.
// VEC = true: 16-byte loads (K % 4 == 0, row 16-byte aligned, q row 4-byte aligned).
template <bool NORM, bool VEC>
__global__ void __launch_bounds__(kActThreads)
act_quant_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ g, float eps, int K,
                 int8_t* __restrict__ q, int64_t ldq, float* __restrict__ s_out, int32_t* __restrict__ sum_out) {
    __shared__ double red_d[32];
    float* red_f = reinterpret_cast<float*>(red_d);
    int* red_i = reinterpret_cast<int*>(red_d);
    const int64_t m = blockIdx.x;
    const float* xr = x + m * ldx;
    int8_t* qr = q + m * ldq;
    griddep_wait();    // x is written by the preceding kernel
    griddep_launch();  // the consuming GEMM may start now: it waits for this grid before reading q

    float nscale = 1.0f;
    if (NORM) {
        double acc = 0.0;
        if (VEC) {
            const float4* x4 = reinterpret_cast<const float4*>(xr);
            for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
                float4 v = x4[i];
                acc += (double)__fmul_rn(v.x, v.x);
                acc += (double)__fmul_rn(v.y, v.y);
                acc += (double)__fmul_rn(v.z, v.z);
                acc += (double)__fmul_rn(v.w, v.w);
            }
        } else {
            for (int i = threadIdx.x; i < K; i += blockDim.x) acc += (double)__fmul_rn(xr[i], xr[i]);
        }
        const double tot = block_sum_d(acc, red_d);
        const float mean = (float)(tot / (double)K);
        nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }

    auto val = [&](float v, int k) -> float {
        if (!NORM) return v;
        float y = __fmul_rn(v, nscale);
        if (g) y = __fmul_rn(y, g[k]);
        return y;
    };

    float amax = 0.0f;
    if (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            float4 v = x4[i];
            amax = fmaxf(amax, fabsf(val(v.x, 4 * i + 0)));
            amax = fmaxf(amax, fabsf(val(v.y, 4 * i + 1)));
            amax = fmaxf(amax, fabsf(val(v.z, 4 * i + 2)));
            amax = fmaxf(amax, fabsf(val(v.w, 4 * i + 3)));
        }
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(val(xr[i], i)));
    }
    amax = block_max(amax, red_f);
    const float s = actq_scale(amax);

    int sum = 0;
    if (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        char4* q4 = reinterpret_cast<char4*>(qr);
        for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
            float4 v = x4[i];
            const int a = actq_round(val(v.x, 4 * i + 0), s);
            const int b = actq_round(val(v.y, 4 * i + 1), s);
            const int c = actq_round(val(v.z, 4 * i + 2), s);
            const int d = actq_round(val(v.w, 4 * i + 3), s);
            q4[i] = make_char4((signed char)a, (signed char)b, (signed char)c, (signed char)d);
            sum += a + b + c + d;
        }
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const int a = actq_round(val(xr[i], i), s);
            qr[i] = (int8_t)a;
            sum += a;
        }
    }
    sum = block_sum_i(sum, red_i);
    if (threadIdx.x == 0) {
        s_out[m] = s;
        if (sum_out) sum_out[m] = sum;
    }
}

// ------------------------------------------------------------------------------------------------
// Register-resident variant for rows of K <= 8192 floats (16-byte aligned, K % 4 == 0): one CTA of TPR
// threads per row (128 or 256, VPT = 3 to 8 float4 per thread) reads the row from memory once into
// registers and runs the norm's sums, the absmax and the code sum as in-register partials combined by
// warp shuffles and one TPR/32-entry shared-memory step. The kernel is latency-bound (a row of P is in
// L2 when it runs): for a prefill batch (a few hundred rows, all resident in one wave) wide CTAs keep the
// per-thread dependency chains short; for thousands of rows the tightest shape keeps more rows resident.
// KIND: 0 RMSNorm, 1 LayerNorm, 2 no norm, 3 GELU then no norm (gelu_tanh, the GEMM epilogue's fp32
// operations, applied here to a GEMM output written without it). The fp32 operation sequence per element
// is the one of act_quant_kernel / norm_kernel; only the (double) summation order differs.
template <int NW>
__device__ __forceinline__ double row_sum_d(double v, double* red) {
    v = warp_sum_d(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) t += red[w];
    __syncthreads();
    return t;
}
template <int NW>
__device__ __forceinline__ float row_max_f(float v, float* red) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) t = fmaxf(t, red[w]);
    __syncthreads();
    return t;
}
template <int NW>
__device__ __forceinline__ int row_sum_i(int v, int* red) {
    v = warp_sum_i(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int t = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) t += red[w];
    __syncthreads();
    return t;
}

template <int KIND, bool QUANT, int TPR, int VPT>
__global__ void __launch_bounds__(TPR)
rowq_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ g, const float* __restrict__ b,
            float eps, int K, float* __restrict__ y, int64_t ldy, int8_t* __restrict__ q, int64_t ldq,
            float* __restrict__ s_out, int32_t* __restrict__ sum_out) {
    constexpr int NW = TPR / 32;
    __shared__ double red_d[NW];
    float* red_f = reinterpret_cast<float*>(red_d);
    int* red_i = reinterpret_cast<int*>(red_d);
    const int64_t m = blockIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x + m * ldx);
    const int K4 = K / 4;
    griddep_wait();    // x is written by the preceding kernel
    griddep_launch();  // the consumer waits for this grid before reading q / y
    float4 r[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + TPR * i;
        r[i] = (c < K4) ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean = 0.0f, nscale = 1.0f;
    if (KIND == 1) {
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            acc += (double)r[i].x;
            acc += (double)r[i].y;
            acc += (double)r[i].z;
            acc += (double)r[i].w;
        }
        mean = (float)(row_sum_d<NW>(acc, red_d) / (double)K);
    }
    if (KIND < 2) {
        double acc2 = 0.0;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            if (threadIdx.x + TPR * i >= K4) continue;
            const float vx = (KIND == 1) ? __fsub_rn(r[i].x, mean) : r[i].x;
            const float vy = (KIND == 1) ? __fsub_rn(r[i].y, mean) : r[i].y;
            const float vz = (KIND == 1) ? __fsub_rn(r[i].z, mean) : r[i].z;
            const float vw = (KIND == 1) ? __fsub_rn(r[i].w, mean) : r[i].w;
            acc2 += (double)__fmul_rn(vx, vx);
            acc2 += (double)__fmul_rn(vy, vy);
            acc2 += (double)__fmul_rn(vz, vz);
            acc2 += (double)__fmul_rn(vw, vw);
        }
        const float var = (float)(row_sum_d<NW>(acc2, red_d) / (double)K);
        nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    auto val = [&](float v, float gv, float bv) -> float {
        if (KIND == 3) return gelu_tanh(v);
        if (KIND == 2) return v;
        if (KIND == 1) v = __fsub_rn(v, mean);
        v = __fmul_rn(v, nscale);
        if (g) v = __fmul_rn(v, gv);
        if (b) v = __fadd_rn(v, bv);
        return v;
    };
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + TPR * i;
        if (c >= K4) continue;
        const float4 gv = (KIND < 2 && g) ? g4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 bv = (KIND < 2 && b) ? b4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        r[i].x = val(r[i].x, gv.x, bv.x);
        r[i].y = val(r[i].y, gv.y, bv.y);
        r[i].z = val(r[i].z, gv.z, bv.z);
        r[i].w = val(r[i].w, gv.w, bv.w);
    }
    if (!QUANT) {
        float4* y4 = reinterpret_cast<float4*>(y + m * ldy);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int c = threadIdx.x + TPR * i;
            if (c < K4) y4[c] = r[i];
        }
        return;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        if (threadIdx.x + TPR * i >= K4) continue;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(r[i].x), fabsf(r[i].y)), fmaxf(fabsf(r[i].z), fabsf(r[i].w))));
    }
    amax = row_max_f<NW>(amax, red_f);
    const float s = actq_scale(amax);
    char4* q4 = reinterpret_cast<char4*>(q + m * ldq);
    int sum = 0;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = threadIdx.x + TPR * i;
        if (c >= K4) continue;
        const int a0 = actq_round(r[i].x, s), a1 = actq_round(r[i].y, s);
        const int a2 = actq_round(r[i].z, s), a3 = actq_round(r[i].w, s);
        q4[c] = make_char4((signed char)a0, (signed char)a1, (signed char)a2, (signed char)a3);
        sum += a0 + a1 + a2 + a3;
    }
    sum = row_sum_i<NW>(sum, red_i);
    if (threadIdx.x == 0) {
        s_out[m] = s;
        if (sum_out) sum_out[m] = sum;
    }
}

template <int KIND, bool QUANT, int TPR, int VPT>
static cudaError_t launch_rowq_tpr(const float* x, int64_t ldx, const float* g, const float* b, float eps,
                                   int64_t M, int K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s,
                                   int32_t* sums, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M);
    cfg.blockDim = dim3(TPR);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rowq_kernel<KIND, QUANT, TPR, VPT>, x, ldx, g, b, eps, K, y, ldy, q, ldq, s,
                              sums);
}

template <int KIND, bool QUANT>
static cudaError_t launch_rowq_k(const float* x, int64_t ldx, const float* g, const float* b, float eps, int64_t M,
                                 int K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                                 cudaStream_t st) {
    const int K4 = K / 4;
    // A few hundred rows (one prefill) are all resident at once whatever the shape: wide CTAs keep each
    // thread's chain short (the M = 300 FFN block took 48.8 µs with the tight shapes below, 47.5 with these).
    if (M < 1024) {
        if (K4 <= 128 * 4)
            return launch_rowq_tpr<KIND, QUANT, 128, 4>(x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st);
        if (K4 <= 256 * 4)
            return launch_rowq_tpr<KIND, QUANT, 256, 4>(x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st);
        return launch_rowq_tpr<KIND, QUANT, 256, 8>(x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st);
    }
    // Thousands of rows run in waves: the fewest float4 slots per thread that hold the row, so more rows are
    // resident per SM (fewer registers) -- 128 threads up to 5 per thread (K = 2560 fills 128 x 5 exactly,
    // 53 registers, 9 CTAs per SM against 5 for 256 x 4), then 256 threads up to 8 (K = 4304 -> 5, K = 6912
    // -> 7). Batch of 8 observations: 14.3 -> 12.1 µs (K = 2560), 28.7 -> 25.1 µs (K = 6912) per launch.
#define B2S_ROWQ(T, V) \
    if (K4 <= (T) * (V)) return launch_rowq_tpr<KIND, QUANT, T, V>(x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st)
    B2S_ROWQ(128, 3);
    B2S_ROWQ(128, 4);
    B2S_ROWQ(128, 5);
    B2S_ROWQ(256, 3);
    B2S_ROWQ(256, 4);
    B2S_ROWQ(256, 5);
    B2S_ROWQ(256, 6);
    B2S_ROWQ(256, 7);
#undef B2S_ROWQ
    return launch_rowq_tpr<KIND, QUANT, 256, 8>(x, ldx, g, b, eps, M, K, y, ldy, q, ldq, s, sums, st);
}

bool rowq_eligible(const float* x, int64_t ldx, const float* g, const float* b, int64_t K, const void* out,
                   int64_t ldo, bool quant) {
    auto a16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool out_ok = quant ? ((reinterpret_cast<uintptr_t>(out) & 3) == 0 && ldo % 4 == 0)
                              : (a16(out) && ldo % 4 == 0);
    return K > 0 && K % 4 == 0 && K <= 4 * 256 * 8 && ldx % 4 == 0 && a16(x) && a16(g) && a16(b) && out_ok;
}

cudaError_t launch_rowq(int kind, bool quant, const float* x, int64_t ldx, const float* g, const float* b, float eps,
                        int64_t M, int64_t K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                        cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    const int k = (int)K;
    if (kind == 0) {
        if (quant) return launch_rowq_k<0, true>(x, ldx, g, b, eps, M, k, y, ldy, q, ldq, s, sums, st);
        return launch_rowq_k<0, false>(x, ldx, g, b, eps, M, k, y, ldy, q, ldq, s, sums, st);
    }
    if (kind == 1) {
        if (quant) return launch_rowq_k<1, true>(x, ldx, g, b, eps, M, k, y, ldy, q, ldq, s, sums, st);
        return launch_rowq_k<1, false>(x, ldx, g, b, eps, M, k, y, ldy, q, ldq, s, sums, st);
    }
    if (kind == 3) return launch_rowq_k<3, true>(x, ldx, nullptr, nullptr, 0.0f, M, k, y, ldy, q, ldq, s, sums, st);
    return launch_rowq_k<2, true>(x, ldx, nullptr, nullptr, 0.0f, M, k, y, ldy, q, ldq, s, sums, st);
}

cudaError_t launch_act_quant(const float* x, int64_t ldx, const float* g, bool norm, float eps, int64_t M, int64_t K,
                             int8_t* q, int64_t ldq, float* s, int32_t* sums, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    if (rowq_eligible(x, ldx, norm ? g : nullptr, nullptr, K, q, ldq, true))
        return launch_rowq(norm ? 0 : 2, true, x, ldx, norm ? g : nullptr, nullptr, eps, M, K, nullptr, 0, q, ldq, s,
                           sums, st);
    const bool vec = (K % 4 == 0) && (ldx % 4 == 0) && (ldq % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)M);
    cfg.blockDim = dim3(kActThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int k = (int)K;
    if (norm) {
        if (vec) return cudaLaunchKernelEx(&cfg, act_quant_kernel<true, true>, x, ldx, g, eps, k, q, ldq, s, sums);
        return cudaLaunchKernelEx(&cfg, act_quant_kernel<true, false>, x, ldx, g, eps, k, q, ldq, s, sums);
    }
    if (vec) return cudaLaunchKernelEx(&cfg, act_quant_kernel<false, true>, x, ldx, g, eps, k, q, ldq, s, sums);
    return cudaLaunchKernelEx(&cfg, act_quant_kernel<false, false>, x, ldx, g, eps, k, q, ldq, s, sums);
}

}  // namespace b2s
