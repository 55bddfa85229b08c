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

cudaError_t launch_act_quant(const float* x, int64_t ldx, const float* g, bool norm, float eps, int64_t M, int64_t K,
                             int8_t* q, int64_t ldq, float* s, int32_t* sums, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
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
