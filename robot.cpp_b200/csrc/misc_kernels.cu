// misc_kernels.cu -- softmax (ggml_soft_max_ext semantics) and the i2_s row-padding repack.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

__device__ unsigned int g_device_error = 0;

// ------------------------------------------------------------------------------------------------
// y[m,:] = softmax(x[m,:] * scale + mask[m % mask_rows, :]), one warp per row.
// Mirrors ggml_soft_max_ext(ctx, kq, mask, scale, 0.0f) as called at
// src/models/smolvla/action_expert.cpp:773 and ggml_soft_max_inplace at src/models/smolvla/vision.cpp:328
// (scale 1, no mask). With causal_rows > 0, row r is query position r % causal_rows and the keys after
// it are masked (the decoder's causal mask without a mask tensor). Rows up to 32*kSmRegs elements stay
// in registers (one HBM read); longer rows take a second pass that hits L1/L2. Masked -inf entries give
// exact zeros.
constexpr int kSmWarps = 8;
constexpr int kSmRegs = 16;  // elements per lane kept in registers (rows <= 512)

__global__ void __launch_bounds__(kSmWarps * 32)
softmax_kernel(const float* __restrict__ x, const float* __restrict__ mask, int64_t mask_rows, int64_t M, int N,
               float scale, int causal_rows, float* __restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kSmWarps + (threadIdx.x >> 5);
    if (row >= M) return;
    const float* xr = x + row * N;
    const float* mr = mask ? mask + (row % mask_rows) * N : nullptr;
    const int qpos = causal_rows > 0 ? (int)(row % causal_rows) : N;  // keys after the query are masked
    float* yr = y + row * N;
    auto logit = [&](int i) -> float {
        if (i > qpos) return -INFINITY;
        float v = __fmul_rn(xr[i], scale);
        if (mr) v = __fadd_rn(v, mr[i]);
        return v;
    };
    float reg[kSmRegs];
    const bool in_regs = N <= 32 * kSmRegs;
    float mx = -INFINITY;
    if (in_regs) {
#pragma unroll
        for (int j = 0; j < kSmRegs; ++j) {
            const int i = lane + 32 * j;
            reg[j] = (i < N) ? logit(i) : -INFINITY;
            mx = fmaxf(mx, reg[j]);
        }
    } else {
        for (int i = lane; i < N; i += 32) mx = fmaxf(mx, logit(i));
    }
    mx = warp_max(mx);
    float sum = 0.0f;
    if (in_regs) {
#pragma unroll
        for (int j = 0; j < kSmRegs; ++j) {
            const float e = (reg[j] == -INFINITY) ? 0.0f : det_expf(__fsub_rn(reg[j], mx));
            reg[j] = e;
            sum += e;
        }
    } else {
        for (int i = lane; i < N; i += 32) {
            const float v = logit(i);
            sum += (v == -INFINITY) ? 0.0f : det_expf(__fsub_rn(v, mx));
        }
    }
    sum = warp_sum_f(sum);
    const float inv = (sum > 0.0f) ? __fdiv_rn(1.0f, sum) : 0.0f;
    if (in_regs) {
#pragma unroll
        for (int j = 0; j < kSmRegs; ++j) {
            const int i = lane + 32 * j;
            if (i < N) yr[i] = __fmul_rn(reg[j], inv);
        }
    } else {
        for (int i = lane; i < N; i += 32) {
            const float v = logit(i);
            yr[i] = __fmul_rn((v == -INFINITY) ? 0.0f : det_expf(__fsub_rn(v, mx)), inv);
        }
    }
}

cudaError_t launch_softmax_rows(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N,
                                float scale, int causal_rows, float* y, cudaStream_t st) {
    if (M <= 0) return cudaSuccess;
    softmax_kernel<<<(unsigned)ceil_div(M, kSmWarps), kSmWarps * 32, 0, st>>>(x, mask, mask_rows, M, (int)N, scale,
                                                                               causal_rows, y);
    return cudaGetLastError();
}

cudaError_t launch_softmax(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N, float scale,
                           float* y, cudaStream_t st) {
    return launch_softmax_rows(x, mask, mask_rows, M, N, scale, 0, y, st);
}

// ------------------------------------------------------------------------------------------------
// Flattened i2_s (block interleave over the whole tensor) -> row-padded i2_s_r (each row padded to
// Kp = roundup(K,128) with code 1, blocks restarting at every row). One thread per output byte;
// every output byte gathers its four 2-bit codes from the flattened positions.
__global__ void repack_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t N, int64_t K,
                                   int64_t Kp) {
    const int64_t rb = Kp / 4;
    const int64_t total = N * rb;
    for (int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; d < total; d += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = d / rb, off = d - r * rb;
        const int64_t b = off / 32, i = off % 32;
        uint32_t out = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int64_t k = kQK * b + 32 * g + i;
            uint32_t code = 1;
            if (k < K) {
                const int64_t flat = r * K + k;
                const int64_t j = flat % kQK;
                code = (src[32 * (flat / kQK) + (j % 32)] >> (6 - 2 * (j / 32))) & 3u;
            }
            out |= code << (6 - 2 * g);
        }
        dst[d] = (uint8_t)out;
    }
    if (blockIdx.x == 0 && threadIdx.x < 32) dst[total + threadIdx.x] = src[N * K / 4 + threadIdx.x];
}

cudaError_t launch_repack_rows(const uint8_t* src, uint8_t* dst, int64_t N, int64_t K, cudaStream_t st) {
    const int64_t Kp = round_up(K, kQK);
    const int64_t total = N * Kp / 4;
    const unsigned blocks = (unsigned)(ceil_div(total, 256) < 148 * 16 ? ceil_div(total, 256) : 148 * 16);
    repack_rows_kernel<<<blocks > 0 ? blocks : 1, 256, 0, st>>>(src, dst, N, K, Kp);
    return cudaGetLastError();
}

}  // namespace b2s
