// b2s_internal.h -- launchers shared between the kernel files and the C-ABI layer (not exported).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace b2s {

// Weight operand as the kernels see it: row-padded i2_s bytes (row stride Kp/4, Kp = roundup(K,128)),
// the per-tensor fp32 scale living in device memory right after the codes.
struct I2sWeight {
    const uint8_t* codes;  // N rows x Kp/4 bytes
    const float* scale;    // device pointer to the fp32 tensor scale
    int64_t N, K, Kp;
};

// Quantized activations: q [M x ldq] int8 (K valid columns), s [M], sums [M].
struct Q8Act {
    const int8_t* q;
    const float* s;
    const int32_t* sums;
    int64_t M, K, ldq;
};

cudaError_t launch_act_quant(const float* x, int64_t ldx, const float* g, bool norm, float eps, int64_t M, int64_t K,
                             int8_t* q, int64_t ldq, float* s, int32_t* sums, cudaStream_t st);

cudaError_t launch_gemv_i2s(const I2sWeight& w, const Q8Act& a, float* y, int64_t ldy, cudaStream_t st);

// Tensor-core path. mode 0: Y = W*q. mode 1 (gate/up): P = relu(Wg*q)^2 * (Wu*q).
// tmap_* are built by the caller (host) for these exact buffers.
struct TcGemmArgs {
    CUtensorMap tmap_w0;  // packed codes of W (or W_gate), 2D u8 [N rows][Kp/4 bytes], box 32 x 128 (64 in mode 1)
    CUtensorMap tmap_w1;  // packed codes of W_up (mode 1), box 32 x 64
    CUtensorMap tmap_q;   // int8 activations 2D [M rows][K], box 128 x bn_sub, 128B swizzle
    const float* w0_scale;
    const float* w1_scale;
    const float* s;       // act scales [M]
    const int32_t* sums;  // act sums [M]
    float* y;
    int64_t ldy;
    int M, N, K, Kp;      // N = output columns (F in mode 1)
    int T;                // tokens per CTA = nsub * bn_sub (<= 320)
    int bn_sub;           // MMA N per sub-tile (multiple of 16, <= 256)
    int nsub;             // 1 or 2 sub-tiles
    int n_tiles, m_tiles, splits;  // grid; splits = K-split CTAs per cluster (1..8)
    int mode;
};
cudaError_t launch_gemm_i2s_tc(const TcGemmArgs& args, cudaStream_t st);

cudaError_t launch_repack_rows(const uint8_t* src, uint8_t* dst, int64_t N, int64_t K, cudaStream_t st);

cudaError_t launch_softmax(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N, float scale,
                           float* y, cudaStream_t st);

// Records `msg` as the calling thread's b2s_last_error() and returns `code`.
int set_last_error(int code, const char* msg);

// Scratch bytes the MUL_MAT node needs for its int8 activations, scales and sums (same layout as the
// caller workspace of b2s_mul_mat); 0 with the error set if W or X is malformed.
size_t mul_mat_scratch_bytes(const void* W, const void* X);

// The MUL_MAT node of b2s_mul_mat run into a scratch region the caller already owns
// (`scratch` device pointer, `capacity` bytes, 256-byte aligned). Validates exactly like b2s_mul_mat.
int mul_mat_into_scratch(const void* W, const void* X, void* Y, void* scratch, size_t capacity, cudaStream_t st);

}  // namespace b2s
