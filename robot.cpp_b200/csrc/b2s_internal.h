// b2s_internal.h -- launchers shared between the kernel files and the C-ABI layer (not exported).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <cuda.h>
#include <cuda_runtime.h>

#include "b2s_common.cuh"

namespace b2s {

// Raises kernel `kfn`'s dynamic shared memory limit to at least `bytes` on the current device. The attribute
// belongs to the function in one device's context, so the size already set is remembered per (function,
// device); thread-safe, for engines driving several GPUs from one process.
cudaError_t ensure_dynamic_smem(const void* kfn, size_t bytes);

// 2D u8 tensor map (inner dim `cols` bytes, `rows` rows of stride `ld` bytes, box box_c x box_r, swizzle
// swz); false when the driver entry point is missing or the base / stride is not TMA-compatible.
bool tmap_u8_2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_c,
                uint32_t box_r, CUtensorMapSwizzle swz);

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

// Register-resident norm / act-quant of rows of K <= 8192 (act_quant.cu); kind 0 RMSNorm, 1 LayerNorm,
// 2 no norm (quant only), 3 GELU (gelu_tanh) then act-quant (quant only). rowq_eligible: K % 4 == 0, 16-byte aligned rows and parameters.
bool rowq_eligible(const float* x, int64_t ldx, const float* g, const float* b, int64_t K, const void* out,
                   int64_t ldo, bool quant);
cudaError_t launch_rowq(int kind, bool quant, const float* x, int64_t ldx, const float* g, const float* b, float eps,
                        int64_t M, int64_t K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                        cudaStream_t st);
cudaError_t launch_act_quant(const float* x, int64_t ldx, const float* g, bool norm, float eps, int64_t M, int64_t K,
                             int8_t* q, int64_t ldq, float* s, int32_t* sums, cudaStream_t st);

// Optional epilogue of the plain GEMM (mode 0 of the tensor-core path and the GEMV), applied in this
// order to v = (float)acc * (w_scale / s[m]):  v += bias[n];  v = gelu_tanh(v) if act == 1;
// v = residual[m * ld_res + n] + v.
// scale_rows > 0 makes the weight scale an array: output row n uses w_scale[n / scale_rows] (several
// ternary tensors stacked row-wise into one weight, e.g. fused q/k/v, each keeping its own scale;
// a multiple of 128 on the tensor-core path).
struct Epilogue {
    const float* bias;      // [N] or nullptr
    const float* residual;  // [M x ld_res] or nullptr (may alias the output)
    int64_t ld_res;
    int act;                // 0 none, 1 GELU (tanh approximation)
    int scale_rows;         // 0: one per-tensor scale
};

// GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x^2))), fp32 ops in this order,
// tanh = det_tanhf (b2s_common.cuh).
__device__ __forceinline__ float gelu_tanh(float x) {
    const float inner = __fmul_rn(__fmul_rn(0.79788456080286535588f, x),
                                  __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, det_tanhf(inner)));
}

// Independent problems of one GEMV launch (grid dimension y): problem b reads the weight codes at
// codes + b * w_stride bytes (the tensor's one scale is shared), activations at q + b * q_stride bytes, scales
// and sums at + b * a_stride elements, and writes y + b * y_stride floats. count = 1 is a plain call.
struct GemvBatch {
    int count = 1;
    int64_t w_stride = 0, q_stride = 0, a_stride = 0, y_stride = 0;
};
cudaError_t launch_gemv_i2s(const I2sWeight& w, const Q8Act& a, float* y, int64_t ldy, const Epilogue& epi,
                            cudaStream_t st, const GemvBatch& bt = GemvBatch{});

// Tensor-core path. mode 0: Y = W*q (+ epilogue). mode 1 (gate/up): P = relu(Wg*q)^2 * (Wu*q).
// tmap_* are built by the caller (host) for these exact buffers.
struct TcGemmArgs {
    CUtensorMap tmap_w0;  // packed codes of W (or W_gate), 2D u8 [N rows][Kp/4 bytes], box 32 x 128 (64 in mode 1)
    CUtensorMap tmap_w1;  // packed codes of W_up (mode 1), box 32 x 64
    CUtensorMap tmap_q;   // int8 activations 2D [M rows][K], box 128 x bn_sub, 128B swizzle
    CUtensorMap tmap_y;   // mode 1: fp32 output 2D [M rows][N] (row stride ldy), box 64 x 16, for TMA stores
    int y_tma;            // tmap_y is valid (y 16-byte aligned, ldy a multiple of 4)
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
    Epilogue epi;
    int32_t* part;        // split-K partials in global memory (n_tiles * m_tiles * splits * T * 128 int32), or
                          // nullptr for the distributed-shared-memory reduction
};
// Global split-K workspace that covers any tiling of an M-token GEMM with n_out outputs per matrix.
size_t splitk_ws_bytes(int64_t M, int64_t n_out, int rows_per_cta);
cudaError_t launch_gemm_i2s_tc(const TcGemmArgs& args, cudaStream_t st);
// Clusters of `size` (1..8) CTAs of the split-K kernel that fit on the device at once; <= 0 if unknown.
int tc_max_active_clusters(int size);
// Persistent variant (gemm_i2s_tcp.cu): `grid` CTAs walk the n_tiles x m_tiles tiles of T <= 224 tokens
// (splits must be 1; tmap_q's box is 128 x T).
int tcp_max_tokens();
cudaError_t launch_gemm_i2s_tcp(const TcGemmArgs& args, int grid, cudaStream_t st);

cudaError_t launch_repack_rows(const uint8_t* src, uint8_t* dst, int64_t N, int64_t K, cudaStream_t st);

cudaError_t launch_softmax(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N, float scale,
                           float* y, cudaStream_t st);
cudaError_t launch_softmax_rows(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N,
                                float scale, int causal_rows, float* y, cudaStream_t st);

// Model operators (model_ops.cu). kind 0 = RMSNorm, 1 = LayerNorm; quant writes int8 codes + s + sums.
cudaError_t launch_norm(int kind, bool quant, const float* x, int64_t ldx, const float* g, const float* b, float eps,
                        int64_t M, int64_t K, float* y, int64_t ldy, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                        cudaStream_t st);
cudaError_t launch_rope_neox(float* x, int64_t M, int n_heads, int hd, int64_t ld, float base, int pos0,
                             cudaStream_t st);
cudaError_t launch_rope_table(float base, int hd, int n_pos, float2* tab, cudaStream_t st);
cudaError_t launch_rope_apply(float* x, int64_t M, int n_heads, int hd, int64_t ld, const float2* tab, int period,
                              cudaStream_t st);
cudaError_t launch_embed_tokens(const int32_t* tokens, int n, int D, uint32_t seed, float* y, int64_t ldy,
                                cudaStream_t st);
cudaError_t launch_patch_embed(const float* img, int batch, int C, int H, int W, int P, const float* w,
                               const float* bias, const float* pos, int D, float* y, int64_t ldy, cudaStream_t st);
// Fused fp32 attention of `batch` sequences of T tokens (operation order in model_ops.cu). A non-NULL
// `rope` (the launch_rope_table table of at least T positions, 16-byte aligned) applies NEOX RoPE to Q and K
// while they are staged, with the same result as launch_rope_apply(period T) on q and k beforehand; q and k
// in memory are left unrotated.
size_t attention_smem_bytes(int T, int hd);
bool attention_supported(int T, int hd, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo, const void* q,
                         const void* k, const void* v, const void* o);
cudaError_t launch_attention(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                             int batch, int T, int heads, int kv_heads, int hd, float scale, bool causal, float* o,
                             int64_t ldo, cudaStream_t st, const float2* rope = nullptr);

// Tensor-core attention (attention_tc.cu): same contract, products as 3xTF32 on tcgen05, exact-max softmax.
// Needs hd % 8 == 0, hd <= 128, 128 % (heads / kv_heads) == 0, at most 384 keys per query block, leading
// dimensions % 4 == 0 and 16-byte aligned tensors.
bool attention_tc_supported(int T, int heads, int kv_heads, int hd, bool causal, int64_t ldq, int64_t ldk, int64_t ldv,
                            int64_t ldo, const void* q, const void* k, const void* v, const void* o);
cudaError_t launch_attention_tc(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                                int batch, int T, int heads, int kv_heads, int hd, float scale, bool causal, float* o,
                                int64_t ldo, cudaStream_t st);

// The library's mul_mat dispatch (b2s status codes; failures recorded for b2s_last_error()).
// path 0 = auto (M <= 16: GEMV, else tensor cores), 1 = GEMV, 2 = tensor cores.
int dispatch_mul_mat_q8(const I2sWeight& w, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums,
                        int64_t M, float* y, int64_t ldy, int path, const Epilogue& epi, cudaStream_t st,
                        void* splitk_ws = nullptr, size_t splitk_bytes = 0);
// FFN gate/up with the squared-ReLU product: p = relu(Wg q)^2 * (Wu q) (tensor cores, mode 1).
int dispatch_gate_up(const I2sWeight& wg, const I2sWeight& wu, const int8_t* q, int64_t ldq, const float* s,
                     const int32_t* sums, int64_t M, float* p, int64_t ldp, cudaStream_t st,
                     void* splitk_ws = nullptr, size_t splitk_bytes = 0);

// Read-only GGUF container (gguf_file.cu): memory-mapped, metadata parsed, tensors indexed by name.
struct GgufValue {
    uint32_t type = 0;
    uint8_t raw[8] = {};
    std::string s;
    uint32_t arr_type = 0;
    uint64_t arr_n = 0;
    const void* arr = nullptr;
};
struct GgufTensor {
    int64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;  // ggml type id (0 F32, 36 I2_S)
    uint64_t offset = 0;
    size_t nbytes = 0;
    const uint8_t* data = nullptr;
};
class GgufFile {
  public:
    GgufFile() = default;
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;
    ~GgufFile();
    bool open(const char* path, std::string* err);
    void close();
    const GgufTensor* tensor(const std::string& name) const;
    bool u32(const std::string& key, uint32_t* out) const;
    bool f32(const std::string& key, float* out) const;
    bool str(const std::string& key, std::string* out) const;
    size_t n_tensors() const { return tensors_.size(); }

  private:
    const void* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::map<std::string, GgufTensor> tensors_;
};

// Records `msg` as the calling thread's b2s_last_error() and returns `code`.
int set_last_error(int code, const char* msg);

// Scratch bytes the MUL_MAT node needs for its int8 activations, scales and sums (same layout as the
// caller workspace of b2s_mul_mat) in *need; returns the same status (and message) b2s_mul_mat gives a
// malformed W or X.
int mul_mat_scratch_bytes(const void* W, const void* X, size_t* need);

// The MUL_MAT node of b2s_mul_mat run into a scratch region the caller already owns
// (`scratch` device pointer, `capacity` bytes, 256-byte aligned): the activation layout first, the rest
// for split-K partials. Validates exactly like b2s_mul_mat.
int mul_mat_into_scratch(const void* W, const void* X, void* Y, void* scratch, size_t capacity, cudaStream_t st);

}  // namespace b2s
