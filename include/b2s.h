/*
 * b2s.h -- C ABI of the B200 (sm_100a) ternary i2_s mul_mat library (libb2s.so).
 *
 * Drop-in boundary for one node type of a ggml graph: MUL_MAT with an i2_s (2-bit ternary, one fp32
 * scale per tensor) weight, as a BitVLA engine would emit it at every linear layer, e.g.
 *   ggml_tensor * q = ggml_mul_mat(ctx0, layer.wq, cur);       (src/models/pi0/vlm.cpp:217-223 pattern)
 * plus the neighbouring nodes that produce and consume its activations (RMSNorm + ggml_mul,
 * squared-ReLU gate product, soft_max_ext). Everything is plain C: pointers, sizes, status codes.
 *
 * Conventions (ggml's):
 *   - A tensor is described by b2s_tensor {type, ne[4], nb[4], data}; ne[0] is the innermost
 *     (contiguous) dimension, nb[] are byte strides (src/models/smolvla/vision.cpp:477-480 builds
 *     weights as ne = [in_features, out_features]).
 *   - mul_mat(W, X): W ne=[K,N] (i2_s), X ne=[K,M] f32 -> Y ne=[N,M] f32, Y[m][n] = sum_k W[n][k] X[m][k]
 *     through per-token int8 quantization of X (see b2s_act_quant).
 *   - Every data pointer passed to an entry point that takes a stream is DEVICE memory of the current
 *     CUDA device; `stream` is a cudaStream_t (NULL = legacy default stream).
 *   - Calls never abort and never throw. They return B2S_OK (0) or a negative b2s_status; the message
 *     of the last failure on the calling thread is b2s_last_error(). Shape, type and alignment errors
 *     are reported before anything is launched.
 *   - Entry points that take a stream only enqueue work; a bounded wait that ran out inside a kernel
 *     is reported by b2s_device_error() after the stream is synchronized.
 *
 * i2_s byte layout (flattened over the tensor, n = ne0*ne1 a multiple of 128): weight g = r*K + k is the
 * 2-bit code at bit shift 6-2*((g%128)/32) of byte 32*(g/128) + (g%128)%32; codes 0,1,2 mean -1,0,+1;
 * the n/4 code bytes are followed by 32 bytes whose first four hold the fp32 scale. nbytes = n/4 + 32.
 * This is the x86 I2_S layout of microsoft/BitNet's ggml fork (quantize_i2_s), which the reference
 * would load through gguf_loader::load as opaque ggml_nbytes() bytes (src/models/gguf_loader.cpp:115-137).
 */
#ifndef B2S_H
#define B2S_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2S_VERSION_MAJOR 0
#define B2S_VERSION_MINOR 1

typedef enum b2s_status {
    B2S_OK = 0,
    B2S_ERR_INVALID_ARG = -1,    /* null pointer, bad shape, inconsistent strides */
    B2S_ERR_UNSUPPORTED = -2,    /* type / layout / alignment this op does not implement */
    B2S_ERR_WORKSPACE = -3,      /* workspace missing or smaller than b2s_mul_mat_workspace_size() */
    B2S_ERR_CUDA = -4,           /* CUDA runtime or launch error (message has the CUDA error string) */
    B2S_ERR_DEVICE = -5,         /* current device is not an sm_100 (B200-class) GPU */
    B2S_ERR_DEVICE_TIMEOUT = -6  /* a kernel's bounded wait ran out (see b2s_device_error) */
} b2s_status;

/* Tensor types. F32/I8/I32 keep ggml's numeric ids (GGML_TYPE_F32=0, I8=24, I32=26). I2_S is the
 * flattened BitNet-fork layout above; I2_S_R is this library's row-padded device layout (each row
 * padded to a multiple of 128 weights with zero codes, scale after the codes), produced by
 * b2s_i2s_repack_rows and required when ne0 % 128 != 0. For ne0 % 128 == 0 the two are identical. */
typedef enum b2s_type {
    B2S_TYPE_F32 = 0,
    B2S_TYPE_I8 = 24,
    B2S_TYPE_I32 = 26,
    B2S_TYPE_I2_S = 36,
    B2S_TYPE_I2_S_R = 1036
} b2s_type;

/* Mirrors the fields of ggml_tensor that an op reads: type, ne[4], nb[4], data. */
typedef struct b2s_tensor {
    int32_t type;
    int64_t ne[4];
    size_t nb[4];
    void *data;
} b2s_tensor;

/* ---------------------------------------------------------------- library / errors */
const char *b2s_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char *b2s_last_error(void);
/* B2S_OK if the current CUDA device is sm_100 (compute capability 10.0). */
int b2s_device_check(void);
/* Reads (and with clear != 0 resets) the device error word of the current device: bit 0 = a pipeline
 * wait timed out, bit 1 = a drain wait at kernel exit timed out. Synchronous. */
int b2s_device_error(uint32_t *out_bits, int clear);

/* Test hook for the failure path of the kernels' bounded waits (no counterpart in the reference; failure
 * detection in the style of its bool/status-plus-message checks). Launches one CTA on `stream` that holds
 * what a GEMM CTA holds -- 32 tensor-memory columns and one bulk copy of `bytes` bytes of src (device memory,
 * 16-byte aligned, 16..4096 bytes, a multiple of 16) in flight -- then waits on an mbarrier that nothing
 * arrives at, bounded by wait_limit_ns (at most one second). When the wait runs out the kernel sets bit 0
 * of the device error word, waits (bounded) for its copy to land, frees its tensor memory and returns: the
 * sequence every pipelined kernel follows on a timeout. Read the result with b2s_device_error. */
int b2s_debug_wait_timeout(const void *src, size_t bytes, uint64_t wait_limit_ns, void *stream);

/* ---------------------------------------------------------------- i2_s type traits (host) */
/* Bytes of an i2_s tensor of nrow rows x n_per_row weights (ggml_nbytes for GGML_TYPE_I2_S). */
size_t b2s_i2s_nbytes(int64_t nrow, int64_t n_per_row);
/* Bytes of the row-padded device layout. */
size_t b2s_i2s_r_nbytes(int64_t nrow, int64_t n_per_row);
/* from_float trait (host): pack float weights that are already ternary times a scale; the scale is
 * max|w| and |w| < 1e-6 counts as zero. Returns nbytes, or 0 if nrow*n_per_row % 128 != 0.
 * Replaces the fork's quantize_i2_s as called by a converter (cf. the ctypes bulk-quantizer of
 * tools/quant/quantize-vla-gguf.py:335-360). */
size_t b2s_i2s_quantize(const float *src, void *dst, int64_t nrow, int64_t n_per_row);
/* to_float trait (host): dst = t * scale. Returns 0 on success, negative on bad arguments. */
int b2s_i2s_dequantize(const void *src, float *dst, int64_t nrow, int64_t n_per_row);

/* ---------------------------------------------------------------- device entry points */
/* Load-time repack (device): flattened i2_s -> row-padded I2_S_R. dst holds b2s_i2s_r_nbytes bytes. */
int b2s_i2s_repack_rows(const void *src, void *dst, int64_t nrow, int64_t n_per_row, void *stream);

/* Per-token act-quant (the vec_dot_type conversion of src1 inside MUL_MAT):
 *   s[m] = 127 / max(1e-5, max_k |x[m,k]|), q[m,k] = clamp(round_half_away(x*s), -128, 127),
 *   sums[m] = sum_k q[m,k] (sums may be NULL). x rows have stride ldx floats, q rows ldq bytes. */
int b2s_act_quant(const float *x, int64_t M, int64_t K, int64_t ldx, int8_t *q, int64_t ldq, float *s,
                  int32_t *sums, void *stream);

/* RMSNorm + weight + act-quant in one pass (ggml_rms_norm(x, eps) then ggml_mul(., g) then the
 * act-quant above; src/models/smolvla/action_expert.cpp:731-736). g may be NULL (no weight). The
 * normalized fp32 row is not written. */
int b2s_rms_norm_act_quant(const float *x, const float *g, int64_t M, int64_t K, int64_t ldx, float eps,
                           int8_t *q, int64_t ldq, float *s, int32_t *sums, void *stream);

/* Workspace bytes b2s_mul_mat needs for these operands: int8 activations, scales and sums, then room for
 * the split-K partials of small-M launches (those reduce through L2 when the room is there, through
 * distributed shared memory otherwise). Any size >= the activation part is accepted. */
size_t b2s_mul_mat_workspace_size(const b2s_tensor *W, const b2s_tensor *X);

/* The MUL_MAT node: Y = mul_mat(W, X). W: I2_S (ne0 % 128 == 0) or I2_S_R, ne=[K,N], contiguous (or
 * ne=[K,N,B] with X ne=[K,M,B] and Y ne=[N,M,B]: ggml's batched matmul, see b2s_mul_mat_q8_batched);
 * X: F32 ne=[K,M], rows contiguous (nb[0] = 4); Y: F32 ne=[N,M], rows contiguous. Uses the caller's
 * workspace for the quantized activations; allocates nothing. Decode sizes run a GEMV (M = 1: dp4a on
 * CUDA cores; M = 2..16: warp-level int8 MMAs), larger M the tcgen05 tensor-core GEMM. */
int b2s_mul_mat(const b2s_tensor *W, const b2s_tensor *X, b2s_tensor *Y, void *workspace, size_t workspace_bytes,
                void *stream);

/* The MUL_MAT node of b2s_mul_mat for callers that cannot allocate: no workspace argument, and the call
 * allocates nothing. This entry point has no counterpart in the reference. It serves code that owns no
 * device workspace and must not call cudaMalloc while it runs: an op inside a ggml backend's compute step
 * (the scheduler has already allocated every buffer and hands the op no allocator), or a robot control
 * loop past start-up (cudaMalloc can synchronize the device and adds latency jitter). The quantized
 * activations go to a library-owned 4 MiB static device array instead (held by every GPU that loads the
 * library until the process exits). Limit: the call's activation scratch, a256(M*roundup(K,16)) +
 * a256(4*M) + a256(4*M) bytes (a256 = rounded up to a multiple of 256), must be at most 4 MiB, else
 * B2S_ERR_WORKSPACE and nothing is launched; the rest of the array holds split-K partials, so the kernels
 * are the ones b2s_mul_mat picks with a full workspace. Malformed W/X/Y get the status b2s_mul_mat gives.
 * The first call on a device looks up the array's address and caches it for the process; make it before
 * any stream capture, and do not reset the device afterwards. All calls on a device share the array:
 * calls that overlap on the GPU race, so serialize them. */
int b2s_mul_mat_static(const b2s_tensor *W, const b2s_tensor *X, b2s_tensor *Y, void *stream);

/* MUL_MAT on already-quantized activations (producer-fused path): q [M x ldq] int8 (ldq % 16 == 0,
 * 16-byte aligned), s [M], sums [M] from b2s_act_quant / b2s_rms_norm_act_quant. Y [M x ldy] f32. */
int b2s_mul_mat_q8(const b2s_tensor *W, const int8_t *q, int64_t ldq, const float *s, const int32_t *sums,
                   int64_t M, float *Y, int64_t ldy, void *stream);
/* ggml's batched MUL_MAT (ne[2] > 1) on quantized activations: B independent problems, problem b = weight
 * matrix b times activations b. W ne=[K,N,B] (I2_S with K % 128 == 0, or I2_S_R): the B matrices back to back
 * (nb[2] = N*K/4 bytes, N*Kp/4 row-padded) sharing the tensor's one fp32 scale, which follows all B*N rows
 * (the flattened i2_s layout over B*N rows). Activations of problem b at q + b*q_bstride bytes, scales and sums
 * at + b*a_bstride elements; outputs at Y + b*y_bstride floats. Decode sizes (M <= 16) stream every matrix in
 * one GEMV launch (grid over rows x problems); larger M runs one tensor-core GEMM per matrix. */
int b2s_mul_mat_q8_batched(const b2s_tensor *W, const int8_t *q, int64_t ldq, int64_t q_bstride, const float *s,
                           const int32_t *sums, int64_t a_bstride, int64_t M, float *Y, int64_t ldy, int64_t y_bstride,
                           void *stream);
/* Same with the kernel chosen explicitly: path 0 = automatic, 1 = GEMV (any M, run in token groups of up to
 * 16: one token on dp4a, 2..16 on warp int8 MMAs), 2 = tcgen05 tensor-core GEMM (any M). For tests and
 * tuning; results are identical. */
int b2s_mul_mat_q8_ex(const b2s_tensor *W, const int8_t *q, int64_t ldq, const float *s, const int32_t *sums,
                      int64_t M, float *Y, int64_t ldy, int path, void *stream);

/* FFN gate/up with the squared-ReLU gate product fused into the epilogue:
 *   P[m,n] = relu(G)^2 * U,  G = mul_mat(W_gate, X), U = mul_mat(W_up, X)  (ggml_relu, ggml_sqr,
 *   ggml_mul in a BitNet-style FFN), from quantized activations as in b2s_mul_mat_q8. */
int b2s_ffn_gate_up_sqrelu_q8(const b2s_tensor *W_gate, const b2s_tensor *W_up, const int8_t *q, int64_t ldq,
                              const float *s, const int32_t *sums, int64_t M, float *P, int64_t ldp, void *stream);

/* Workspace bytes for b2s_ffn_block with M tokens, hidden H and FFN width F. */
size_t b2s_ffn_block_workspace_size(int64_t M, int64_t H, int64_t F);

/* Whole FFN block: Y = down(rms_norm2(relu(gate(xn))^2 * up(xn))), xn = rms_norm1(X); the BitNet
 * FFN (RMSNorm(H) -> gate/up H->F -> squared-ReLU product -> RMSNorm(F) -> down F->H). X, Y [M x H]
 * f32 contiguous; g1 [H], g2 [F] norm weights (may be NULL). Four kernel launches, no allocation. */
int b2s_ffn_block(const float *X, int64_t M, const float *g1, const float *g2, float eps, const b2s_tensor *W_gate,
                  const b2s_tensor *W_up, const b2s_tensor *W_down, float *Y, void *workspace,
                  size_t workspace_bytes, void *stream);

/* MUL_MAT on quantized activations with a fused epilogue, applied in this order to y = acc*w_scale/s[m]:
 * y += bias[n] (bias may be NULL); y = gelu_tanh(y) if act == 1 (ggml_gelu, tanh approximation);
 * y = residual[m*ld_res + n] + y (residual may be NULL; it may alias Y). Covers the ggml_add(bias),
 * ggml_gelu and residual ggml_add nodes that follow a linear layer (src/models/smolvla/vision.cpp:314-345). */
int b2s_mul_mat_q8_epi(const b2s_tensor *W, const int8_t *q, int64_t ldq, const float *s, const int32_t *sums,
                       int64_t M, float *Y, int64_t ldy, const float *bias, const float *residual, int64_t ld_res,
                       int act, void *stream);

/* Normalization of M rows of K floats, written as fp32: kind 0 = ggml_rms_norm, kind 1 = ggml_norm
 * (LayerNorm), then * g (ggml_mul, g may be NULL) and + b (ggml_add, b may be NULL). eps as in ggml. */
int b2s_norm(const float *x, const float *g, const float *b, int64_t M, int64_t K, int64_t ldx, float eps, int kind,
             float *y, int64_t ldy, void *stream);
/* The same normalization followed by the per-token act-quant (b2s_act_quant semantics). */
int b2s_norm_act_quant(const float *x, const float *g, const float *b, int64_t M, int64_t K, int64_t ldx, float eps,
                       int kind, int8_t *q, int64_t ldq, float *s, int32_t *sums, void *stream);

/* In-place NEOX rotary embedding (ggml_rope_ext, mode NEOX; src/models/pi0/vlm.cpp:223-235) of M rows of
 * n_heads heads of head_dim floats at row stride ld; token m has position pos0 + m. */
int b2s_rope_neox(float *x, int64_t M, int n_heads, int head_dim, int64_t ld, float theta_base, int pos0, void *stream);

/* Multi-head attention softmax(Q K^T * scale [+ causal mask]) V over M tokens, fp32, with n_heads query
 * heads sharing n_kv_heads key/value heads (GQA; n_heads % n_kv_heads == 0). Q/K/V/O rows hold the heads
 * side by side (head h at columns [h*head_dim, (h+1)*head_dim)). The ggml sequence mul_mat(K, Q) ->
 * soft_max_ext -> mul_mat(V, KQ) (src/models/smolvla/action_expert.cpp:771-774) as one fused kernel with
 * an online softmax over chunks of 64 keys (the evaluation order of ggml_flash_attn_ext, used by
 * src/models/pi0/vlm.cpp) in a fixed fp32 operation order: scores are fma-accumulated dot products
 * (d ascending) times scale; per chunk the running max, the rescale det_exp(m - m'), the chunk's
 * probabilities and its sum (fixed butterfly order) update l and the fma-accumulated outputs; outputs are
 * finally multiplied by 1/l. Needs head_dim % 8 == 0, head_dim <= 128, leading dimensions % 4 == 0 and
 * 16-byte aligned tensors (B2S_ERR_UNSUPPORTED otherwise); any M. */
int b2s_attention(const float *q, int64_t ldq, const float *k, int64_t ldk, const float *v, int64_t ldv, int64_t M,
                  int n_heads, int n_kv_heads, int head_dim, float scale, int causal, float *o, int64_t ldo,
                  void *stream);

/* The same attention on the tcgen05 tensor cores. Products are 3xTF32 (each fp32 operand split into a TF32
 * part and its fp32 remainder; big*big + big*small + small*big accumulated in fp32, about 2^-21 relative
 * error per product) and the softmax takes the exact row maximum before exponentiating (exp2 on the
 * special-function unit), so results match b2s_attention to about 1e-6 relative, not bit for bit. One CTA
 * holds 128 rows = (n_heads / n_kv_heads) query heads x the queries of a block, sharing one K/V head.
 * Needs head_dim % 8 == 0 and <= 128, 128 % (n_heads / n_kv_heads) == 0, at most 384 keys visible to a
 * query block (M <= 384 without the causal mask), leading dimensions % 4 == 0 and 16-byte aligned tensors
 * (B2S_ERR_UNSUPPORTED otherwise). */
int b2s_attention_tc(const float *q, int64_t ldq, const float *k, int64_t ldk, const float *v, int64_t ldv, int64_t M,
                     int n_heads, int n_kv_heads, int head_dim, float scale, int causal, float *o, int64_t ldo,
                     void *stream);

/* Patch embedding of a CHW fp32 image: non-overlapping P x P patches (row-major patch order) times the
 * [D][C*P*P] weight, plus bias[D] and the position embedding pos[n_patches][D] (either may be NULL):
 * y = (bias + pos) + acc, acc fma-accumulated over k = c*P*P + ky*P + kx ascending. */
int b2s_patch_embed(const float *img, int C, int H, int W, int P, const float *w, const float *bias, const float *pos,
                    int D, float *y, int64_t ldy, void *stream);

/* Random-init token embeddings: y[i][c] = -0.02 + 0.04 * ((b2s_bitvla_param_bits(seed, 0x80000000 | tokens[i], c)
 * >> 8) * 2^-24) for c < dim, fp32 (the BitVLA engine's text embedding; no 128256-row table is materialized). */
int b2s_embed_tokens_hash(const int32_t *tokens, int n, int dim, uint32_t seed, float *y, int64_t ldy, void *stream);

/* ggml_soft_max_ext(x, mask, scale, 0.0f): y[m,:] = softmax(x[m,:]*scale + mask[m % mask_rows,:]).
 * mask may be NULL. Rows contiguous, N columns (src/models/smolvla/action_expert.cpp:773). */
int b2s_soft_max_ext(const float *x, const float *mask, int64_t mask_rows, int64_t M, int64_t N, float scale,
                     float *y, void *stream);

/* ---------------------------------------------------------------- N-split over several GPUs (host side)
 * A MUL_MAT of very many tokens split over the output rows of W across g GPUs (one process per GPU): rank r
 * computes Y[:, n0_r:n1_r) and its GEMM epilogue stores the slice straight into the root GPU's output over
 * NVLink (plain peer stores; no gather kernel, no collective). The root exports its output buffer with
 * b2s_peer_export, the handle's 72 bytes reach the other ranks by any transport, each opens it with
 * b2s_peer_open and passes (peer_ptr + n0_r floats, ldy = N) as the Y of b2s_mul_mat_q8. The reference
 * has no multi-GPU path (one ggml CUDA backend on device 0, src/models/ggml_backend.cpp:62-202); these
 * calls are the plumbing that replaces a ggml tensor split plus gather for this op. */
#define B2S_PEER_HANDLE_BYTES 72
/* Balanced contiguous split of n_rows over `world` ranks: rank gets [*n0, *n1) (sizes differ by <= 1). */
int b2s_nsplit_range(int64_t n_rows, int world, int rank, int64_t *n0, int64_t *n1);
/* Host: rows [r0, r1) of an I2_S (n_per_row % 128 == 0) or I2_S_R tensor as a standalone tensor of the same
 * type (code bytes, then the 32-byte trailer with the fp32 scale) at dst. Returns the bytes written, 0 on
 * error. */
size_t b2s_i2s_shard_rows(const void *src, int32_t type, int64_t nrow, int64_t n_per_row, int64_t r0, int64_t r1,
                          void *dst);
/* Export of a device buffer of the current device into B2S_PEER_HANDLE_BYTES bytes: the CUDA IPC handle of the
 * allocation that contains dev_ptr and dev_ptr's offset in it (so pointers from a sub-allocating allocator
 * work). */
int b2s_peer_export(const void *dev_ptr, void *handle, size_t handle_bytes);
/* Maps a peer's exported allocation into the current device's address space (peer access enabled). */
int b2s_peer_open(const void *handle, size_t handle_bytes, void **dev_ptr);
/* Unmaps a pointer returned by b2s_peer_open (B2S_ERR_INVALID_ARG for any other pointer). */
int b2s_peer_close(void *dev_ptr);

#ifdef __cplusplus
}
#endif
#endif /* B2S_H */
