// bitvla_engine.cu -- random-init BitVLA-shape forward on the library's kernels (C ABI in b2s_bitvla.h).
//
// Per observation: patch embedding (the library's fixed-order fp32 kernel) -> vit_layers x ViT block ->
// post-LayerNorm ->
// two-layer ternary connector -> [image tokens | hash-embedded text tokens] -> dec_layers x decoder layer
// -> final RMSNorm -> linear action head on the last token. The ViT block mirrors
// src/models/smolvla/vision.cpp:305-345, the decoder layer src/models/pi0/vlm.cpp:196-246, with every
// linear layer a ternary i2_s weight and BitNet b1.58's sub-norms in front of o and down.
//
// Every linear layer runs through the library's int8 activation path: the producer kernel (norm or
// act-quant) writes int8 codes + per-token scale + code sum, the ternary GEMM consumes them, and the
// GEMM's epilogue adds bias and adds the residual in place; GELU runs in the act-quant kernel that reads
// the GEMM output for the next layer. q/k/v of a layer are one stacked ternary weight (each part keeps its
// own scale), so one GEMM produces [q | k | v] rows, and the fp32 attention kernel rotates the q and k heads
// (RoPE) as it stages them. Attention is one fused fp32 kernel over all
// (query block, head, observation) triples of the batch.
//
// HBM layout: one arena for all weights (packed ternary rows padded to 128 weights, scales, fp32
// parameters) and one for the activation buffers of max_batch observations; a batch of B observations
// is B stacked row blocks in every activation buffer. The forward for each batch size is captured once
// into a CUDA graph (programmatic dependent launch edges between the library kernels) and replayed.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <vector>

#include "b2s.h"
#include "b2s_bitvla.h"
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace {

using b2s::ceil_div;
using b2s::round_up;

// ------------------------------------------------------------------------------------------ parameters
using b2s::param_bits;  // generator shared with the token embedding (b2s_common.cuh)
constexpr uint32_t kTernLo = 5033165u;   // 0.3 * 2^24 (rounded up): u < kTernLo -> -1
constexpr uint32_t kTernHi = 11744051u;  // 0.7 * 2^24 (rounded down): u < kTernHi -> 0, else +1

// Tensor ids: global tensors, then 16 slots per ViT layer and per decoder layer.
enum : uint32_t {
    kIdPatchW = 1, kIdPatchB, kIdPos, kIdPostW, kIdPostB, kIdConn1, kIdConn1B, kIdConn2, kIdConn2B, kIdFinalNorm,
    kIdActW, kIdActB
};
inline uint32_t vit_id(int l, int slot) { return 0x100u + 16u * (uint32_t)l + (uint32_t)slot; }
inline uint32_t dec_id(int l, int slot) { return 0x10000u + 16u * (uint32_t)l + (uint32_t)slot; }
enum VitSlot { kVLn1W, kVLn1B, kVQ, kVK, kVV, kVQB, kVKB, kVVB, kVO, kVOB, kVLn2W, kVLn2B, kVFc1, kVFc1B, kVFc2, kVFc2B };
enum DecSlot { kDAttnNorm, kDQ, kDK, kDV, kDAttnSub, kDO, kDFfnNorm, kDGate, kDUp, kDFfnSub, kDDown };

// Per-tensor ternary scale: U(0.5, 2) / sqrt(0.6 K) (0.6 = P(w != 0)), fp32 host arithmetic.
float ternary_scale(uint32_t seed, uint32_t tensor, int64_t K) {
    const float u = (float)(param_bits(seed, tensor, 0xFFFFFFFFu) >> 8) * (1.0f / 16777216.0f);
    const float a = 0.5f + 1.5f * u;
    const float r = sqrtf(0.6f * (float)K);
    return a / r;
}

// Rows [0, rows) of tensor `tensor` (K weights each) into row-padded i2_s bytes (Kp/4 per row,
// pad code 1 = 0). One thread per output byte; byte j of a row holds weights 128(j/32) + 32g + j%32.
__global__ void gen_ternary_kernel(uint8_t* __restrict__ dst, int64_t rows, int64_t K, int64_t Kp, uint32_t seed,
                                   uint32_t tensor) {
    const int64_t rb = Kp / 4, total = rows * rb;
    for (int64_t d = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; d < total; d += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = d / rb, off = d - r * rb;
        const int64_t b = off / 32, i = off % 32;
        uint32_t out = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int64_t k = 128 * b + 32 * g + i;
            uint32_t code = 1;
            if (k < K) {
                const uint32_t u = param_bits(seed, tensor, (uint32_t)(r * K + k)) >> 8;
                code = (u < kTernLo) ? 0u : (u < kTernHi ? 1u : 2u);
            }
            out |= code << (6 - 2 * g);
        }
        dst[d] = (uint8_t)out;
    }
}

__global__ void gen_uniform_kernel(float* __restrict__ dst, int64_t n, uint32_t seed, uint32_t tensor, float lo,
                                   float width) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float u = (float)(param_bits(seed, tensor, (uint32_t)i) >> 8) * (1.0f / 16777216.0f);
        dst[i] = __fadd_rn(lo, __fmul_rn(width, u));
    }
}

// ------------------------------------------------------------------------------------------ small kernels
// Text-token embedding rows: token i of observation b goes to row b * seq + n_img + i.
__global__ void embed_text_kernel(const int32_t* __restrict__ tokens, int batch, int n_text, int n_img, int seq,
                                  int D, uint32_t seed, float* __restrict__ y) {
    const int64_t total = (int64_t)batch * n_text * D;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e % D);
        const int64_t t = e / D;
        const int b = (int)(t / n_text), i = (int)(t % n_text);
        const uint32_t tok = (uint32_t)tokens[t];
        const float u = (float)(param_bits(seed, 0x80000000u | tok, (uint32_t)c) >> 8) * (1.0f / 16777216.0f);
        y[((int64_t)b * seq + n_img + i) * D + c] = __fadd_rn(-0.02f, __fmul_rn(0.04f, u));
    }
}

// Action head: actions[b][j] = bias[j] + sum_c h[b * seq + seq - 1][c] * W[j][c]; one warp per output,
// lane l sums c = l, l + 32, ... in fp32 (multiply, then add), then an xor-butterfly over the lanes.
__global__ void action_head_kernel(const float* __restrict__ h, int batch, int seq, int D, const float* __restrict__ W,
                                   const float* __restrict__ bias, int A, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (o >= batch * A) return;
    const int b = o / A, j = o % A;
    const float* hr = h + ((int64_t)b * seq + seq - 1) * D;
    const float* wr = W + (int64_t)j * D;
    float acc = 0.0f;
    for (int c = lane; c < D; c += 32) acc = __fadd_rn(acc, __fmul_rn(hr[c], wr[c]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    if (lane == 0) out[o] = __fadd_rn(acc, bias[j]);
}

// uint8 HWC images (value / 255) -> fp32 CHW.
__global__ void image_u8_kernel(const uint8_t* __restrict__ src, int batch, int S, float* __restrict__ dst) {
    const int64_t total = (int64_t)batch * 3 * S * S;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int x = (int)(e % S);
        const int y = (int)((e / S) % S);
        const int c = (int)((e / ((int64_t)S * S)) % 3);
        const int64_t b = e / (3LL * S * S);
        dst[e] = __fdiv_rn((float)src[((b * S + y) * S + x) * 3 + c], 255.0f);
    }
}

unsigned grid_of(int64_t total) {
    const int64_t b = (total + 255) / 256;
    return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

// ------------------------------------------------------------------------------------------ model
struct Tern {  // ternary weight, possibly several tensors stacked by rows (scale per 128-row tile)
    b2s::I2sWeight w{};
    float* scales = nullptr;
};

struct VitLayer {
    float *ln1_w, *ln1_b, *qkv_b, *o_b, *ln2_w, *ln2_b, *fc1_b, *fc2_b;
    Tern qkv, o, fc1, fc2;
};
struct DecLayer {
    float *attn_norm, *attn_sub, *ffn_norm, *ffn_sub;
    Tern qkv, o, gate, up, down;
};

struct Graph {
    cudaGraphExec_t exec = nullptr;
};

// Bump allocator over one cudaMalloc: sized by a first pass with base == nullptr.
struct Arena {
    uint8_t* base = nullptr;
    size_t off = 0;
    void* take(size_t bytes) {
        const size_t o = (off + 255) & ~size_t(255);
        off = o + bytes;
        return base ? base + o : nullptr;
    }
    template <typename T>
    T* arr(size_t n) {
        return static_cast<T*>(take(n * sizeof(T)));
    }
};

int errf(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return b2s::set_last_error(code, buf);
}
int cuda_err(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return B2S_OK;
    (void)cudaGetLastError();
    return errf(B2S_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define TRY_CUDA(expr, what)                                  \
    do {                                                      \
        int rc_ = cuda_err((expr), what);                     \
        if (rc_) return rc_;                                  \
    } while (0)
#define TRY_B2S(expr)          \
    do {                       \
        int rc_ = (expr);      \
        if (rc_) return rc_;   \
    } while (0)

}  // namespace

struct b2s_bitvla {
    b2s_bitvla_config cfg{};
    uint32_t seed = 0;
    int device = 0, max_batch = 0;
    int np = 0, seq = 0, ldq = 0;
    size_t ternary_bytes = 0;
    void* wmem = nullptr;
    size_t wbytes = 0;
    void* amem = nullptr;
    size_t abytes = 0;
    void* splitk_ws = nullptr;  // split-K partials of the GEMMs (global memory, reused by every launch)
    size_t splitk_bytes = 0;
    // weights
    float *patch_w = nullptr, *patch_b = nullptr, *pos = nullptr, *post_w = nullptr, *post_b = nullptr;
    float *conn1_b = nullptr, *conn2_b = nullptr, *final_norm = nullptr, *act_w = nullptr, *act_b = nullptr;
    Tern conn1, conn2;
    std::vector<VitLayer> vit;
    std::vector<DecLayer> dec;
    float2* rope = nullptr;
    // activations (max_batch observations)
    float *img = nullptr, *vx = nullptr, *vqkv = nullptr, *vattn = nullptr, *vh = nullptr, *ch = nullptr;
    float *dx = nullptr, *dqkv = nullptr, *dattn = nullptr, *dp = nullptr, *hidden = nullptr, *actions = nullptr;
    int32_t* tok = nullptr;
    int8_t* q8 = nullptr;
    float* qs = nullptr;
    int32_t* qsum = nullptr;
    // host staging for predict
    uint8_t* h_img = nullptr;
    int32_t* h_tok = nullptr;
    float* h_act = nullptr;
    uint8_t* d_img_u8 = nullptr;
    std::map<int, Graph> graphs;
    std::mutex mu;
};

namespace {

int check_cfg(const b2s_bitvla_config& c) {
    if (c.image_size <= 0 || c.patch <= 0 || c.image_size % c.patch) return errf(B2S_ERR_INVALID_ARG, "image_size % patch != 0");
    if (c.vit_layers < 0 || c.dec_layers < 0) return errf(B2S_ERR_INVALID_ARG, "negative layer count");
    if (c.vit_hidden <= 0 || c.vit_hidden % 128 || c.vit_heads <= 0 || c.vit_hidden % c.vit_heads)
        return errf(B2S_ERR_UNSUPPORTED, "vit_hidden must be a multiple of 128 and of vit_heads");
    if (c.dec_heads <= 0 || c.dec_kv_heads <= 0 || c.dec_heads % c.dec_kv_heads || c.head_dim <= 0 || c.head_dim % 2)
        return errf(B2S_ERR_INVALID_ARG, "bad decoder head layout");
    if (c.dec_heads * c.head_dim != c.dec_hidden || (c.dec_kv_heads * c.head_dim) % 128 || c.dec_hidden % 128)
        return errf(B2S_ERR_UNSUPPORTED, "dec_hidden = dec_heads * head_dim and the k/v width must be multiples of 128");
    if (c.vit_ffn <= 0 || c.dec_ffn <= 0 || c.conn_hidden <= 0 || c.vit_ffn % 16 || c.dec_ffn % 16 || c.conn_hidden % 16)
        return errf(B2S_ERR_UNSUPPORTED, "FFN / connector widths must be multiples of 16");
    if (c.vocab <= 0 || c.n_text < 0 || c.action_chunk <= 0 || c.action_dim <= 0)
        return errf(B2S_ERR_INVALID_ARG, "bad vocab / n_text / action shape");
    return B2S_OK;
}

// Where the weights come from: the seeded generator or a GGUF file. Tensor names are the ones written by
// b2s/gguf.py (llama.cpp conventions: "v.blk.N.*" for the vision tower, "blk.N.*" for the decoder).
struct WeightSource {
    virtual ~WeightSource() = default;
    // Rows [0, rows) of ternary tensor (id, name) with K inputs, as row-padded codes at dst (Kp/4 bytes
    // per row, pad code 1); its fp32 scale in *scale.
    virtual int ternary(uint8_t* dst, int64_t rows, int64_t K, uint32_t id, const std::string& name, float* scale,
                        cudaStream_t st) = 0;
    virtual int uniform(float* dst, int64_t n, uint32_t id, const std::string& name, float lo, float hi,
                        cudaStream_t st) = 0;
};

struct GenSource : WeightSource {
    uint32_t seed;
    explicit GenSource(uint32_t s) : seed(s) {}
    int ternary(uint8_t* dst, int64_t rows, int64_t K, uint32_t id, const std::string&, float* scale,
                cudaStream_t st) override {
        *scale = ternary_scale(seed, id, K);
        const int64_t Kp = round_up(K, (int64_t)128);
        gen_ternary_kernel<<<grid_of(rows * Kp / 4), 256, 0, st>>>(dst, rows, K, Kp, seed, id);
        return cuda_err(cudaGetLastError(), "ternary generation");
    }
    int uniform(float* dst, int64_t n, uint32_t id, const std::string&, float lo, float hi, cudaStream_t st) override {
        gen_uniform_kernel<<<grid_of(n), 256, 0, st>>>(dst, n, seed, id, lo, hi - lo);
        return cuda_err(cudaGetLastError(), "parameter generation");
    }
};

// Tensors of a GGUF file: I2_S (flattened i2_s bytes + scale trailer, repacked to row-padded rows on
// the device through two staging buffers) and F32.
struct GgufSource : WeightSource {
    const b2s::GgufFile* f = nullptr;
    uint8_t* stage_in = nullptr;
    uint8_t* stage_out = nullptr;
    size_t stage_bytes = 0;
    int ternary(uint8_t* dst, int64_t rows, int64_t K, uint32_t, const std::string& name, float* scale,
                cudaStream_t st) override {
        const b2s::GgufTensor* t = f->tensor(name);
        if (!t) return errf(B2S_ERR_INVALID_ARG, "GGUF: missing tensor '%s'", name.c_str());
        if (t->type != 36 || t->ne[0] != K || t->ne[1] != rows || t->ne[2] != 1 || t->ne[3] != 1)
            return errf(B2S_ERR_INVALID_ARG, "GGUF: tensor '%s' must be I2_S [%lld, %lld]", name.c_str(),
                        (long long)K, (long long)rows);
        const int64_t Kp = round_up(K, (int64_t)128);
        if (t->nbytes > stage_bytes || (size_t)(rows * Kp / 4 + 32) > stage_bytes)
            return errf(B2S_ERR_INVALID_ARG, "GGUF: tensor '%s' larger than the staging buffer", name.c_str());
        memcpy(scale, t->data + rows * K / 4, sizeof(float));
        TRY_CUDA(cudaMemcpyAsync(stage_in, t->data, t->nbytes, cudaMemcpyHostToDevice, st), "GGUF upload");
        TRY_CUDA(b2s::launch_repack_rows(stage_in, stage_out, rows, K, st), "GGUF row repack");
        TRY_CUDA(cudaMemcpyAsync(dst, stage_out, (size_t)(rows * Kp / 4), cudaMemcpyDeviceToDevice, st), "GGUF copy");
        return B2S_OK;
    }
    int uniform(float* dst, int64_t n, uint32_t, const std::string& name, float, float, cudaStream_t st) override {
        const b2s::GgufTensor* t = f->tensor(name);
        if (!t) return errf(B2S_ERR_INVALID_ARG, "GGUF: missing tensor '%s'", name.c_str());
        if (t->type != 0 || t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3] != n)
            return errf(B2S_ERR_INVALID_ARG, "GGUF: tensor '%s' must be F32 with %lld elements", name.c_str(),
                        (long long)n);
        TRY_CUDA(cudaMemcpyAsync(dst, t->data, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice, st), "GGUF upload");
        return B2S_OK;
    }
};

struct Part {
    int64_t rows;
    uint32_t id;
    std::string name;
};

// Lays out the weight arena; with a source (and A.base set) it also fills every tensor.
struct Builder {
    Arena& A;
    WeightSource* src;
    cudaStream_t st;
    std::vector<float>* hs;
    std::vector<std::pair<float*, size_t>>* fills;
    size_t* tern_bytes;
    int rc = B2S_OK;

    // Stacked ternary weight of `parts` tensors over K inputs; one scale per 128-row tile.
    void tern(Tern& t, int64_t K, std::initializer_list<Part> parts) {
        int64_t N = 0;
        for (auto& p : parts) N += p.rows;
        t.w.N = N;
        t.w.K = K;
        t.w.Kp = round_up(K, (int64_t)128);
        uint8_t* codes = static_cast<uint8_t*>(A.take((size_t)(N * t.w.Kp / 4)));
        t.scales = A.arr<float>((size_t)ceil_div(N, (int64_t)128));
        *tern_bytes += (size_t)(N * t.w.Kp / 4);
        if (!A.base) return;
        t.w.codes = codes;
        t.w.scale = t.scales;
        const size_t first = hs->size();
        int64_t row0 = 0;
        for (auto& p : parts) {
            float sc = 0.0f;
            if (!rc) rc = src->ternary(codes + row0 * (t.w.Kp / 4), p.rows, K, p.id, p.name, &sc, st);
            for (int64_t r = row0; r < row0 + p.rows; r += 128) hs->push_back(sc);
            row0 += p.rows;
        }
        fills->push_back({t.scales, first});
    }
    float* f32(int64_t n, uint32_t id, const std::string& name, float lo, float hi) {
        float* p = A.arr<float>((size_t)n);
        if (A.base && !rc) rc = src->uniform(p, n, id, name, lo, hi, st);
        return p;
    }
};

std::string vn(int l, const char* what) { return "v.blk." + std::to_string(l) + "." + what; }
std::string dn(int l, const char* what) { return "blk." + std::to_string(l) + "." + what; }

// Lays out (and, with a source, fills) every weight.
int build_weights(b2s_bitvla* m, Arena& A, WeightSource* src, cudaStream_t st, std::vector<float>* hs,
                  std::vector<std::pair<float*, size_t>>* fills) {
    const b2s_bitvla_config& c = m->cfg;
    const int D = c.vit_hidden, P = c.patch, kdim = 3 * P * P;
    const float pa = 1.0f / sqrtf((float)kdim);
    m->ternary_bytes = 0;
    Builder B{A, src, st, hs, fills, &m->ternary_bytes};
    m->patch_w = B.f32((int64_t)D * kdim, kIdPatchW, "v.patch_embd.weight", -pa, pa);
    m->patch_b = B.f32(D, kIdPatchB, "v.patch_embd.bias", -0.02f, 0.02f);
    m->pos = B.f32((int64_t)m->np * D, kIdPos, "v.position_embd.weight", -0.02f, 0.02f);
    m->vit.resize((size_t)c.vit_layers);
    for (int l = 0; l < c.vit_layers; ++l) {
        VitLayer& L = m->vit[(size_t)l];
        L.ln1_w = B.f32(D, vit_id(l, kVLn1W), vn(l, "ln1.weight"), 0.9f, 1.1f);
        L.ln1_b = B.f32(D, vit_id(l, kVLn1B), vn(l, "ln1.bias"), -0.02f, 0.02f);
        B.tern(L.qkv, D, {{D, vit_id(l, kVQ), vn(l, "attn_q.weight")}, {D, vit_id(l, kVK), vn(l, "attn_k.weight")},
                          {D, vit_id(l, kVV), vn(l, "attn_v.weight")}});
        L.qkv_b = B.f32(D, vit_id(l, kVQB), vn(l, "attn_q.bias"), -0.02f, 0.02f);
        B.f32(D, vit_id(l, kVKB), vn(l, "attn_k.bias"), -0.02f, 0.02f);  // contiguous after the q bias
        B.f32(D, vit_id(l, kVVB), vn(l, "attn_v.bias"), -0.02f, 0.02f);
        B.tern(L.o, D, {{D, vit_id(l, kVO), vn(l, "attn_out.weight")}});
        L.o_b = B.f32(D, vit_id(l, kVOB), vn(l, "attn_out.bias"), -0.02f, 0.02f);
        L.ln2_w = B.f32(D, vit_id(l, kVLn2W), vn(l, "ln2.weight"), 0.9f, 1.1f);
        L.ln2_b = B.f32(D, vit_id(l, kVLn2B), vn(l, "ln2.bias"), -0.02f, 0.02f);
        B.tern(L.fc1, D, {{c.vit_ffn, vit_id(l, kVFc1), vn(l, "ffn_up.weight")}});
        L.fc1_b = B.f32(c.vit_ffn, vit_id(l, kVFc1B), vn(l, "ffn_up.bias"), -0.02f, 0.02f);
        B.tern(L.fc2, c.vit_ffn, {{D, vit_id(l, kVFc2), vn(l, "ffn_down.weight")}});
        L.fc2_b = B.f32(D, vit_id(l, kVFc2B), vn(l, "ffn_down.bias"), -0.02f, 0.02f);
    }
    m->post_w = B.f32(D, kIdPostW, "v.post_ln.weight", 0.9f, 1.1f);
    m->post_b = B.f32(D, kIdPostB, "v.post_ln.bias", -0.02f, 0.02f);
    B.tern(m->conn1, D, {{c.conn_hidden, kIdConn1, "mm.0.weight"}});
    m->conn1_b = B.f32(c.conn_hidden, kIdConn1B, "mm.0.bias", -0.02f, 0.02f);
    B.tern(m->conn2, c.conn_hidden, {{c.dec_hidden, kIdConn2, "mm.2.weight"}});
    m->conn2_b = B.f32(c.dec_hidden, kIdConn2B, "mm.2.bias", -0.02f, 0.02f);
    const int H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim;
    m->dec.resize((size_t)c.dec_layers);
    for (int l = 0; l < c.dec_layers; ++l) {
        DecLayer& L = m->dec[(size_t)l];
        L.attn_norm = B.f32(H, dec_id(l, kDAttnNorm), dn(l, "attn_norm.weight"), 0.9f, 1.1f);
        B.tern(L.qkv, H, {{H, dec_id(l, kDQ), dn(l, "attn_q.weight")}, {KV, dec_id(l, kDK), dn(l, "attn_k.weight")},
                          {KV, dec_id(l, kDV), dn(l, "attn_v.weight")}});
        L.attn_sub = B.f32(H, dec_id(l, kDAttnSub), dn(l, "attn_sub_norm.weight"), 0.9f, 1.1f);
        B.tern(L.o, H, {{H, dec_id(l, kDO), dn(l, "attn_output.weight")}});
        L.ffn_norm = B.f32(H, dec_id(l, kDFfnNorm), dn(l, "ffn_norm.weight"), 0.9f, 1.1f);
        B.tern(L.gate, H, {{c.dec_ffn, dec_id(l, kDGate), dn(l, "ffn_gate.weight")}});
        B.tern(L.up, H, {{c.dec_ffn, dec_id(l, kDUp), dn(l, "ffn_up.weight")}});
        L.ffn_sub = B.f32(c.dec_ffn, dec_id(l, kDFfnSub), dn(l, "ffn_sub_norm.weight"), 0.9f, 1.1f);
        B.tern(L.down, c.dec_ffn, {{H, dec_id(l, kDDown), dn(l, "ffn_down.weight")}});
    }
    m->final_norm = B.f32(H, kIdFinalNorm, "output_norm.weight", 0.9f, 1.1f);
    const int NA = c.action_chunk * c.action_dim;
    const float aa = 1.0f / sqrtf((float)H);
    m->act_w = B.f32((int64_t)NA * H, kIdActW, "action_head.weight", -aa, aa);
    m->act_b = B.f32(NA, kIdActB, "action_head.bias", -0.02f, 0.02f);
    m->rope = A.arr<float2>((size_t)m->seq * (size_t)(c.head_dim / 2));
    return B.rc;
}

void build_acts(b2s_bitvla* m, Arena& A) {
    const b2s_bitvla_config& c = m->cfg;
    const int64_t B = m->max_batch, Mv = B * m->np, Md = B * m->seq;
    const int D = c.vit_hidden, H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim;
    m->img = A.arr<float>((size_t)(B * 3 * c.image_size * c.image_size));
    m->d_img_u8 = A.arr<uint8_t>((size_t)(B * 3 * c.image_size * c.image_size));
    m->tok = A.arr<int32_t>((size_t)(B * (c.n_text > 0 ? c.n_text : 1)));
    m->vx = A.arr<float>((size_t)(Mv * D));
    m->vqkv = A.arr<float>((size_t)(Mv * 3 * D));
    m->vattn = A.arr<float>((size_t)(Mv * D));
    m->vh = A.arr<float>((size_t)(Mv * c.vit_ffn));
    m->ch = A.arr<float>((size_t)(Mv * c.conn_hidden));
    m->dx = A.arr<float>((size_t)(Md * H));
    m->dqkv = A.arr<float>((size_t)(Md * (H + 2 * KV)));
    m->dattn = A.arr<float>((size_t)(Md * H));
    m->dp = A.arr<float>((size_t)(Md * c.dec_ffn));
    m->hidden = A.arr<float>((size_t)(Md * H));
    m->actions = A.arr<float>((size_t)(B * c.action_chunk * c.action_dim));
    int kmax = D;
    for (int k : {c.vit_ffn, c.conn_hidden, H, c.dec_ffn}) kmax = k > kmax ? k : kmax;
    m->ldq = (int)round_up((int64_t)kmax, (int64_t)16);
    const int64_t Mmax = Md > Mv ? Md : Mv;
    {
        size_t sk = 0;
        const int64_t Ms[2] = {Mv, Md};
        const int64_t outs[6] = {3 * (int64_t)D, D, c.vit_ffn, c.conn_hidden, H + 2 * (int64_t)KV, H};
        for (int64_t mm : Ms)
            for (int64_t n : outs) sk = std::max(sk, b2s::splitk_ws_bytes(mm, n, 128));
        sk = std::max(sk, b2s::splitk_ws_bytes(Md, c.dec_ffn, 64));
        m->splitk_bytes = sk;
        m->splitk_ws = A.take(sk);
    }
    m->q8 = A.arr<int8_t>((size_t)(Mmax * m->ldq));
    m->qs = A.arr<float>((size_t)Mmax);
    m->qsum = A.arr<int32_t>((size_t)Mmax);
}


// Enqueues the forward of `B` observations already in m->img / m->tok (results in m->hidden, m->actions).
int enqueue_forward(b2s_bitvla* m, int B, cudaStream_t st) {
    const b2s_bitvla_config& c = m->cfg;
    const int D = c.vit_hidden, H = c.dec_hidden, KV = c.dec_kv_heads * c.head_dim, F = c.vit_ffn;
    const int64_t Mv = (int64_t)B * m->np, Md = (int64_t)B * m->seq;
    const int ldq = m->ldq;
    auto gemm = [&](const Tern& t, int64_t M, float* y, int64_t ldy, const float* bias, const float* res, int act) {
        b2s::Epilogue e{bias, res, res ? ldy : 0, act, 128};
        return b2s::dispatch_mul_mat_q8(t.w, m->q8, ldq, m->qs, m->qsum, M, y, ldy, 2, e, st, m->splitk_ws,
                                        m->splitk_bytes);
    };
    // The bit-reproducible fp32 attention kernel unless the config asks for the tensor-core one (and the
    // shape is one it takes).
    // With `rope` (decoder layers) the fp32 kernel rotates Q and K as it stages them; the tensor-core one reads
    // them rotated in place by a separate pass over the q and k heads.
    auto attention = [&](float* q, int64_t ldq_, float* k, int64_t ldk, const float* v, int64_t ldv, int batch, int T,
                         int heads, int kv_heads, int hd, float scale, bool causal, float* o, int64_t ldo,
                         const float2* rope) {
        if (c.attention_tc &&
            b2s::attention_tc_supported(T, heads, kv_heads, hd, causal, ldq_, ldk, ldv, ldo, q, k, v, o)) {
            if (rope) {  // q heads then k heads, adjacent columns of one row
                cudaError_t e = b2s::launch_rope_apply(q, (int64_t)batch * T, heads + kv_heads, hd, ldq_, rope, T, st);
                if (e != cudaSuccess) return e;
            }
            return b2s::launch_attention_tc(q, ldq_, k, ldk, v, ldv, batch, T, heads, kv_heads, hd, scale, causal, o,
                                            ldo, st);
        }
        return b2s::launch_attention(q, ldq_, k, ldk, v, ldv, batch, T, heads, kv_heads, hd, scale, causal, o, ldo,
                                     st, rope);
    };
    // ---------------------------------------------------------------- vision tower
    TRY_CUDA(b2s::launch_patch_embed(m->img, B, 3, c.image_size, c.image_size, c.patch, m->patch_w, m->patch_b, m->pos,
                                     D, m->vx, D, st),
             "patch_embed");
    const float vit_scale = 1.0f / sqrtf((float)(D / c.vit_heads));
    // GELU of the fc1 and first connector outputs runs in the act-quant kernel that reads them for the next
    // GEMM (the epilogue's fp32 operations, applied at full occupancy instead of by the GEMM's epilogue warps)
    // whenever that kernel takes the shape; otherwise the GEMM epilogue applies it.
    const bool vit_gelu_q = b2s::rowq_eligible(m->vh, F, nullptr, nullptr, F, m->q8, ldq, true);
    const bool conn_gelu_q = b2s::rowq_eligible(m->ch, c.conn_hidden, nullptr, nullptr, c.conn_hidden, m->q8, ldq, true);
    for (int l = 0; l < c.vit_layers; ++l) {
        const VitLayer& L = m->vit[(size_t)l];
        TRY_CUDA(b2s::launch_norm(1, true, m->vx, D, L.ln1_w, L.ln1_b, c.vit_eps, Mv, D, nullptr, 0, m->q8, ldq, m->qs,
                                  m->qsum, st),
                 "vit ln1");
        TRY_B2S(gemm(L.qkv, Mv, m->vqkv, 3 * D, L.qkv_b, nullptr, 0));
        TRY_CUDA(attention(m->vqkv, 3 * D, m->vqkv + D, 3 * D, m->vqkv + 2 * D, 3 * D, B, m->np, c.vit_heads,
                           c.vit_heads, D / c.vit_heads, vit_scale, false, m->vattn, D, nullptr),
                 "vit attention");
        TRY_CUDA(b2s::launch_act_quant(m->vattn, D, nullptr, false, 0.0f, Mv, D, m->q8, ldq, m->qs, m->qsum, st),
                 "vit o act_quant");
        TRY_B2S(gemm(L.o, Mv, m->vx, D, L.o_b, m->vx, 0));
        TRY_CUDA(b2s::launch_norm(1, true, m->vx, D, L.ln2_w, L.ln2_b, c.vit_eps, Mv, D, nullptr, 0, m->q8, ldq, m->qs,
                                  m->qsum, st),
                 "vit ln2");
        TRY_B2S(gemm(L.fc1, Mv, m->vh, F, L.fc1_b, nullptr, vit_gelu_q ? 0 : 1));
        TRY_CUDA(vit_gelu_q ? b2s::launch_rowq(3, true, m->vh, F, nullptr, nullptr, 0.0f, Mv, F, nullptr, 0, m->q8, ldq,
                                               m->qs, m->qsum, st)
                            : b2s::launch_act_quant(m->vh, F, nullptr, false, 0.0f, Mv, F, m->q8, ldq, m->qs, m->qsum,
                                                    st),
                 "vit fc2 act_quant");
        TRY_B2S(gemm(L.fc2, Mv, m->vx, D, L.fc2_b, m->vx, 0));
    }
    // ---------------------------------------------------------------- connector
    TRY_CUDA(b2s::launch_norm(1, true, m->vx, D, m->post_w, m->post_b, c.vit_eps, Mv, D, nullptr, 0, m->q8, ldq, m->qs,
                              m->qsum, st),
             "post layernorm");
    TRY_B2S(gemm(m->conn1, Mv, m->ch, c.conn_hidden, m->conn1_b, nullptr, conn_gelu_q ? 0 : 1));
    TRY_CUDA(conn_gelu_q ? b2s::launch_rowq(3, true, m->ch, c.conn_hidden, nullptr, nullptr, 0.0f, Mv, c.conn_hidden,
                                            nullptr, 0, m->q8, ldq, m->qs, m->qsum, st)
                         : b2s::launch_act_quant(m->ch, c.conn_hidden, nullptr, false, 0.0f, Mv, c.conn_hidden, m->q8,
                                                 ldq, m->qs, m->qsum, st),
             "connector act_quant");
    if (B == 1) {
        TRY_B2S(gemm(m->conn2, Mv, m->dx, H, m->conn2_b, nullptr, 0));
    } else {  // image rows of observation b go to decoder rows [b * seq, b * seq + np)
        TRY_B2S(gemm(m->conn2, Mv, m->dattn, H, m->conn2_b, nullptr, 0));
        TRY_CUDA(cudaMemcpy2DAsync(m->dx, (size_t)m->seq * H * sizeof(float), m->dattn,
                                   (size_t)m->np * H * sizeof(float), (size_t)m->np * H * sizeof(float), (size_t)B,
                                   cudaMemcpyDeviceToDevice, st),
                 "image rows");
    }
    if (c.n_text > 0) {
        embed_text_kernel<<<grid_of((int64_t)B * c.n_text * H), 256, 0, st>>>(m->tok, B, c.n_text, m->np, m->seq, H,
                                                                              m->seed, m->dx);
        TRY_CUDA(cudaGetLastError(), "embed text");
    }
    // ---------------------------------------------------------------- decoder
    const int ldqkv = H + 2 * KV;
    const float dec_scale = 1.0f / sqrtf((float)c.head_dim);
    for (int l = 0; l < c.dec_layers; ++l) {
        const DecLayer& L = m->dec[(size_t)l];
        TRY_CUDA(b2s::launch_act_quant(m->dx, H, L.attn_norm, true, c.dec_eps, Md, H, m->q8, ldq, m->qs, m->qsum, st),
                 "attn_norm");
        TRY_B2S(gemm(L.qkv, Md, m->dqkv, ldqkv, nullptr, nullptr, 0));
        TRY_CUDA(attention(m->dqkv, ldqkv, m->dqkv + H, ldqkv, m->dqkv + H + KV, ldqkv, B, m->seq, c.dec_heads,
                           c.dec_kv_heads, c.head_dim, dec_scale, true, m->dattn, H, m->rope),
                 "decoder attention");
        TRY_CUDA(b2s::launch_act_quant(m->dattn, H, L.attn_sub, true, c.dec_eps, Md, H, m->q8, ldq, m->qs, m->qsum, st),
                 "attn_sub_norm");
        TRY_B2S(gemm(L.o, Md, m->dx, H, nullptr, m->dx, 0));
        TRY_CUDA(b2s::launch_act_quant(m->dx, H, L.ffn_norm, true, c.dec_eps, Md, H, m->q8, ldq, m->qs, m->qsum, st),
                 "ffn_norm");
        TRY_B2S(b2s::dispatch_gate_up(L.gate.w, L.up.w, m->q8, ldq, m->qs, m->qsum, Md, m->dp, c.dec_ffn, st,
                                      m->splitk_ws, m->splitk_bytes));
        TRY_CUDA(b2s::launch_act_quant(m->dp, c.dec_ffn, L.ffn_sub, true, c.dec_eps, Md, c.dec_ffn, m->q8, ldq, m->qs,
                                       m->qsum, st),
                 "ffn_sub_norm");
        TRY_B2S(gemm(L.down, Md, m->dx, H, nullptr, m->dx, 0));
    }
    TRY_CUDA(b2s::launch_norm(0, false, m->dx, H, m->final_norm, nullptr, c.dec_eps, Md, H, m->hidden, H, nullptr, 0,
                              nullptr, nullptr, st),
             "final norm");
    const int NA = c.action_chunk * c.action_dim;
    action_head_kernel<<<(unsigned)ceil_div((int64_t)B * NA, (int64_t)8), 256, 0, st>>>(m->hidden, B, m->seq, H,
                                                                                       m->act_w, m->act_b, NA,
                                                                                       m->actions);
    return cuda_err(cudaGetLastError(), "action head");
}

int get_graph(b2s_bitvla* m, int B, Graph** out) {
    auto it = m->graphs.find(B);
    if (it != m->graphs.end()) {
        *out = &it->second;
        return B2S_OK;
    }
    cudaStream_t cs = nullptr;
    TRY_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "graph stream");
    // One eager pass first: every kernel module is loaded and every launch attribute is set before the
    // capture (it overwrites only this model's activation buffers).
    int rc = enqueue_forward(m, B, cs);
    if (!rc) rc = cuda_err(cudaStreamSynchronize(cs), "warm-up forward");
    cudaGraph_t graph = nullptr;
    if (!rc) {
        cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess) {
            rc = enqueue_forward(m, B, cs);
            cudaError_t e2 = cudaStreamEndCapture(cs, &graph);
            if (!rc && e2 != cudaSuccess) rc = cuda_err(e2, "graph capture");
        } else {
            rc = cuda_err(e, "begin capture");
        }
    }
    Graph g;
    if (!rc) rc = cuda_err(cudaGraphInstantiate(&g.exec, graph, 0), "graph instantiate");
    if (graph) cudaGraphDestroy(graph);
    cudaStreamDestroy(cs);
    if (rc) return rc;
    *out = &(m->graphs[B] = g);
    return B2S_OK;
}

}  // namespace

extern "C" {

void b2s_bitvla_default_config(b2s_bitvla_config* c) {
    if (!c) return;
    c->image_size = 224;
    c->patch = 14;
    c->vit_layers = 27;
    c->vit_hidden = 1152;
    c->vit_ffn = 4304;
    c->vit_heads = 16;
    c->vit_eps = 1e-6f;
    c->conn_hidden = 2560;
    c->dec_layers = 30;
    c->dec_hidden = 2560;
    c->dec_ffn = 6912;
    c->dec_heads = 20;
    c->dec_kv_heads = 5;
    c->head_dim = 128;
    c->rope_theta = 500000.0f;
    c->dec_eps = 1e-5f;
    c->vocab = 128256;
    c->n_text = 32;
    c->action_chunk = 8;
    c->action_dim = 7;
    c->attention_tc = 0;
}

int b2s_bitvla_seq_len(const b2s_bitvla_config* c) {
    if (!c || c->patch <= 0) return 0;
    const int g = c->image_size / c->patch;
    return g * g + c->n_text;
}

double b2s_bitvla_ternary_ops(const b2s_bitvla_config* c) {
    if (!c || c->patch <= 0) return 0.0;
    const double np = (double)(c->image_size / c->patch) * (c->image_size / c->patch);
    const double seq = np + c->n_text;
    const double D = c->vit_hidden, F = c->vit_ffn, H = c->dec_hidden, KV = (double)c->dec_kv_heads * c->head_dim;
    const double vit = 4.0 * D * D + 2.0 * D * F;
    const double conn = D * c->conn_hidden + (double)c->conn_hidden * H;
    const double dec = 2.0 * H * H + 2.0 * H * KV + 3.0 * H * c->dec_ffn;
    return 2.0 * (np * (c->vit_layers * vit + conn) + seq * c->dec_layers * dec);
}

uint32_t b2s_bitvla_param_bits(uint32_t seed, uint32_t tensor, uint32_t idx) { return param_bits(seed, tensor, idx); }

}  // extern "C"

namespace {

// Shared by both constructors: lays out and allocates the arenas, fills the weights from `src`, zeroes
// the activations and builds the RoPE table.
int create_model(const b2s_bitvla_config* cfg, uint32_t seed, int max_batch, WeightSource* src, b2s_bitvla** out) {
    *out = nullptr;
    int rc = b2s_device_check();
    if (rc) return rc;
    if ((rc = check_cfg(*cfg))) return rc;
    b2s_bitvla* m = new (std::nothrow) b2s_bitvla();
    if (!m) return errf(B2S_ERR_INVALID_ARG, "out of host memory");
    m->cfg = *cfg;
    m->seed = seed;
    m->max_batch = max_batch;
    cudaGetDevice(&m->device);
    m->np = (cfg->image_size / cfg->patch) * (cfg->image_size / cfg->patch);
    m->seq = m->np + cfg->n_text;
    std::vector<float> hs;
    std::vector<std::pair<float*, size_t>> fills;
    Arena wa;
    build_weights(m, wa, nullptr, nullptr, &hs, &fills);
    Arena aa;
    build_acts(m, aa);
    m->wbytes = wa.off;
    m->abytes = aa.off;
    cudaError_t e = cudaMalloc(&m->wmem, m->wbytes);
    if (e == cudaSuccess) e = cudaMalloc(&m->amem, m->abytes);
    const size_t img_bytes = (size_t)max_batch * 3 * cfg->image_size * cfg->image_size;
    const size_t tok_bytes = sizeof(int32_t) * (size_t)max_batch * (cfg->n_text > 0 ? cfg->n_text : 1);
    const size_t act_bytes = sizeof(float) * (size_t)max_batch * cfg->action_chunk * cfg->action_dim;
    if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&m->h_img), img_bytes);
    if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&m->h_tok), tok_bytes);
    if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&m->h_act), act_bytes);
    cudaStream_t st = nullptr;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        b2s_bitvla_free(m);
        return cuda_err(e, "bitvla_create allocation");
    }
    wa = Arena{static_cast<uint8_t*>(m->wmem), 0};
    rc = build_weights(m, wa, src, st, &hs, &fills);
    aa = Arena{static_cast<uint8_t*>(m->amem), 0};
    build_acts(m, aa);
    // Upload the per-tile scales (each stacked weight appended ceil(N/128) entries starting at f.second).
    for (size_t i = 0; i < fills.size() && !rc; ++i) {
        const size_t first = fills[i].second;
        const size_t last = (i + 1 < fills.size()) ? fills[i + 1].second : hs.size();
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(fills[i].first, hs.data() + first, (last - first) * sizeof(float),
                                cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(m->amem, 0, m->abytes, st);
    if (e == cudaSuccess) e = b2s::launch_rope_table(cfg->rope_theta, cfg->head_dim, m->seq, m->rope, st);
    cudaError_t es = cudaStreamSynchronize(st);  // also before any error return: staged copies must finish
    if (e == cudaSuccess) e = es;
    if (e == cudaSuccess) e = cudaGetLastError();
    cudaStreamDestroy(st);
    if (rc || e != cudaSuccess) {
        b2s_bitvla_free(m);
        return rc ? rc : cuda_err(e, "bitvla_create weight upload");
    }
    *out = m;
    return B2S_OK;
}

}  // namespace

extern "C" {

int b2s_bitvla_create(const b2s_bitvla_config* cfg, uint32_t seed, int max_batch, b2s_bitvla** out) {
    if (!cfg || !out || max_batch <= 0) return errf(B2S_ERR_INVALID_ARG, "bitvla_create: bad arguments");
    GenSource gen(seed);
    return create_model(cfg, seed, max_batch, &gen, out);
}

int b2s_bitvla_create_from_gguf(const char* path, int max_batch, b2s_bitvla** out) {
    if (!path || !out || max_batch <= 0) return errf(B2S_ERR_INVALID_ARG, "bitvla_create_from_gguf: bad arguments");
    *out = nullptr;
    b2s::GgufFile f;
    std::string err;
    if (!f.open(path, &err)) return errf(B2S_ERR_INVALID_ARG, "%s", err.c_str());
    std::string arch;
    if (!f.str("general.architecture", &arch) || arch != "bitvla")
        return errf(B2S_ERR_INVALID_ARG, "GGUF: general.architecture is '%s', expected 'bitvla'", arch.c_str());
    b2s_bitvla_config c;
    b2s_bitvla_default_config(&c);
    struct U { const char* key; int* dst; } us[] = {
        {"bitvla.image_size", &c.image_size}, {"bitvla.patch_size", &c.patch},
        {"bitvla.vision.block_count", &c.vit_layers}, {"bitvla.vision.embedding_length", &c.vit_hidden},
        {"bitvla.vision.feed_forward_length", &c.vit_ffn}, {"bitvla.vision.attention.head_count", &c.vit_heads},
        {"bitvla.connector.embedding_length", &c.conn_hidden}, {"bitvla.block_count", &c.dec_layers},
        {"bitvla.embedding_length", &c.dec_hidden}, {"bitvla.feed_forward_length", &c.dec_ffn},
        {"bitvla.attention.head_count", &c.dec_heads}, {"bitvla.attention.head_count_kv", &c.dec_kv_heads},
        {"bitvla.attention.key_length", &c.head_dim}, {"bitvla.vocab_size", &c.vocab},
        {"bitvla.text_tokens", &c.n_text}, {"bitvla.action.chunk_size", &c.action_chunk},
        {"bitvla.action.dim", &c.action_dim}};
    for (auto& u : us) {
        uint32_t v;
        if (!f.u32(u.key, &v)) return errf(B2S_ERR_INVALID_ARG, "GGUF: missing u32 key '%s'", u.key);
        *u.dst = (int)v;
    }
    struct F { const char* key; float* dst; } fs[] = {
        {"bitvla.vision.attention.layer_norm_epsilon", &c.vit_eps},
        {"bitvla.attention.layer_norm_rms_epsilon", &c.dec_eps}, {"bitvla.rope.freq_base", &c.rope_theta}};
    for (auto& x : fs)
        if (!f.f32(x.key, x.dst)) return errf(B2S_ERR_INVALID_ARG, "GGUF: missing f32 key '%s'", x.key);
    uint32_t seed = 0;
    if (!f.u32("bitvla.token_embd.seed", &seed)) return errf(B2S_ERR_INVALID_ARG, "GGUF: missing bitvla.token_embd.seed");
    int rc = b2s_device_check();
    if (rc) return rc;
    if ((rc = check_cfg(c))) return rc;
    // staging for the largest ternary tensor (flattened bytes in, row-padded bytes out)
    const int64_t Kmax = std::max({(int64_t)c.vit_hidden, (int64_t)c.vit_ffn, (int64_t)c.conn_hidden,
                                   (int64_t)c.dec_hidden, (int64_t)c.dec_ffn});
    const int64_t Nmax = std::max({(int64_t)c.vit_ffn, (int64_t)c.conn_hidden, (int64_t)c.dec_hidden,
                                   (int64_t)c.dec_ffn, (int64_t)c.vit_hidden});
    GgufSource src;
    src.f = &f;
    src.stage_bytes = (size_t)(Nmax * round_up(Kmax, (int64_t)128) / 4 + 64);
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&src.stage_in), src.stage_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&src.stage_out), src.stage_bytes);
    if (e != cudaSuccess) {
        cudaFree(src.stage_in);
        return cuda_err(e, "GGUF staging buffers");
    }
    rc = create_model(&c, seed, max_batch, &src, out);
    cudaFree(src.stage_in);
    cudaFree(src.stage_out);
    return rc;
}

void b2s_bitvla_free(b2s_bitvla* m) {
    if (!m) return;
    for (auto& kv : m->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    cudaFree(m->wmem);
    cudaFree(m->amem);
    cudaFreeHost(m->h_img);
    cudaFreeHost(m->h_tok);
    cudaFreeHost(m->h_act);
    delete m;
}

int b2s_bitvla_get_config(const b2s_bitvla* m, b2s_bitvla_config* cfg) {
    if (!m || !cfg) return errf(B2S_ERR_INVALID_ARG, "bitvla_get_config: bad arguments");
    *cfg = m->cfg;
    return B2S_OK;
}

size_t b2s_bitvla_ternary_bytes(const b2s_bitvla* m) { return m ? m->ternary_bytes : 0; }
size_t b2s_bitvla_weight_bytes(const b2s_bitvla* m) { return m ? m->wbytes : 0; }
size_t b2s_bitvla_activation_bytes(const b2s_bitvla* m) { return m ? m->abytes : 0; }

int b2s_bitvla_forward(b2s_bitvla* m, int batch, const float* images, const int32_t* tokens, float* hidden,
                       float* actions, void* stream) {
    if (!m || batch <= 0 || batch > m->max_batch || !images || (!tokens && m->cfg.n_text > 0))
        return errf(B2S_ERR_INVALID_ARG, "bitvla_forward: bad arguments (batch %d, max %d)", batch, m ? m->max_batch : 0);
    std::lock_guard<std::mutex> lock(m->mu);
    const b2s_bitvla_config& c = m->cfg;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Graph* g = nullptr;
    int rc = get_graph(m, batch, &g);
    if (rc) return rc;
    const size_t img = sizeof(float) * (size_t)batch * 3 * c.image_size * c.image_size;
    TRY_CUDA(cudaMemcpyAsync(m->img, images, img, cudaMemcpyDeviceToDevice, st), "images");
    if (c.n_text > 0)
        TRY_CUDA(cudaMemcpyAsync(m->tok, tokens, sizeof(int32_t) * (size_t)batch * c.n_text, cudaMemcpyDeviceToDevice, st),
                 "tokens");
    TRY_CUDA(cudaGraphLaunch(g->exec, st), "graph launch");
    if (hidden)
        TRY_CUDA(cudaMemcpyAsync(hidden, m->hidden, sizeof(float) * (size_t)batch * m->seq * c.dec_hidden,
                                 cudaMemcpyDeviceToDevice, st),
                 "hidden");
    if (actions)
        TRY_CUDA(cudaMemcpyAsync(actions, m->actions, sizeof(float) * (size_t)batch * c.action_chunk * c.action_dim,
                                 cudaMemcpyDeviceToDevice, st),
                 "actions");
    return B2S_OK;
}

int b2s_bitvla_predict(b2s_bitvla* m, int batch, const uint8_t* images_hwc, const int32_t* tokens, float* actions,
                       void* stream) {
    if (!m || batch <= 0 || batch > m->max_batch || !images_hwc || !actions || (!tokens && m->cfg.n_text > 0))
        return errf(B2S_ERR_INVALID_ARG, "bitvla_predict: bad arguments");
    std::lock_guard<std::mutex> lock(m->mu);
    const b2s_bitvla_config& c = m->cfg;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Graph* g = nullptr;
    int rc = get_graph(m, batch, &g);
    if (rc) return rc;
    const size_t img = (size_t)batch * 3 * c.image_size * c.image_size;
    const size_t tok = sizeof(int32_t) * (size_t)batch * c.n_text;
    const size_t act = sizeof(float) * (size_t)batch * c.action_chunk * c.action_dim;
    memcpy(m->h_img, images_hwc, img);
    if (tok) memcpy(m->h_tok, tokens, tok);
    TRY_CUDA(cudaMemcpyAsync(m->d_img_u8, m->h_img, img, cudaMemcpyHostToDevice, st), "images H2D");
    if (tok) TRY_CUDA(cudaMemcpyAsync(m->tok, m->h_tok, tok, cudaMemcpyHostToDevice, st), "tokens H2D");
    image_u8_kernel<<<grid_of((int64_t)img), 256, 0, st>>>(m->d_img_u8, batch, c.image_size, m->img);
    TRY_CUDA(cudaGetLastError(), "image convert");
    TRY_CUDA(cudaGraphLaunch(g->exec, st), "graph launch");
    TRY_CUDA(cudaMemcpyAsync(m->h_act, m->actions, act, cudaMemcpyDeviceToHost, st), "actions D2H");
    TRY_CUDA(cudaStreamSynchronize(st), "predict sync");
    memcpy(actions, m->h_act, act);
    return B2S_OK;
}

}  // extern "C"
