// b2s_api.cu -- the extern "C" boundary of libb2s.so (declared in include/b2s.h).
//
// Validates ggml-style tensor descriptors, owns no device memory (callers pass workspaces), builds the
// TMA descriptors for the tensor-core path and dispatches between the decode GEMV and the tcgen05 GEMM.
// Error convention follows the reference's bool/status-plus-message style
// (src/models/gguf_loader.cpp:246-254, robot_server/session.cpp:132-135): negative status + message.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "b2s.h"
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(B2S_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ---------------------------------------------------------------- device check (cached per device)
int check_device() {
    static std::atomic<int> cache[128];  // 0 unknown, 1 ok, 2 bad
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 128) return fail(B2S_ERR_DEVICE, "device index %d out of range", dev);
    if (cache[dev] == 0) {
        int major = 0, minor = 0;
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        cache[dev] = (major == 10 && minor == 0) ? 1 : 2;
        if (cache[dev] == 2) return fail(B2S_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                                         major, minor);
    }
    return cache[dev] == 1 ? B2S_OK : fail(B2S_ERR_DEVICE, "device %d is not sm_100", dev);
}

// ---------------------------------------------------------------- TMA descriptor encoding
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2D u8 tensor map: inner dim `cols` bytes, `rows` rows of stride `ld` bytes, box box_c x box_r, shared-memory
// swizzle `swz` (the activation tiles use 128-byte swizzle for the MMA descriptors; the 32-byte packed weight
// rows use 32-byte swizzle, which swaps the two 16-byte halves of every other group of four rows so that the
// converter warps' row reads are free of bank conflicts).
int make_tmap_u8(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_c,
                 uint32_t box_r, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(B2S_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return fail(B2S_ERR_UNSUPPORTED, "TMA base not 16-byte aligned");
    if (ld % 16 != 0) return fail(B2S_ERR_UNSUPPORTED, "TMA row stride %llu not a multiple of 16 bytes",
                                  (unsigned long long)ld);
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {box_c, box_r};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(B2S_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return B2S_OK;
}

// 2D fp32 tensor map without swizzle: `cols` floats per row, `rows` rows of stride `ld` floats, box
// box_c x box_r. Returns false (no error recorded) when the base or stride is not TMA-compatible.
bool make_tmap_f32(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_c,
                   uint32_t box_r) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (ld * 4) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 4};
    cuuint32_t box[2] = {box_c, box_r};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- descriptor validation
int weight_view(const b2s_tensor* W, b2s::I2sWeight* out, const char* name) {
    if (!W) return fail(B2S_ERR_INVALID_ARG, "%s is NULL", name);
    if (!W->data) return fail(B2S_ERR_INVALID_ARG, "%s->data is NULL", name);
    const int64_t K = W->ne[0], N = W->ne[1];
    if (K <= 0 || N <= 0 || W->ne[2] != 1 || W->ne[3] != 1)
        return fail(B2S_ERR_INVALID_ARG, "%s must be 2-D with positive ne0/ne1 (got %lld x %lld x %lld x %lld)", name,
                    (long long)W->ne[0], (long long)W->ne[1], (long long)W->ne[2], (long long)W->ne[3]);
    if ((reinterpret_cast<uintptr_t>(W->data) & 15) != 0)
        return fail(B2S_ERR_UNSUPPORTED, "%s->data must be 16-byte aligned", name);
    if (K % 16 != 0) return fail(B2S_ERR_UNSUPPORTED, "%s: ne0 (K=%lld) must be a multiple of 16", name, (long long)K);
    const int64_t Kp = b2s::round_up(K, b2s::kQK);
    if (W->type == B2S_TYPE_I2_S) {
        if (K % b2s::kQK != 0)
            return fail(B2S_ERR_UNSUPPORTED,
                        "%s: i2_s with ne0 %% 128 != 0 (K=%lld) must be repacked with b2s_i2s_repack_rows first", name,
                        (long long)K);
    } else if (W->type != B2S_TYPE_I2_S_R) {
        return fail(B2S_ERR_UNSUPPORTED, "%s: type %d is not i2_s", name, (int)W->type);
    }
    out->codes = static_cast<const uint8_t*>(W->data);
    out->scale = reinterpret_cast<const float*>(static_cast<const uint8_t*>(W->data) + N * Kp / 4);
    out->N = N;
    out->K = K;
    out->Kp = Kp;
    return B2S_OK;
}

// A batched i2_s weight, ne = [K, N, B, 1]: B matrices of N rows stored back to back (matrix b at byte
// b * N * Kp / 4, nb[2] = N * Kp / 4) with the tensor's one fp32 scale after all B * N rows -- the flattened
// i2_s layout over B * N rows. Returns the view of matrix 0 and the byte stride between matrices.
int weight_view_batched(const b2s_tensor* W, b2s::I2sWeight* out, int64_t* count, int64_t* stride, const char* name) {
    if (!W) return fail(B2S_ERR_INVALID_ARG, "%s is NULL", name);
    if (W->ne[2] <= 0 || W->ne[3] != 1)
        return fail(B2S_ERR_INVALID_ARG, "%s: batched weight needs ne[2] >= 1 and ne[3] == 1", name);
    b2s_tensor flat = *W;  // the B * N rows as one 2-D tensor validates every byte-level rule
    flat.ne[1] = W->ne[1] * W->ne[2];
    flat.ne[2] = 1;
    int rc = weight_view(&flat, out, name);
    if (rc) return rc;
    out->N = W->ne[1];
    *count = W->ne[2];
    *stride = out->N * out->Kp / 4;
    if (W->ne[2] > 1 && W->nb[2] != (size_t)*stride)
        return fail(B2S_ERR_UNSUPPORTED, "%s: nb[2] (%zu) must be N * K / 4 = %lld (matrices back to back)", name,
                    W->nb[2], (long long)*stride);
    return B2S_OK;
}

// Rows of a ggml f32 tensor as a 2-D [rows x ne0] view with row stride ld (elements).
int f32_rows(const b2s_tensor* T, const char* name, int64_t* rows, int64_t* cols, int64_t* ld) {
    if (!T) return fail(B2S_ERR_INVALID_ARG, "%s is NULL", name);
    if (!T->data) return fail(B2S_ERR_INVALID_ARG, "%s->data is NULL", name);
    if (T->type != B2S_TYPE_F32) return fail(B2S_ERR_UNSUPPORTED, "%s must be f32 (type %d)", name, (int)T->type);
    if (T->nb[0] != sizeof(float)) return fail(B2S_ERR_UNSUPPORTED, "%s rows must be contiguous (nb0=4)", name);
    if (T->ne[0] <= 0 || T->ne[1] <= 0 || T->ne[2] <= 0 || T->ne[3] <= 0)
        return fail(B2S_ERR_INVALID_ARG, "%s has a non-positive dimension", name);
    if (T->nb[1] % sizeof(float) != 0 || T->nb[1] < T->ne[0] * sizeof(float))
        return fail(B2S_ERR_INVALID_ARG, "%s: nb1 (%zu) inconsistent with ne0 (%lld)", name, T->nb[1], (long long)T->ne[0]);
    // Higher dims must collapse into rows with a uniform stride.
    if ((T->ne[2] > 1 && T->nb[2] != T->nb[1] * T->ne[1]) || (T->ne[3] > 1 && T->nb[3] != T->nb[2] * T->ne[2]))
        return fail(B2S_ERR_UNSUPPORTED, "%s: dims 2/3 must be contiguous over rows", name);
    *rows = T->ne[1] * T->ne[2] * T->ne[3];
    *cols = T->ne[0];
    *ld = (int64_t)(T->nb[1] / sizeof(float));
    return B2S_OK;
}

struct WsLayout {
    size_t q_off, s_off, sum_off, total;
    int64_t ldq;
};
size_t a256(size_t v) { return (v + 255) & ~size_t(255); }
WsLayout act_ws(int64_t M, int64_t K, size_t base = 0) {
    WsLayout l;
    l.ldq = b2s::round_up(K, 16);
    l.q_off = a256(base);
    l.s_off = a256(l.q_off + (size_t)(M * l.ldq));
    l.sum_off = a256(l.s_off + sizeof(float) * (size_t)M);
    l.total = a256(l.sum_off + sizeof(int32_t) * (size_t)M);
    return l;
}

int launched(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        (void)cudaGetLastError();  // a failed launch must not leak into the next call's error check
        return cuda_fail(e, what);
    }
    return B2S_OK;
}

// Tensor-core tiling. A CTA covers up to 320 tokens as one (<= 256) or two MMA sub-tiles; M is split into
// the fewest such spans (fewer CTA waves beat full-width 256-token MMAs on a non-persistent grid). When
// the output tiles cannot fill the GPU's SMs, the K loop is split across the CTAs of a cluster (up to 8,
// each keeping at least two 128-wide K steps).
struct TcTiling {
    int T, bn_sub, nsub, m_tiles, n_tiles, splits;
};
TcTiling pick_tiling(int64_t M, int64_t n_out, int rows_per_cta, int64_t Kp, int num_sms) {
    TcTiling t;
    t.m_tiles = (int)b2s::ceil_div(M, 320);
    const int64_t t0 = b2s::ceil_div(M, t.m_tiles);
    if (t0 <= 256) {
        t.nsub = 1;
        t.bn_sub = (int)b2s::round_up(t0 < 16 ? 16 : t0, 16);
    } else {
        t.nsub = 2;
        t.bn_sub = (int)b2s::round_up(b2s::ceil_div(t0, 2), 16);
    }
    t.T = t.nsub * t.bn_sub;
    t.n_tiles = (int)b2s::ceil_div(n_out, rows_per_cta);
    const int64_t tiles = (int64_t)t.n_tiles * t.m_tiles;
    int s = 1;
    if (tiles < num_sms) s = (int)(num_sms / tiles);
    const int64_t nkt = Kp / b2s::kQK;
    if (s > nkt / 2) s = (int)(nkt / 2);
    if (s > 8) s = 8;
    if (s < 1) s = 1;
    // A cluster must fit inside one GPC: take the largest split whose clusters all fit at once (one wave).
    while (s > 1) {
        const int act = b2s::tc_max_active_clusters(s);
        if (act <= 0 || tiles <= act) break;
        --s;
    }
    t.splits = s;
    return t;
}

int num_sms_current() {
    static std::atomic<int> cache[128];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int run_tc(const b2s::I2sWeight& w0, const b2s::I2sWeight* w1, const int8_t* q, int64_t ldq, const float* s,
           const int32_t* sums, int64_t M, float* Y, int64_t ldy, int mode, cudaStream_t st,
           const b2s::Epilogue& epi = b2s::Epilogue{}, void* splitk_ws = nullptr, size_t splitk_bytes = 0) {
    if ((reinterpret_cast<uintptr_t>(q) & 15) != 0 || ldq % 16 != 0)
        return fail(B2S_ERR_UNSUPPORTED, "tensor-core path needs 16-byte aligned q with ldq %% 16 == 0");
    if (M > (int64_t)0x7fffffff || w0.N > (int64_t)0x7fffffff) return fail(B2S_ERR_UNSUPPORTED, "size exceeds int32");
    const int rows = (mode == 1) ? 64 : 128;
    const int nsm = num_sms_current();
    TcTiling t = pick_tiling(M, w0.N, rows, w0.Kp, nsm);
    // Persistent kernel when the one-tile-per-CTA kernel would need more than one wave (its tiles of up to
    // 320 tokens exceed the SM count): choose the token tile that minimises (tiles per SM) x (tile tokens +
    // 64), the 64 standing for the per-tile fixed costs. Up to 8 more token tiles than the minimum are
    // tried, so that a shape whose fewest tiles leave a thin last wave can take smaller ones (the ViT's
    // 2048 x 1152 -> 3456 GEMM: 16 tiles of 128 tokens fill 97% of the SMs' slots, 13 of 160 only 79%).
    // Where the one-tile-per-CTA kernel would split K instead, a persistent grid of one wave wins when a
    // token tile of at least 64 gives 90-100% of the SMs exactly one tile each (no split-K exchange, two
    // K steps per handoff): the ViT's 2048 x 1152 -> 1152 (+bias, +residual) 17.4 -> 13.7 µs and
    // 2048 x 4304 -> 1152 24.2 -> 19.3 µs with 144 tiles of 128 tokens.
    const bool one_wave = (int64_t)t.n_tiles * t.m_tiles <= nsm && t.splits > 1;
    int p_grid = 0;
    if ((int64_t)t.n_tiles * t.m_tiles > nsm || one_wave) {
        const int64_t n_tiles = b2s::ceil_div(w0.N, rows), mt0 = b2s::ceil_div(M, b2s::tcp_max_tokens());
        int64_t best = -1;
        for (int64_t mt = mt0; mt <= mt0 + 8; ++mt) {
            const int64_t T = b2s::round_up(b2s::ceil_div(M, mt), 16);
            if (T > b2s::tcp_max_tokens() || b2s::ceil_div(M, T) != mt) continue;
            const int64_t tiles = n_tiles * mt;
            if (one_wave ? (tiles > nsm || tiles * 10 < (int64_t)nsm * 9 || T < 64) : tiles < nsm) continue;
            const int64_t cost = b2s::ceil_div(tiles, nsm) * (T + 64);
            if (best < 0 || cost < best) {
                best = cost;
                t.T = t.bn_sub = (int)T;
                t.nsub = 1;
                t.m_tiles = (int)mt;
                t.n_tiles = (int)n_tiles;
                t.splits = 1;
                p_grid = (int)(tiles < nsm ? tiles : nsm);
            }
        }
    }
    b2s::TcGemmArgs a;
    memset(&a, 0, sizeof(a));
    int rc;
    if ((rc = make_tmap_u8(&a.tmap_q, q, (uint64_t)w0.K, (uint64_t)M, (uint64_t)ldq, 128, (uint32_t)t.bn_sub,
                           CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tmap_u8(&a.tmap_w0, w0.codes, (uint64_t)(w0.Kp / 4), (uint64_t)w0.N, (uint64_t)(w0.Kp / 4), 32,
                           (uint32_t)rows, CU_TENSOR_MAP_SWIZZLE_32B)))
        return rc;
    if (mode == 1) {
        if ((rc = make_tmap_u8(&a.tmap_w1, w1->codes, (uint64_t)(w1->Kp / 4), (uint64_t)w1->N, (uint64_t)(w1->Kp / 4),
                               32, (uint32_t)rows, CU_TENSOR_MAP_SWIZZLE_32B)))
            return rc;
        a.y_tma = make_tmap_f32(&a.tmap_y, Y, (uint64_t)w0.N, (uint64_t)M, (uint64_t)ldy, 64, 16) ? 1 : 0;
    } else {
        a.tmap_w1 = a.tmap_w0;
    }
    if (!a.y_tma) a.tmap_y = a.tmap_w0;  // unused placeholder
    a.w0_scale = w0.scale;
    a.w1_scale = (mode == 1) ? w1->scale : w0.scale;
    a.s = s;
    a.sums = sums;
    a.y = Y;
    a.ldy = ldy;
    a.M = (int)M;
    a.N = (int)w0.N;
    a.K = (int)w0.K;
    a.Kp = (int)w0.Kp;
    a.T = t.T;
    a.bn_sub = t.bn_sub;
    a.nsub = t.nsub;
    a.n_tiles = t.n_tiles;
    a.m_tiles = t.m_tiles;
    a.splits = t.splits;
    a.mode = mode;
    a.epi = epi;
    a.part = nullptr;
    if (t.splits > 1 && splitk_ws && ((reinterpret_cast<uintptr_t>(splitk_ws) & 255) == 0) &&
        splitk_bytes >= (size_t)t.n_tiles * t.m_tiles * t.splits * t.T * 128 * sizeof(int32_t))
        a.part = static_cast<int32_t*>(splitk_ws);
    if (p_grid > 0) return launched(b2s::launch_gemm_i2s_tcp(a, p_grid, st), "gemm_i2s_tcp launch");
    return launched(b2s::launch_gemm_i2s_tc(a, st), "gemm_i2s_tc launch");
}

// path: 0 auto, 1 GEMV, 2 tensor cores
int mul_mat_q8_impl(const b2s::I2sWeight& w, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums,
                    int64_t M, float* Y, int64_t ldy, int path, cudaStream_t st,
                    const b2s::Epilogue& epi = b2s::Epilogue{}, void* splitk_ws = nullptr,
                    size_t splitk_bytes = 0) {
    if (M <= 0) return B2S_OK;
    if (path == 0) path = (M <= 16) ? 1 : 2;
    if (path == 1) {
        b2s::Q8Act a{q, s, sums, M, w.K, ldq};
        return launched(b2s::launch_gemv_i2s(w, a, Y, ldy, epi, st), "gemv_i2s launch");
    }
    return run_tc(w, nullptr, q, ldq, s, sums, M, Y, ldy, 0, st, epi, splitk_ws, splitk_bytes);
}

// B independent problems: decode sizes (M <= 16) as one batched GEMV launch, larger M one tensor-core GEMM
// per matrix.
int mul_mat_q8_batched_impl(const b2s::I2sWeight& w, int64_t B, int64_t w_stride, const int8_t* q, int64_t ldq,
                            int64_t q_bstride, const float* s, const int32_t* sums, int64_t a_bstride, int64_t M, float* Y,
                            int64_t ldy, int64_t y_bstride, cudaStream_t st, void* splitk_ws = nullptr,
                            size_t splitk_bytes = 0) {
    if (M <= 0 || B <= 0) return B2S_OK;
    if (M <= 16 && B <= 65535) {
        b2s::GemvBatch bt;
        bt.count = (int)B;
        bt.w_stride = w_stride;
        bt.q_stride = q_bstride;
        bt.a_stride = a_bstride;
        bt.y_stride = y_bstride;
        b2s::Q8Act a{q, s, sums, M, w.K, ldq};
        return launched(b2s::launch_gemv_i2s(w, a, Y, ldy, b2s::Epilogue{}, st, bt), "gemv_i2s batched launch");
    }
    for (int64_t b = 0; b < B; ++b) {
        b2s::I2sWeight wb = w;
        wb.codes = w.codes + b * w_stride;
        const int rc = mul_mat_q8_impl(wb, q + b * q_bstride, ldq, s + b * a_bstride, sums + b * a_bstride, M,
                                       Y + b * y_bstride, ldy, 0, st, b2s::Epilogue{}, splitk_ws, splitk_bytes);
        if (rc) return rc;
    }
    return B2S_OK;
}

}  // namespace

namespace b2s {

int dispatch_mul_mat_q8(const I2sWeight& w, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums,
                        int64_t M, float* y, int64_t ldy, int path, const Epilogue& epi, cudaStream_t st,
                        void* splitk_ws, size_t splitk_bytes) {
    if (epi.scale_rows < 0 || (epi.scale_rows % 128 != 0 && path != 1))
        return fail(B2S_ERR_UNSUPPORTED, "stacked weight scales need scale_rows %% 128 == 0");
    return mul_mat_q8_impl(w, q, ldq, s, sums, M, y, ldy, path, st, epi, splitk_ws, splitk_bytes);
}

int dispatch_gate_up(const I2sWeight& wg, const I2sWeight& wu, const int8_t* q, int64_t ldq, const float* s,
                     const int32_t* sums, int64_t M, float* p, int64_t ldp, cudaStream_t st, void* splitk_ws,
                     size_t splitk_bytes) {
    if (M <= 0) return B2S_OK;
    return run_tc(wg, &wu, q, ldq, s, sums, M, p, ldp, 1, st, Epilogue{}, splitk_ws, splitk_bytes);
}

size_t splitk_ws_bytes(int64_t M, int64_t n_out, int rows_per_cta) {
    // A K split is chosen only while tiles x splits <= the SM count; tiles hold at most 320 tokens.
    const int64_t nsm = num_sms_current();
    const int64_t m_tiles = ceil_div(M, 320), n_tiles = ceil_div(n_out, rows_per_cta);
    if (M <= 0 || n_tiles * m_tiles >= nsm) return 0;
    const int64_t T = round_up(ceil_div(M, m_tiles), 32);
    return (size_t)(nsm * (T < 320 ? T : 320) * 128) * sizeof(int32_t);
}

int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

int mul_mat_scratch_bytes(const void* Wv, const void* Xv, size_t* need) {
    const b2s_tensor* W = static_cast<const b2s_tensor*>(Wv);
    const b2s_tensor* X = static_cast<const b2s_tensor*>(Xv);
    b2s::I2sWeight w{};
    int64_t M = 0, Kx = 0, ldx = 0;
    int rc;
    *need = 0;
    if ((rc = weight_view(W, &w, "W"))) return rc;
    if ((rc = f32_rows(X, "X", &M, &Kx, &ldx))) return rc;
    *need = act_ws(M, w.K).total;
    return B2S_OK;
}

int mul_mat_into_scratch(const void* Wv, const void* Xv, void* Yv, void* scratch, size_t capacity, cudaStream_t st) {
    const b2s_tensor* W = static_cast<const b2s_tensor*>(Wv);
    const b2s_tensor* X = static_cast<const b2s_tensor*>(Xv);
    const b2s_tensor* Y = static_cast<const b2s_tensor*>(Yv);
    b2s::I2sWeight w{};
    int rc;
    if ((rc = weight_view(W, &w, "W"))) return rc;
    int64_t M = 0, Kx = 0, ldx = 0, My = 0, Ny = 0, ldy = 0;
    if ((rc = f32_rows(X, "X", &M, &Kx, &ldx))) return rc;
    if ((rc = f32_rows(Y, "Y", &My, &Ny, &ldy))) return rc;
    if (Kx != w.K) return fail(B2S_ERR_INVALID_ARG, "X ne0 (%lld) != W ne0 (%lld)", (long long)Kx, (long long)w.K);
    if (Ny != w.N || My != M)
        return fail(B2S_ERR_INVALID_ARG, "Y must be ne=[%lld,%lld], got [%lld,%lld]", (long long)w.N, (long long)M,
                    (long long)Ny, (long long)My);
    const WsLayout l = act_ws(M, w.K);
    if (!scratch || capacity < l.total)
        return fail(B2S_ERR_WORKSPACE, "mul_mat needs %zu scratch bytes, %zu available", l.total, capacity);
    uint8_t* ws = static_cast<uint8_t*>(scratch);
    int8_t* q = reinterpret_cast<int8_t*>(ws + l.q_off);
    float* s = reinterpret_cast<float*>(ws + l.s_off);
    int32_t* sums = reinterpret_cast<int32_t*>(ws + l.sum_off);
    if ((rc = launched(b2s::launch_act_quant(static_cast<const float*>(X->data), ldx, nullptr, false, 0.0f, M, w.K, q,
                                             l.ldq, s, sums, st),
                       "act_quant launch")))
        return rc;
    // The rest of the region (past the activation layout) holds split-K partials, as in b2s_mul_mat.
    const size_t sk_off = a256(l.total);
    void* sk = capacity > sk_off ? static_cast<void*>(ws + sk_off) : nullptr;
    return mul_mat_q8_impl(w, q, l.ldq, s, sums, M, static_cast<float*>(Y->data), ldy, 0, st, b2s::Epilogue{}, sk,
                           sk ? capacity - sk_off : 0);
}

}  // namespace b2s

namespace {

// MUL_MAT over ne[2] (ggml's batched matmul, one weight matrix per batch entry): W ne=[K,N,B], X ne=[K,M,B],
// Y ne=[N,M,B], X and Y rows contiguous across the batch. All B*M tokens are quantized in one launch.
int mul_mat_batched(const b2s_tensor* W, const b2s_tensor* X, const b2s_tensor* Y, void* workspace,
                    size_t workspace_bytes, cudaStream_t st) {
    b2s::I2sWeight w{};
    int64_t B = 0, wstride = 0;
    int rc;
    if ((rc = weight_view_batched(W, &w, &B, &wstride, "W"))) return rc;
    if (!X || !Y) return fail(B2S_ERR_INVALID_ARG, "X and Y must be non-NULL");
    if (X->ne[2] != B || Y->ne[2] != B || X->ne[3] != 1 || Y->ne[3] != 1)
        return fail(B2S_ERR_INVALID_ARG, "batched mul_mat: X and Y need ne[2] == W ne[2] (%lld) and ne[3] == 1",
                    (long long)B);
    int64_t rows, Kx, ldx, yrows, Ny, ldy;
    if ((rc = f32_rows(X, "X", &rows, &Kx, &ldx))) return rc;
    if ((rc = f32_rows(Y, "Y", &yrows, &Ny, &ldy))) return rc;
    if (Kx != w.K) return fail(B2S_ERR_INVALID_ARG, "X ne0 (%lld) != W ne0 (%lld)", (long long)Kx, (long long)w.K);
    const int64_t M = X->ne[1];
    if (Ny != w.N || Y->ne[1] != M) return fail(B2S_ERR_INVALID_ARG, "Y must be ne=[N, M, B]");
    const WsLayout l = act_ws(rows, w.K);
    if (!workspace || workspace_bytes < l.total)
        return fail(B2S_ERR_WORKSPACE, "mul_mat needs %zu workspace bytes, got %zu", l.total, workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(B2S_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int8_t* q = reinterpret_cast<int8_t*>(ws + l.q_off);
    float* s = reinterpret_cast<float*>(ws + l.s_off);
    int32_t* sums = reinterpret_cast<int32_t*>(ws + l.sum_off);
    if ((rc = launched(b2s::launch_act_quant(static_cast<const float*>(X->data), ldx, nullptr, false, 0.0f, rows, w.K,
                                             q, l.ldq, s, sums, st),
                       "act_quant launch")))
        return rc;
    const size_t sk_off = a256(l.total);
    void* sk = workspace_bytes > sk_off ? ws + sk_off : nullptr;
    return mul_mat_q8_batched_impl(w, B, wstride, q, l.ldq, M * l.ldq, s, sums, M, M, static_cast<float*>(Y->data),
                                   ldy, M * ldy, st, sk, sk ? workspace_bytes - sk_off : 0);
}

}  // namespace

// ==================================================================================================
extern "C" {

const char* b2s_version(void) { return "b2s 0.1 (sm_100a)"; }

const char* b2s_last_error(void) { return t_last_error.c_str(); }

int b2s_device_check(void) { return check_device(); }

int b2s_device_error(uint32_t* out_bits, int clear) {
    if (!out_bits) return fail(B2S_ERR_INVALID_ARG, "out_bits is NULL");
    int rc = check_device();
    if (rc) return rc;
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, b2s::g_device_error, sizeof(v));
    if (e != cudaSuccess) return cuda_fail(e, "read device error word");
    if (clear) {
        const unsigned int z = 0;
        e = cudaMemcpyToSymbol(b2s::g_device_error, &z, sizeof(z));
        if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
    }
    *out_bits = v;
    return B2S_OK;
}

size_t b2s_i2s_nbytes(int64_t nrow, int64_t n_per_row) {
    if (nrow <= 0 || n_per_row <= 0) return 0;
    return (size_t)(nrow * n_per_row / 4) + 32;
}

size_t b2s_i2s_r_nbytes(int64_t nrow, int64_t n_per_row) {
    if (nrow <= 0 || n_per_row <= 0) return 0;
    return (size_t)(nrow * b2s::round_up(n_per_row, b2s::kQK) / 4) + 32;
}

size_t b2s_i2s_quantize(const float* src, void* dst, int64_t nrow, int64_t n_per_row) {
    if (!src || !dst || nrow <= 0 || n_per_row <= 0) {
        fail(B2S_ERR_INVALID_ARG, "b2s_i2s_quantize: bad arguments");
        return 0;
    }
    const int64_t n = nrow * n_per_row;
    if (n % b2s::kQK != 0) {
        fail(B2S_ERR_UNSUPPORTED, "b2s_i2s_quantize: nrow*n_per_row must be a multiple of 128");
        return 0;
    }
    uint8_t* out = static_cast<uint8_t*>(dst);
    double amax = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double a = src[i] < 0 ? -(double)src[i] : (double)src[i];
        if (a > amax) amax = a;
    }
    memset(out, 0, (size_t)(n / 4) + 32);
    for (int64_t blk = 0; blk < n / b2s::kQK; ++blk) {
        for (int j = 0; j < b2s::kQK; ++j) {
            const float v = src[blk * b2s::kQK + j];
            const double av = v < 0 ? -(double)v : (double)v;
            const unsigned code = (av < 1e-6) ? 1u : ((double)v * amax > 0 ? 2u : 0u);
            out[32 * blk + (j & 31)] |= (uint8_t)(code << (6 - 2 * (j >> 5)));
        }
    }
    const float sc = (float)amax;
    memcpy(out + n / 4, &sc, sizeof(float));
    return (size_t)(n / 4) + 32;
}

int b2s_i2s_dequantize(const void* src, float* dst, int64_t nrow, int64_t n_per_row) {
    if (!src || !dst || nrow <= 0 || n_per_row <= 0) return fail(B2S_ERR_INVALID_ARG, "b2s_i2s_dequantize: bad arguments");
    const int64_t n = nrow * n_per_row;
    if (n % b2s::kQK != 0) return fail(B2S_ERR_UNSUPPORTED, "b2s_i2s_dequantize: n must be a multiple of 128");
    const uint8_t* in = static_cast<const uint8_t*>(src);
    float sc;
    memcpy(&sc, in + n / 4, sizeof(float));
    for (int64_t g = 0; g < n; ++g) {
        const int64_t blk = g / b2s::kQK;
        const int j = (int)(g % b2s::kQK);
        const int code = (in[32 * blk + (j & 31)] >> (6 - 2 * (j >> 5))) & 3;
        dst[g] = (float)(code - 1) * sc;
    }
    return B2S_OK;
}

int b2s_i2s_repack_rows(const void* src, void* dst, int64_t nrow, int64_t n_per_row, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!src || !dst || nrow <= 0 || n_per_row <= 0) return fail(B2S_ERR_INVALID_ARG, "b2s_i2s_repack_rows: bad arguments");
    if ((nrow * n_per_row) % b2s::kQK != 0) return fail(B2S_ERR_UNSUPPORTED, "i2_s needs n %% 128 == 0");
    return launched(b2s::launch_repack_rows(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), nrow,
                                            n_per_row, static_cast<cudaStream_t>(stream)),
                    "repack_rows launch");
}

static int act_quant_common(const float* x, const float* g, bool norm, float eps, int64_t M, int64_t K, int64_t ldx,
                            int8_t* q, int64_t ldq, float* s, int32_t* sums, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!x || !q || !s) return fail(B2S_ERR_INVALID_ARG, "act_quant: x, q and s must be non-NULL");
    if (M < 0 || K <= 0 || ldx < K || ldq < K) return fail(B2S_ERR_INVALID_ARG, "act_quant: bad shape/strides");
    if (K > (int64_t)0x7fffffff || M > (int64_t)0x7fffffff) return fail(B2S_ERR_UNSUPPORTED, "act_quant: size exceeds int32");
    return launched(b2s::launch_act_quant(x, ldx, g, norm, eps, M, K, q, ldq, s, sums, static_cast<cudaStream_t>(stream)),
                    "act_quant launch");
}

int b2s_act_quant(const float* x, int64_t M, int64_t K, int64_t ldx, int8_t* q, int64_t ldq, float* s, int32_t* sums,
                  void* stream) {
    return act_quant_common(x, nullptr, false, 0.0f, M, K, ldx, q, ldq, s, sums, stream);
}

int b2s_rms_norm_act_quant(const float* x, const float* g, int64_t M, int64_t K, int64_t ldx, float eps, int8_t* q,
                           int64_t ldq, float* s, int32_t* sums, void* stream) {
    return act_quant_common(x, g, true, eps, M, K, ldx, q, ldq, s, sums, stream);
}

size_t b2s_mul_mat_workspace_size(const b2s_tensor* W, const b2s_tensor* X) {
    if (!W || !X) return 0;
    const int64_t M = X->ne[1] * (X->ne[2] > 0 ? X->ne[2] : 1) * (X->ne[3] > 0 ? X->ne[3] : 1);
    return a256(act_ws(M, W->ne[0]).total) + b2s::splitk_ws_bytes(M, W->ne[1], 128);
}

int b2s_mul_mat_q8_ex(const b2s_tensor* W, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums,
                      int64_t M, float* Y, int64_t ldy, int path, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    b2s::I2sWeight w;
    if ((rc = weight_view(W, &w, "W"))) return rc;
    if (!q || !s || !sums || !Y) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8: q, s, sums and Y must be non-NULL");
    if (M < 0 || ldq < w.K || ldy < w.N) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8: bad M/ldq/ldy");
    if (path < 0 || path > 2) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8: path must be 0, 1 or 2");
    return mul_mat_q8_impl(w, q, ldq, s, sums, M, Y, ldy, path, static_cast<cudaStream_t>(stream));
}

int b2s_mul_mat_q8_batched(const b2s_tensor* W, const int8_t* q, int64_t ldq, int64_t q_bstride, const float* s,
                           const int32_t* sums, int64_t a_bstride, int64_t M, float* Y, int64_t ldy, int64_t y_bstride,
                           void* stream) {
    int rc = check_device();
    if (rc) return rc;
    b2s::I2sWeight w;
    int64_t B = 0, wstride = 0;
    if ((rc = weight_view_batched(W, &w, &B, &wstride, "W"))) return rc;
    if (!q || !s || !sums || !Y) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_batched: q, s, sums and Y must be non-NULL");
    if (M < 0 || ldq < w.K || ldy < w.N || q_bstride < M * ldq || a_bstride < M || y_bstride < M * ldy)
        return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_batched: bad M / leading dimensions / batch strides");
    return mul_mat_q8_batched_impl(w, B, wstride, q, ldq, q_bstride, s, sums, a_bstride, M, Y, ldy, y_bstride,
                                   static_cast<cudaStream_t>(stream));
}

int b2s_mul_mat_q8(const b2s_tensor* W, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums, int64_t M,
                   float* Y, int64_t ldy, void* stream) {
    return b2s_mul_mat_q8_ex(W, q, ldq, s, sums, M, Y, ldy, 0, stream);
}

int b2s_mul_mat_q8_epi(const b2s_tensor* W, const int8_t* q, int64_t ldq, const float* s, const int32_t* sums,
                       int64_t M, float* Y, int64_t ldy, const float* bias, const float* residual, int64_t ld_res,
                       int act, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    b2s::I2sWeight w;
    if ((rc = weight_view(W, &w, "W"))) return rc;
    if (!q || !s || !sums || !Y) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_epi: q, s, sums and Y must be non-NULL");
    if (M < 0 || ldq < w.K || ldy < w.N) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_epi: bad M/ldq/ldy");
    if (act != 0 && act != 1) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_epi: act must be 0 (none) or 1 (gelu)");
    if (residual && ld_res < w.N) return fail(B2S_ERR_INVALID_ARG, "mul_mat_q8_epi: ld_res < N");
    b2s::Epilogue epi{bias, residual, ld_res, act};
    return mul_mat_q8_impl(w, q, ldq, s, sums, M, Y, ldy, 0, static_cast<cudaStream_t>(stream), epi);
}

int b2s_mul_mat(const b2s_tensor* W, const b2s_tensor* X, b2s_tensor* Y, void* workspace, size_t workspace_bytes,
                void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (W && W->ne[2] > 1) return mul_mat_batched(W, X, Y, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
    b2s::I2sWeight w;
    if ((rc = weight_view(W, &w, "W"))) return rc;
    int64_t M, Kx, ldx, My, Ny, ldy;
    if ((rc = f32_rows(X, "X", &M, &Kx, &ldx))) return rc;
    if ((rc = f32_rows(Y, "Y", &My, &Ny, &ldy))) return rc;
    if (Kx != w.K) return fail(B2S_ERR_INVALID_ARG, "X ne0 (%lld) != W ne0 (%lld)", (long long)Kx, (long long)w.K);
    if (Ny != w.N || My != M)
        return fail(B2S_ERR_INVALID_ARG, "Y must be ne=[%lld,%lld], got [%lld,%lld]", (long long)w.N, (long long)M,
                    (long long)Ny, (long long)My);
    const WsLayout l = act_ws(M, w.K);
    if (!workspace || workspace_bytes < l.total)
        return fail(B2S_ERR_WORKSPACE, "mul_mat needs %zu workspace bytes, got %zu", l.total, workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(B2S_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int8_t* q = reinterpret_cast<int8_t*>(ws + l.q_off);
    float* s = reinterpret_cast<float*>(ws + l.s_off);
    int32_t* sums = reinterpret_cast<int32_t*>(ws + l.sum_off);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = launched(b2s::launch_act_quant(static_cast<const float*>(X->data), ldx, nullptr, false, 0.0f, M, w.K, q,
                                             l.ldq, s, sums, st),
                       "act_quant launch")))
        return rc;
    // workspace beyond the activation layout (b2s_mul_mat_workspace_size includes it) holds split-K partials
    const size_t sk_off = a256(l.total);
    void* sk = workspace_bytes > sk_off ? ws + sk_off : nullptr;
    return mul_mat_q8_impl(w, q, l.ldq, s, sums, M, static_cast<float*>(Y->data), ldy, 0, st, b2s::Epilogue{}, sk,
                           sk ? workspace_bytes - sk_off : 0);
}

int b2s_ffn_gate_up_sqrelu_q8(const b2s_tensor* W_gate, const b2s_tensor* W_up, const int8_t* q, int64_t ldq,
                              const float* s, const int32_t* sums, int64_t M, float* P, int64_t ldp, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    b2s::I2sWeight wg, wu;
    if ((rc = weight_view(W_gate, &wg, "W_gate"))) return rc;
    if ((rc = weight_view(W_up, &wu, "W_up"))) return rc;
    if (wg.N != wu.N || wg.K != wu.K) return fail(B2S_ERR_INVALID_ARG, "W_gate and W_up shapes differ");
    if (!q || !s || !sums || !P) return fail(B2S_ERR_INVALID_ARG, "gate_up: q, s, sums and P must be non-NULL");
    if (M < 0 || ldq < wg.K || ldp < wg.N) return fail(B2S_ERR_INVALID_ARG, "gate_up: bad M/ldq/ldp");
    if (M == 0) return B2S_OK;
    return run_tc(wg, &wu, q, ldq, s, sums, M, P, ldp, 1, static_cast<cudaStream_t>(stream));
}

static void ffn_layout(int64_t M, int64_t H, int64_t F, WsLayout* l1, size_t* p_off, WsLayout* l2,
                       size_t* sk_off, size_t* sk_bytes) {
    *l1 = act_ws(M, H);
    *p_off = a256(l1->total);
    *l2 = act_ws(M, F, *p_off + sizeof(float) * (size_t)(M * F));
    *sk_off = a256(l2->total);
    *sk_bytes = std::max(b2s::splitk_ws_bytes(M, F, 64), b2s::splitk_ws_bytes(M, H, 128));
}

size_t b2s_ffn_block_workspace_size(int64_t M, int64_t H, int64_t F) {
    if (M <= 0 || H <= 0 || F <= 0) return 0;
    WsLayout l1, l2;
    size_t p_off, sk_off, sk_bytes;
    ffn_layout(M, H, F, &l1, &p_off, &l2, &sk_off, &sk_bytes);
    return sk_off + sk_bytes;
}

int b2s_ffn_block(const float* X, int64_t M, const float* g1, const float* g2, float eps, const b2s_tensor* W_gate,
                  const b2s_tensor* W_up, const b2s_tensor* W_down, float* Y, void* workspace, size_t workspace_bytes,
                  void* stream) {
    int rc = check_device();
    if (rc) return rc;
    b2s::I2sWeight wg, wu, wd;
    if ((rc = weight_view(W_gate, &wg, "W_gate"))) return rc;
    if ((rc = weight_view(W_up, &wu, "W_up"))) return rc;
    if ((rc = weight_view(W_down, &wd, "W_down"))) return rc;
    const int64_t H = wg.K, F = wg.N;
    if (wu.K != H || wu.N != F || wd.K != F || wd.N != H)
        return fail(B2S_ERR_INVALID_ARG, "FFN weights must be gate/up [H->F] and down [F->H]");
    if (!X || !Y) return fail(B2S_ERR_INVALID_ARG, "ffn_block: X and Y must be non-NULL");
    if (M <= 0) return M == 0 ? B2S_OK : fail(B2S_ERR_INVALID_ARG, "ffn_block: M < 0");
    WsLayout l1, l2;
    size_t p_off, sk_off, sk_bytes;
    ffn_layout(M, H, F, &l1, &p_off, &l2, &sk_off, &sk_bytes);
    if (!workspace || workspace_bytes < sk_off + sk_bytes)
        return fail(B2S_ERR_WORKSPACE, "ffn_block needs %zu workspace bytes, got %zu", sk_off + sk_bytes,
                    workspace_bytes);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return fail(B2S_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int8_t* q1 = reinterpret_cast<int8_t*>(ws + l1.q_off);
    float* s1 = reinterpret_cast<float*>(ws + l1.s_off);
    int32_t* u1 = reinterpret_cast<int32_t*>(ws + l1.sum_off);
    float* P = reinterpret_cast<float*>(ws + p_off);
    int8_t* q2 = reinterpret_cast<int8_t*>(ws + l2.q_off);
    float* s2 = reinterpret_cast<float*>(ws + l2.s_off);
    int32_t* u2 = reinterpret_cast<int32_t*>(ws + l2.sum_off);
    if ((rc = launched(b2s::launch_act_quant(X, H, g1, true, eps, M, H, q1, l1.ldq, s1, u1, st), "rms_norm_act_quant 1")))
        return rc;
    void* sk = ws + sk_off;
    if ((rc = run_tc(wg, &wu, q1, l1.ldq, s1, u1, M, P, F, 1, st, b2s::Epilogue{}, sk, sk_bytes))) return rc;
    if ((rc = launched(b2s::launch_act_quant(P, F, g2, true, eps, M, F, q2, l2.ldq, s2, u2, st), "rms_norm_act_quant 2")))
        return rc;
    return mul_mat_q8_impl(wd, q2, l2.ldq, s2, u2, M, Y, H, 0, st, b2s::Epilogue{}, sk, sk_bytes);
}

int b2s_norm(const float* x, const float* g, const float* b, int64_t M, int64_t K, int64_t ldx, float eps, int kind,
             float* y, int64_t ldy, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!x || !y) return fail(B2S_ERR_INVALID_ARG, "norm: x and y must be non-NULL");
    if (kind != 0 && kind != 1) return fail(B2S_ERR_INVALID_ARG, "norm: kind must be 0 (RMSNorm) or 1 (LayerNorm)");
    if (M < 0 || K <= 0 || ldx < K || ldy < K || K > 0x7fffffff) return fail(B2S_ERR_INVALID_ARG, "norm: bad shape");
    return launched(b2s::launch_norm(kind, false, x, ldx, g, b, eps, M, K, y, ldy, nullptr, 0, nullptr, nullptr,
                                     static_cast<cudaStream_t>(stream)),
                    "norm launch");
}

int b2s_norm_act_quant(const float* x, const float* g, const float* b, int64_t M, int64_t K, int64_t ldx, float eps,
                       int kind, int8_t* q, int64_t ldq, float* s, int32_t* sums, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!x || !q || !s) return fail(B2S_ERR_INVALID_ARG, "norm_act_quant: x, q and s must be non-NULL");
    if (kind != 0 && kind != 1) return fail(B2S_ERR_INVALID_ARG, "norm_act_quant: kind must be 0 or 1");
    if (M < 0 || K <= 0 || ldx < K || ldq < K || K > 0x7fffffff) return fail(B2S_ERR_INVALID_ARG, "norm_act_quant: bad shape");
    return launched(b2s::launch_norm(kind, true, x, ldx, g, b, eps, M, K, nullptr, 0, q, ldq, s, sums,
                                     static_cast<cudaStream_t>(stream)),
                    "norm_act_quant launch");
}

int b2s_rope_neox(float* x, int64_t M, int n_heads, int head_dim, int64_t ld, float theta_base, int pos0,
                  void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!x || M < 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1) || ld < (int64_t)n_heads * head_dim)
        return fail(B2S_ERR_INVALID_ARG, "rope_neox: bad arguments");
    return launched(b2s::launch_rope_neox(x, M, n_heads, head_dim, ld, theta_base, pos0, static_cast<cudaStream_t>(stream)),
                    "rope launch");
}

int b2s_attention(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv, int64_t M,
                  int n_heads, int n_kv_heads, int head_dim, float scale, int causal, float* o, int64_t ldo,
                  void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!q || !k || !v || !o) return fail(B2S_ERR_INVALID_ARG, "attention: NULL tensor");
    if (M <= 0 || M > 65536 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0)
        return fail(B2S_ERR_INVALID_ARG, "attention: bad shape");
    if (ldq < (int64_t)n_heads * head_dim || ldo < (int64_t)n_heads * head_dim || ldk < (int64_t)n_kv_heads * head_dim ||
        ldv < (int64_t)n_kv_heads * head_dim)
        return fail(B2S_ERR_INVALID_ARG, "attention: leading dimensions too small");
    if (!b2s::attention_supported((int)M, head_dim, ldq, ldk, ldv, ldo, q, k, v, o))
        return fail(B2S_ERR_UNSUPPORTED,
                    "attention: needs head_dim %% 8 == 0 and <= 128, leading dimensions %% 4 == 0 and 16-byte "
                    "aligned tensors");
    return launched(b2s::launch_attention(q, ldq, k, ldk, v, ldv, 1, (int)M, n_heads, n_kv_heads, head_dim, scale,
                                          causal != 0, o, ldo, static_cast<cudaStream_t>(stream)),
                    "attention");
}

int b2s_attention_tc(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv, int64_t M,
                     int n_heads, int n_kv_heads, int head_dim, float scale, int causal, float* o, int64_t ldo,
                     void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!q || !k || !v || !o) return fail(B2S_ERR_INVALID_ARG, "attention_tc: NULL tensor");
    if (M <= 0 || M > 65536 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0)
        return fail(B2S_ERR_INVALID_ARG, "attention_tc: bad shape");
    if (ldq < (int64_t)n_heads * head_dim || ldo < (int64_t)n_heads * head_dim || ldk < (int64_t)n_kv_heads * head_dim ||
        ldv < (int64_t)n_kv_heads * head_dim)
        return fail(B2S_ERR_INVALID_ARG, "attention_tc: leading dimensions too small");
    if (!b2s::attention_tc_supported((int)M, n_heads, n_kv_heads, head_dim, causal != 0, ldq, ldk, ldv, ldo, q, k, v,
                                     o))
        return fail(B2S_ERR_UNSUPPORTED,
                    "attention_tc: needs head_dim %% 8 == 0 and <= 128, 128 %% (n_heads / n_kv_heads) == 0, at most "
                    "384 keys per query block, leading dimensions %% 4 == 0 and 16-byte aligned tensors");
    return launched(b2s::launch_attention_tc(q, ldq, k, ldk, v, ldv, 1, (int)M, n_heads, n_kv_heads, head_dim, scale,
                                             causal != 0, o, ldo, static_cast<cudaStream_t>(stream)),
                    "attention_tc");
}

int b2s_patch_embed(const float* img, int C, int H, int W, int P, const float* w, const float* bias, const float* pos,
                    int D, float* y, int64_t ldy, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!img || !w || !y || C <= 0 || P <= 0 || H % P || W % P || D <= 0 || ldy < D)
        return fail(B2S_ERR_INVALID_ARG, "patch_embed: bad arguments");
    return launched(b2s::launch_patch_embed(img, 1, C, H, W, P, w, bias, pos, D, y, ldy,
                                            static_cast<cudaStream_t>(stream)),
                    "patch_embed");
}

int b2s_embed_tokens_hash(const int32_t* tokens, int n, int dim, uint32_t seed, float* y, int64_t ldy, void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!tokens || !y || n < 0 || dim <= 0 || ldy < dim) return fail(B2S_ERR_INVALID_ARG, "embed_tokens: bad arguments");
    if (n == 0) return B2S_OK;
    return launched(b2s::launch_embed_tokens(tokens, n, dim, seed, y, ldy, static_cast<cudaStream_t>(stream)),
                    "embed_tokens launch");
}

int b2s_soft_max_ext(const float* x, const float* mask, int64_t mask_rows, int64_t M, int64_t N, float scale, float* y,
                     void* stream) {
    int rc = check_device();
    if (rc) return rc;
    if (!x || !y) return fail(B2S_ERR_INVALID_ARG, "soft_max_ext: x and y must be non-NULL");
    if (M < 0 || N <= 0 || N > (int64_t)0x7fffffff) return fail(B2S_ERR_INVALID_ARG, "soft_max_ext: bad shape");
    if (mask && mask_rows <= 0) return fail(B2S_ERR_INVALID_ARG, "soft_max_ext: mask_rows must be positive");
    return launched(b2s::launch_softmax(x, mask, mask ? mask_rows : 1, M, N, scale, y, static_cast<cudaStream_t>(stream)),
                    "softmax launch");
}

}  // extern "C"

namespace b2s {

bool tmap_u8_2d(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_c,
                uint32_t box_r, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || ld % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld};
    cuuint32_t box[2] = {box_c, box_r};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t ensure_dynamic_smem(const void* kfn, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;  // (kernel, device) -> size set
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    size_t& have = done[{kfn, dev}];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

}  // namespace b2s
