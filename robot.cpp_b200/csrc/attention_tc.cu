// attention_tc.cu -- softmax(Q K^T * scale [+ causal mask]) V on the tcgen05 tensor cores (sm_100a).
//
// The ggml sequence mul_mat(K, Q) -> soft_max_ext -> mul_mat(V, KQ) of one attention layer
// (src/models/smolvla/action_expert.cpp:771-774; ggml_flash_attn_ext in src/models/pi0/vlm.cpp:223-235) for
// `batch` sequences of T tokens, with GQA (heads / kv_heads query heads per K/V head).
//
// Precision: fp32 in and out, products on the tensor cores as 3xTF32. Every operand x is split by the
// threads that stage it into big = x rounded to TF32 (low 13 mantissa bits zero) and small = x - big (exact
// in fp32); each product is big*big + big*small + small*big with fp32 accumulation in tensor memory, which
// leaves a relative error of about 2^-21 per product (the small*small term and small's own TF32 rounding),
// inside the path's 1e-5 per-operator bar. The softmax uses the exact row maximum (all scores of a row are
// in tensor memory at once), exp2 on the special-function unit and an fp32 row sum.
//
// One CTA per (sequence, K/V head, block of 128 MMA rows); the 128 rows are G = heads / kv_heads query heads
// x 128 / G consecutive queries, so the heads that share a K/V head share its K and V tiles. 256 threads:
//   1. S = Q K^T: for each chunk of DC head dimensions, the threads load Q[128 rows][DC] and K[keys][DC]
//      (the next chunk's global loads in flight while the current chunk's MMAs run), split them into
//      no-swizzle K-major shared-memory tiles, and one thread issues kind::tf32 MMAs (M=128, N <= 256,
//      K=8) accumulating S[128][keys] in tensor memory columns [0, 384).
//   2. Row maxima: thread pairs (warps w and w+4 share TMEM lanes) read their row's S from tensor memory.
//   3. In stages of 64 keys: p = exp2((s - max) * scale * log2 e) (0 for masked keys), split into big/small
//      A tiles; V[64 keys][hd] split and transposed into K-major B tiles; 3x8 MMAs accumulate
//      O[128][hd] in tensor memory columns [384, 512).
//   4. O / row sum to global memory.
// Every mbarrier wait is bounded; on a timeout the CTA records the error word, drains its MMAs, frees tensor
// memory and returns.
#include <cuda_runtime.h>

#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

namespace atc {
constexpr int kThreads = 256;
constexpr int kRows = 128;        // MMA M: G heads x (128 / G) queries
constexpr int kOcol = 384;        // O accumulator columns [384, 384 + Npad); S uses [0, 384)
constexpr int kMaxKeys = 384;
constexpr int kPvKeys = 64;       // keys per P.V stage (two 32-column halves)
constexpr int kTmemCols = 512;
constexpr int kRegionBytes = 128 * 1024;  // operand tiles (phase 1 and phase 3 reuse the same bytes)
constexpr int kQv = kRows * 32 / 4 / kThreads;      // float4 per thread of a Q slice (DC <= 32)
constexpr int kKv = kMaxKeys * 32 / 4 / kThreads;   // float4 per thread of a K slice
constexpr int kVv = kPvKeys * 128 / 4 / kThreads;   // float4 per thread of a V stage (hd <= 128)
constexpr size_t kSmemBytes = kRegionBytes + 4 * kRows * sizeof(float) + 64 + 128;
}  // namespace atc

namespace {

// Byte offset of element (r, k) in a K-major, no-swizzle tile with Kc columns: 8-row x 16-byte core
// matrices, the Kc/4 core matrices of an 8-row group consecutive (LBO = 128 bytes), 8-row groups
// (Kc/4) * 128 bytes apart (SBO).
__device__ __forceinline__ uint32_t cm_off(int r, int k, int Kc) {
    return (uint32_t)((((r >> 3) * (Kc >> 2) + (k >> 2)) << 7) + ((r & 7) << 4) + ((k & 3) << 2));
}

// UMMA shared-memory descriptor, no swizzle: start, LBO (K direction), SBO (M/N direction), version 1.
__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    return d;  // layout type 0 (SWIZZLE_NONE) in bits 61-63
}

// Instruction descriptor, kind::tf32: D f32, A and B tf32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// x = big + small: big is x rounded to the nearest TF32 value (ties to even), small = x - big exactly.
__device__ __forceinline__ void tf32_split(float x, float& big, float& small) {
    const uint32_t u = __float_as_uint(x);
    big = __uint_as_float((u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u);
    small = __fsub_rn(x, big);
}

__device__ __forceinline__ void st_split4(uint8_t* big_tile, uint8_t* small_tile, uint32_t off, float4 x) {
    float4 b, s;
    tf32_split(x.x, b.x, s.x);
    tf32_split(x.y, b.y, s.y);
    tf32_split(x.z, b.z, s.z);
    tf32_split(x.w, b.w, s.w);
    *reinterpret_cast<float4*>(big_tile + off) = b;
    *reinterpret_cast<float4*>(small_tile + off) = s;
}

}  // namespace

__global__ void __launch_bounds__(atc::kThreads, 1)
attention_tc_kernel(const float* __restrict__ q, int64_t ldq, const float* __restrict__ k, int64_t ldk,
                    const float* __restrict__ v, int64_t ldv, float* __restrict__ o, int64_t ldo, int T, int heads,
                    int kv_heads, int hd, int DC, int Npad, float scale_log2e, int causal) {
    using namespace atc;
    extern __shared__ uint8_t at_smem_raw[];
    uint8_t* region = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_smem_raw) + 127) & ~uintptr_t(127));
    float* red = reinterpret_cast<float*>(region + kRegionBytes);  // [4][128]: max/sum partials of both halves
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 4 * kRows);  // 0: S MMAs, 1: P.V stage, 2: drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = heads / kv_heads, QB = kRows / G;
    const int g = blockIdx.x, b = blockIdx.y;
    const int qb = (int)(gridDim.z - 1u - blockIdx.z);  // heaviest (last) query block first
    const int q0 = qb * QB;
    const int n_keys = causal ? min(T, q0 + QB) : T;
    const int Tpad = (n_keys + 15) & ~15;
    const int64_t row0 = (int64_t)b * T;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // q/k/v come from the preceding kernels

    // One thread waits on a barrier phase; everyone learns whether it completed.
    auto wait_phase = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (tid == 0 && !mbar_wait(bar, parity)) *abort_flag = 1;
        __syncthreads();
        return *abort_flag == 0;
    };
    bool issued = false;

    // ------------------------------------------------------------------ 1. S = Q K^T
    const int ndc = hd / DC, f4r = DC / 4;
    const int qf4 = kRows * f4r, kf4 = Tpad * f4r;
    uint8_t* sQb = region;
    uint8_t* sQs = sQb + kRows * DC * 4;
    uint8_t* sKb = sQs + kRows * DC * 4;
    uint8_t* sKs = sKb + (size_t)Tpad * DC * 4;
    float4 rq[kQv], rk[kKv];
    auto load_slices = [&](int dc) {
        const int d0 = dc * DC;
#pragma unroll
        for (int i = 0; i < kQv; ++i) {
            const int f = tid + i * kThreads;
            rq[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (f < qf4) {
                const int r = f / f4r, c4 = f - r * f4r;
                const int qi = q0 + r % QB, h = g * G + r / QB;
                if (qi < T) rq[i] = __ldg(reinterpret_cast<const float4*>(q + (row0 + qi) * ldq + (int64_t)h * hd + d0) + c4);
            }
        }
#pragma unroll
        for (int i = 0; i < kKv; ++i) {
            const int f = tid + i * kThreads;
            rk[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (f < kf4) {
                const int j = f / f4r, c4 = f - j * f4r;
                if (j < n_keys) rk[i] = __ldg(reinterpret_cast<const float4*>(k + (row0 + j) * ldk + (int64_t)g * hd + d0) + c4);
            }
        }
    };
    auto store_slices = [&]() {
#pragma unroll
        for (int i = 0; i < kQv; ++i) {
            const int f = tid + i * kThreads;
            if (f < qf4) {
                const int r = f / f4r, c4 = f - r * f4r;
                st_split4(sQb, sQs, cm_off(r, 4 * c4, DC), rq[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < kKv; ++i) {
            const int f = tid + i * kThreads;
            if (f < kf4) {
                const int j = f / f4r, c4 = f - j * f4r;
                st_split4(sKb, sKs, cm_off(j, 4 * c4, DC), rk[i]);
            }
        }
    };
    load_slices(0);
    bool ok = true;
    for (int dc = 0; dc < ndc && ok; ++dc) {
        if (dc > 0 && !(ok = wait_phase(&bars[0], (uint32_t)(dc - 1) & 1u))) break;
        store_slices();
        if (dc + 1 < ndc) load_slices(dc + 1);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sbo = (uint32_t)f4r * 128u;
            const uint32_t aQ[3] = {smem_u32(sQb), smem_u32(sQb), smem_u32(sQs)};
            const uint32_t aK[3] = {smem_u32(sKb), smem_u32(sKs), smem_u32(sKb)};
            for (int n0 = 0; n0 < Tpad; n0 += 256) {
                const int N = min(256, Tpad - n0);
                const uint32_t idesc = idesc_tf32(kRows, N);
                for (int term = 0; term < 3; ++term)
                    for (int s = 0; s < DC / 8; ++s)
                        mma_tf32_ss(tmem + (uint32_t)n0, desc_noswz(aQ[term] + 256u * s, 128u, sbo),
                                    desc_noswz(aK[term] + (uint32_t)(n0 >> 3) * sbo + 256u * s, 128u, sbo), idesc,
                                    (dc > 0 || term > 0 || s > 0) ? 1u : 0u);
            }
            tc_commit(&bars[0]);
        }
        issued = true;
    }
    if (ok) ok = wait_phase(&bars[0], (uint32_t)(ndc - 1) & 1u);

    // ------------------------------------------------------------------ 2. row maxima
    const int quad = warp & 3, hf = warp >> 2;
    const int row = 32 * quad + lane;
    const int qi = q0 + row % QB, h = g * G + row / QB;
    const int nk_row = (qi < T) ? (causal ? qi + 1 : T) : 0;  // this row's keys: j < nk_row
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * quad) << 16);
    float m = -INFINITY, l = 0.0f;
    if (ok) {
        tc_fence_after();
        for (int c = hf; 32 * c < Tpad; c += 2) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(lane_addr + 32u * c, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (32 * c + j < nk_row) m = fmaxf(m, __uint_as_float(r[j]));
        }
        red[hf * kRows + row] = m;
        __syncthreads();
        m = fmaxf(red[row], red[kRows + row]);
    }

    // ------------------------------------------------------------------ 3. P = softmax numerators, O = P V
    uint8_t* sPb = region;
    uint8_t* sPs = sPb + kRows * kPvKeys * 4;
    uint8_t* sVb = sPs + kRows * kPvKeys * 4;
    uint8_t* sVs = sVb + (size_t)Npad * kPvKeys * 4;
    const int nst = (n_keys + kPvKeys - 1) / kPvKeys;
    const int hd4 = hd / 4, vf4 = kPvKeys * hd4;
    float4 rv[kVv];
    auto load_v = [&](int st_i) {
        const int j0 = st_i * kPvKeys;
#pragma unroll
        for (int i = 0; i < kVv; ++i) {
            const int f = tid + i * kThreads;
            rv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (f < vf4) {
                const int j = f / hd4, c4 = f - j * hd4;
                if (j0 + j < n_keys)
                    rv[i] = __ldg(reinterpret_cast<const float4*>(v + (row0 + j0 + j) * ldv + (int64_t)g * hd) + c4);
            }
        }
    };
    if (ok) {
        // rows hd..Npad-1 of the transposed V tiles stay zero for the whole phase
        for (int e = tid; e < (Npad - hd) * kPvKeys; e += kThreads) {
            const int n = hd + e / kPvKeys, kk = e % kPvKeys;
            *reinterpret_cast<float*>(sVb + cm_off(n, kk, kPvKeys)) = 0.0f;
            *reinterpret_cast<float*>(sVs + cm_off(n, kk, kPvKeys)) = 0.0f;
        }
        load_v(0);
    }
    for (int st_i = 0; st_i < nst && ok; ++st_i) {
        if (st_i > 0 && !(ok = wait_phase(&bars[1], (uint32_t)(st_i - 1) & 1u))) break;
        {
            const int c = 2 * st_i + hf;  // this half's 32 keys of the stage
            uint32_t r[32];
            tmem_ld_32x32b_x32(lane_addr + 32u * c, r);
            tc_wait_ld();
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
                float4 p;
                float* pp = &p.x;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int key = 32 * c + 4 * j4 + t;
                    const float e = (key < nk_row) ? ex2_approx((__uint_as_float(r[4 * j4 + t]) - m) * scale_log2e) : 0.0f;
                    pp[t] = e;
                    l += e;
                }
                st_split4(sPb, sPs, cm_off(row, 32 * hf + 4 * j4, kPvKeys), p);
            }
        }
#pragma unroll
        for (int i = 0; i < kVv; ++i) {  // V[key][d..d+3] -> B tile rows d..d+3 (N = head dim), column key
            const int f = tid + i * kThreads;
            if (f < vf4) {
                const int j = f / hd4, d = 4 * (f - j * hd4);
                const float x[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    float bg, sm;
                    tf32_split(x[t], bg, sm);
                    *reinterpret_cast<float*>(sVb + cm_off(d + t, j, kPvKeys)) = bg;
                    *reinterpret_cast<float*>(sVs + cm_off(d + t, j, kPvKeys)) = sm;
                }
            }
        }
        if (st_i + 1 < nst) load_v(st_i + 1);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sbo = (uint32_t)(kPvKeys / 4) * 128u;
            const uint32_t aP[3] = {smem_u32(sPb), smem_u32(sPb), smem_u32(sPs)};
            const uint32_t bV[3] = {smem_u32(sVb), smem_u32(sVs), smem_u32(sVb)};
            const uint32_t idesc = idesc_tf32(kRows, Npad);
            for (int term = 0; term < 3; ++term)
                for (int s = 0; s < kPvKeys / 8; ++s)
                    mma_tf32_ss(tmem + (uint32_t)kOcol, desc_noswz(aP[term] + 256u * s, 128u, sbo),
                                desc_noswz(bV[term] + 256u * s, 128u, sbo), idesc,
                                (st_i > 0 || term > 0 || s > 0) ? 1u : 0u);
            tc_commit(&bars[1]);
        }
    }
    if (ok && nst > 0) ok = wait_phase(&bars[1], (uint32_t)(nst - 1) & 1u);

    // ------------------------------------------------------------------ 4. O / l to global memory
    if (ok) {
        red[(2 + hf) * kRows + row] = l;
        __syncthreads();
        const float lt = red[2 * kRows + row] + red[3 * kRows + row];
        const float inv = (lt > 0.0f) ? __fdiv_rn(1.0f, lt) : 0.0f;
        tc_fence_after();
        for (int c = hf; 16 * c < Npad; c += 2) {
            uint32_t r[16];
            tmem_ld16(lane_addr + (uint32_t)kOcol + 16u * c, r);
            tc_wait_ld();
            if (qi < T) {
                float* orow = o + (row0 + qi) * ldo + (int64_t)h * hd + 16 * c;
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4)
                    if (16 * c + 4 * j4 < hd)
                        *reinterpret_cast<float4*>(orow + 4 * j4) =
                            make_float4(__uint_as_float(r[4 * j4]) * inv, __uint_as_float(r[4 * j4 + 1]) * inv,
                                        __uint_as_float(r[4 * j4 + 2]) * inv, __uint_as_float(r[4 * j4 + 3]) * inv);
            }
        }
    } else if (tid == 0 && issued) {  // a wait ran out: let the issued MMAs finish before TMEM is released
        tc_commit(&bars[2]);
        mbar_wait(&bars[2], 0, 2u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    griddep_launch();
}

// Largest multiple of 8 (<= 32) dividing hd: the head-dimension chunk of the S phase.
static int atc_dc(int hd) {
    for (int dc = 32; dc >= 8; dc -= 8)
        if (hd % dc == 0) return dc;
    return 0;
}

bool attention_tc_supported(int T, int heads, int kv_heads, int hd, bool causal, int64_t ldq, int64_t ldk, int64_t ldv,
                            int64_t ldo, const void* q, const void* k, const void* v, const void* o) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (T <= 0 || hd <= 0 || hd % 8 != 0 || hd > 128 || kv_heads <= 0 || heads % kv_heads != 0) return false;
    const int G = heads / kv_heads;
    if (atc::kRows % G != 0) return false;
    const int max_keys = causal ? min(T, (T + atc::kRows / G - 1) / (atc::kRows / G) * (atc::kRows / G)) : T;
    return max_keys <= atc::kMaxKeys && atc_dc(hd) > 0 && ldq % 4 == 0 && ldk % 4 == 0 && ldv % 4 == 0 &&
           ldo % 4 == 0 && a16(q) && a16(k) && a16(v) && a16(o);
}

cudaError_t launch_attention_tc(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                                int batch, int T, int heads, int kv_heads, int hd, float scale, bool causal, float* o,
                                int64_t ldo, cudaStream_t st) {
    if (batch <= 0 || T <= 0) return cudaSuccess;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(attention_tc_kernel), atc::kSmemBytes);
    if (e != cudaSuccess) return e;
    const int G = heads / kv_heads, QB = atc::kRows / G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)kv_heads, (unsigned)batch, (unsigned)((T + QB - 1) / QB));
    cfg.blockDim = dim3(atc::kThreads);
    cfg.dynamicSmemBytes = atc::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const float scale_log2e = scale * 1.4426950408889634f;
    const int Npad = (hd + 15) & ~15;
    return cudaLaunchKernelEx(&cfg, attention_tc_kernel, q, ldq, k, ldk, v, ldv, o, ldo, T, heads, kv_heads, hd,
                              atc_dc(hd), Npad, scale_log2e, causal ? 1 : 0);
}

}  // namespace b2s
