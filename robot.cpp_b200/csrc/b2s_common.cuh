// b2s_common.cuh -- shared device helpers for the sm_100a i2_s kernels.
//
// Inline PTX wrappers for mbarriers, TMA tile loads (no multicast, local memory only), and the
// tcgen05 tensor-memory / MMA instructions; every spin-wait is bounded and reports through a
// device-side error word instead of hanging.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace b2s {

// Error word set by kernels whose bounded waits ran out (read back by b2s_device_error()).
// Bit 0: a pipeline mbarrier wait gave up. Bit 1: a drain wait at exit gave up.
extern __device__ unsigned int g_device_error;

constexpr int kQK = 128;  // weights per i2_s interleave block

__host__ __device__ constexpr int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }
__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------- act-quant scalar semantics
// Per-token scale of the act-quant: 127/max(1e-5, amax). For amax <= 1e-5f the reference keeps its
// double 1e-5 floor, whose quotient rounds to 12700000.0f; otherwise the fp32 quotient is correctly
// rounded, equal to rounding the double quotient (double rounding is innocuous for division).
__device__ __forceinline__ float actq_scale(float amax) {
    return (amax <= 1e-5f) ? 12700000.0f : __fdiv_rn(127.0f, amax);
}
// round-half-away-from-zero of the fp32 product, clamped to int8.
__device__ __forceinline__ int actq_round(float x, float s) {
    float r = roundf(__fmul_rn(x, s));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int)r;
}

// ---------------------------------------------------------------- warp / block reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- deterministic transcendental functions
// exp and tanh of the library's fp32 kernels, built from IEEE operations only (fused multiply-adds,
// products, sums) so that the CPU oracle reproduces them bit for bit: Cody and Waite's range
// reduction x = n ln2 + r (|r| <= ln2/2, ln2 split into a 16-bit head and a tail) and the degree-7
// Taylor polynomial of e^r in Horner form, scaled by 2^n. Relative error below 2 ulp; inputs below
// -86 return 0 (no subnormal results), above 88 saturate at e^88. Written without branches (the
// out-of-range inputs are clamped and their result selected away) so that unrolled loops of independent
// calls interleave.
__device__ __forceinline__ float det_expf(float x) {
    const bool low = !(x >= -86.0f);  // also NaN -> 0
    const float xc = low ? -86.0f : fminf(x, 88.0f);
    const float n = rintf(__fmul_rn(xc, 1.44269502162933349609375f));
    float r = __fmaf_rn(-n, 0.693145751953125f, xc);
    r = __fmaf_rn(-n, 1.428606765330187045e-06f, r);
    float p = 1.98412698412698412698e-04f;
    p = __fmaf_rn(p, r, 1.38888888888888888889e-03f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-03f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-02f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const float v = __fmul_rn(p, __int_as_float(((int)n + 127) << 23));
    return low ? 0.0f : v;
}
// 1 / d for a normal d > 0: the bit-pattern seed 0x7EF311C3 - bits(d) (within 12.5%) and three
// Newton-Raphson steps y <- y + y (1 - d y), each two fused multiply-adds; relative error below 2^-22.
// Every step is an IEEE operation, so the CPU oracle's restatement gives the same bits.
__device__ __forceinline__ float det_recipf(float d) {
    float y = __uint_as_float(0x7EF311C3u - __float_as_uint(d));
#pragma unroll
    for (int i = 0; i < 3; ++i) y = __fmaf_rn(y, __fmaf_rn(-d, y, 1.0f), y);
    return y;
}
// tanh(u) = sign(u) (1 - 2 / (e^{2|u|} + 1)) with the reciprocal of det_recipf; |u| > 9 gives +-1. No
// branches: a NaN or |u| > 9 is clamped before the exponential and its result selected away.
__device__ __forceinline__ float det_tanhf(float u) {
    const float a = fminf(fabsf(u), 9.5f);
    const float t = __fsub_rn(1.0f, __fmul_rn(2.0f, det_recipf(__fadd_rn(det_expf(__fmul_rn(2.0f, a)), 1.0f))));
    return copysignf(fabsf(u) > 9.0f ? 1.0f : t, u);
}

// ---------------------------------------------------------------- programmatic dependent launch
// griddep_wait(): block until the preceding kernel in the stream (launched before this one with
// programmatic stream serialization allowed) has completed and its memory is visible; a no-op otherwise.
// griddep_launch(): allow the next such kernel to start launching its CTAs now.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- shared-memory addresses
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// d0 = fma(a0, b0, d0), d1 = fma(a1, b1, d1) as one paired fp32 instruction (each lane an IEEE fma, round to
// nearest, no flush to zero: the same results as two __fmaf_rn).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    uint64_t a, b, c;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(d0), "f"(d1));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(b));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(c));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on one mbarrier phase: gives up after limit_ns of wall time (one second by default;
// try_wait may itself suspend for an implementation-defined interval, so the bound is on %globaltimer,
// not on a poll count). Returns false on timeout and records it in g_device_error.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int err_bit = 1u,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 15u && global_timer_ns() - t0 > limit_ns) break;
        if (i > 64) __nanosleep(64);
    }
    atomicOr(&g_device_error, err_bit);
    return false;
}

// ---------------------------------------------------------------- TMA (tile mode, no multicast)
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// Non-tensor bulk copy global -> shared completing on an mbarrier (addresses 16-byte aligned, bytes a
// multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Tile store shared -> global (bulk-group completion). Coordinates are never negative here; rows and
// columns outside the tensor map's extent are not written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store of this thread has completed (its global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA store reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::i8, int32 accumulate.
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] += A[tmem] * B[smem desc], kind::i8, always accumulating (no per-call predicate computation).
__device__ __forceinline__ void tc_mma_i8_ts_acc(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.eq.u32 p, 1, 1;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc)
        : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::i8.
__device__ __forceinline__ void tc_mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread i of the warp moves lane (base_lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 16 lanes x 16 columns of 32-bit: thread i of the warp gets lane (base_lane + (i >> 2) + 8 * (i & 1)),
// columns col + ((i >> 1) & 1) + 2 * j for j = 0..7 (the 16x64b shape, 8 repetitions along the columns).
__device__ __forceinline__ void tmem_ld_16x64b_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.16x64b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
// 32 lanes x 16 columns of 32-bit: thread i of the warp gets lane (base_lane + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// UMMA shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// rows of 128 bytes, 8-row atoms of 1024 bytes (stride byte offset), leading byte offset unused (1),
// version 1 (sm_100), layout type 2 (SWIZZLE_128B). The start address must lie in a 1024-byte
// aligned atom; advancing along K inside the 128-byte row adds the byte offset to the start address.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);  // start address [0,14)
    d |= (uint64_t)1u << 16;                       // leading byte offset (16 B units) [16,30)
    d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset [32,46)
    d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                       // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::i8: D s32, A and B signed int8, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4)                          // D format: s32
           | (1u << 7)                        // A: signed 8-bit
           | (1u << 10)                       // B: signed 8-bit
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Parameter generator of the random-init models: 32 hash bits of element idx of tensor `tensor`
// (murmur3's 32-bit finalizer applied to the seed, the tensor id and the index).
__host__ __device__ __forceinline__ uint32_t param_mix(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}
__host__ __device__ __forceinline__ uint32_t param_bits(uint32_t seed, uint32_t tensor, uint32_t idx) {
    const uint32_t t = param_mix(seed ^ param_mix(tensor * 0x9E3779B1u + 0x7F4A7C15u));
    return param_mix(t ^ (idx * 0x85EBCA77u + 0x165667B1u));
}

}  // namespace b2s
