// gemm_i2s_tc.cu -- prefill-size i2_s x int8 GEMM on the sm_100a tensor cores (tcgen05 kind::i8).
//
// Output tile: 128 weight rows (n) x BN tokens (m), BN a multiple of 16 up to 256.
// The weights are the MMA's A operand and live in tensor memory; the activations are the B operand
// in shared memory:
//   * warp 4 (producer) TMA-loads, per 128-wide K step, the packed weight tile (128 rows x 32 bytes,
//     local HBM, no multicast) and the int8 activation tile (BN rows x 128 bytes, 128B swizzle) into a
//     ring of shared-memory stages;
//   * warps 0-3 (converters) each own 32 TMEM lanes = 32 weight rows: a thread reads its row's
//     32 packed bytes from shared memory, decodes the 2-bit codes to signed int8 {-1,0,1} in
//     registers ((c + 0x7F) ^ 0x80 per byte) and stores the 128 int8 values with one
//     tcgen05.st.32x32b.x32 into a ring of TMEM A stages, so the unpacked weights never touch
//     shared-memory bandwidth;
//   * warp 5 (MMA) issues, per K step, four tcgen05.mma.cta_group::1.kind::i8 (M=128, N=BN, K=32)
//     reading A from TMEM and B through a K-major SW128 descriptor, accumulating int32 in TMEM;
//   * warps 0-3 then read the accumulator back (tcgen05.ld) and write fp32
//     y = (float)acc * (w_scale / s[m]) with coalesced 128-byte stores (32 consecutive n per warp).
// Mode 1 (FFN gate/up) runs two weight matrices against the same activation tile into two
// accumulators and writes p = relu(g)^2 * u, fusing the squared-ReLU gate product into the epilogue.
//
// All waits are bounded; on a timeout the kernel records the error in g_device_error, drains what it
// issued (bounded), frees its TMEM and returns.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

namespace tc {
constexpr int kStages = 4;           // shared-memory ring (TMA)
constexpr int kAStages = 4;          // TMEM A ring, 32 columns each
constexpr int kBK = 128;             // K per stage (one 128-byte swizzle row of int8)
constexpr int kActStageBytes = 256 * 128;
constexpr int kWStageBytes = 128 * 32;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 128;    // accumulators start after the A ring

struct alignas(8) Bars {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t afull[kAStages];
    uint64_t aempty[kAStages];
    uint64_t accfull;
    uint64_t drain;
    uint32_t tmem_slot;
    uint32_t abort;
};

constexpr size_t kSmemAct = (size_t)kStages * kActStageBytes;
constexpr size_t kSmemW = (size_t)kStages * 2 * kWStageBytes;
constexpr size_t kSmemBytes = 1024 /*align slack*/ + kSmemAct + kSmemW + 2 * 256 * sizeof(float) + sizeof(Bars);
}  // namespace tc

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Packed word (4 bytes = 4 consecutive k of each bit-plane) -> signed int8 {-1,0,1} for plane g.
__device__ __forceinline__ uint32_t decode_plane(uint32_t w, int g) {
    const uint32_t c = (w >> (6 - 2 * g)) & 0x03030303u;
    return (c + 0x7F7F7F7Fu) ^ 0x80808080u;
}

__global__ void __launch_bounds__(tc::kThreads, 1)
gemm_i2s_tc_kernel(const __grid_constant__ CUtensorMap tmap_w0, const __grid_constant__ CUtensorMap tmap_w1,
                   const __grid_constant__ CUtensorMap tmap_q, const float* __restrict__ w0_scale,
                   const float* __restrict__ w1_scale, const float* __restrict__ s_act, float* __restrict__ y,
                   int64_t ldy, int M, int N, int Kp, int bn, int mode) {
    using namespace tc;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* act_sm = base;
    uint8_t* w_sm = base + kSmemAct;
    float* rfac = reinterpret_cast<float*>(w_sm + kSmemW);  // [2][256]
    Bars* bars = reinterpret_cast<Bars*>(rfac + 2 * 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * 128;
    const int m0 = blockIdx.y * bn;
    const int nkt = Kp / kBK;
    const int nw = mode == 1 ? 2 : 1;
    const uint32_t acc_stride = (uint32_t)((bn + 31) / 32 * 32);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->empty[i], 1 + 128);
        }
        for (int i = 0; i < kAStages; ++i) {
            mbar_init(&bars->afull[i], 128);
            mbar_init(&bars->aempty[i], 1);
        }
        mbar_init(&bars->accfull, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 4 && lane == 0) {
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_w0);
        if (mode == 1) tma_prefetch_desc(&tmap_w1);
    }
    if (warp == 0) {
        tmem_alloc(&bars->tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    // Per-token rescale factors w_scale / s[m] (one IEEE division per token and matrix).
    for (int i = threadIdx.x; i < nw * bn; i += blockDim.x) {
        const int j = i / bn, t = i - j * bn, m = m0 + t;
        const float ws = __ldg(j == 0 ? w0_scale : w1_scale);
        rfac[j * 256 + t] = (m < M) ? __fdiv_rn(ws, s_act[m]) : 0.0f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_slot;
    volatile uint32_t* abort_flag = &bars->abort;

    if (warp == 4) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint32_t tx = (uint32_t)bn * 128u + (uint32_t)nw * kWStageBytes;
            int issued = 0;
            for (int kt = 0; kt < nkt; ++kt) {
                const int s = kt % kStages;
                const uint32_t ph = (uint32_t)(kt / kStages) & 1u;
                if (*abort_flag || !mbar_wait(&bars->empty[s], ph ^ 1u)) { *abort_flag = 1; break; }
                mbar_arrive_expect_tx(&bars->full[s], tx);
                tma_load_2d(act_sm + (size_t)s * kActStageBytes, &tmap_q, &bars->full[s], kt * kBK, m0);
                tma_load_2d(w_sm + (size_t)(s * 2 + 0) * kWStageBytes, &tmap_w0, &bars->full[s], kt * 32, n0);
                if (mode == 1)
                    tma_load_2d(w_sm + (size_t)(s * 2 + 1) * kWStageBytes, &tmap_w1, &bars->full[s], kt * 32, n0);
                ++issued;
            }
            if (*abort_flag) {  // drain copies still in flight before the CTA's shared memory goes away
                for (int kt = (issued > kStages ? issued - kStages : 0); kt < issued; ++kt)
                    mbar_wait(&bars->full[kt % kStages], (uint32_t)(kt / kStages) & 1u, 2u);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_i8(128, bn);
            int ai = 0;
            bool issued_any = false;
            for (int kt = 0; kt < nkt && !*abort_flag; ++kt) {
                const int s = kt % kStages;
                const uint32_t ph = (uint32_t)(kt / kStages) & 1u;
                if (!mbar_wait(&bars->full[s], ph)) { *abort_flag = 1; break; }
                const uint32_t b_base = smem_u32(act_sm + (size_t)s * kActStageBytes);
                bool ok = true;
                for (int j = 0; j < nw; ++j, ++ai) {
                    const int a = ai % kAStages;
                    const uint32_t aph = (uint32_t)(ai / kAStages) & 1u;
                    if (!mbar_wait(&bars->afull[a], aph)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + kAccCol + (uint32_t)j * acc_stride;
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk) {
                        const uint64_t bdesc = umma_desc_k_sw128(b_base + kk * 32);
                        const uint32_t a_tmem = tmem_base + (uint32_t)(a * 32 + kk * 8);
                        tc_mma_i8_ts(d_tmem, a_tmem, bdesc, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
                    }
                    issued_any = true;
                    tc_commit(&bars->aempty[a]);
                }
                if (!ok) { *abort_flag = 1; break; }
                tc_commit(&bars->empty[s]);
            }
            if (!*abort_flag) {
                tc_commit(&bars->accfull);
            } else if (issued_any) {
                tc_commit(&bars->drain);
                mbar_wait(&bars->drain, 0, 2u);
            }
        }
    } else {
        // ------------------------------------------------------------------ converters (warps 0-3)
        const int row = threadIdx.x;  // TMEM lane == weight row within the tile
        const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
        int ai = 0;
        for (int kt = 0; kt < nkt && !*abort_flag; ++kt) {
            const int s = kt % kStages;
            const uint32_t ph = (uint32_t)(kt / kStages) & 1u;
            if (!mbar_wait(&bars->full[s], ph)) { *abort_flag = 1; break; }
            uint4 pk[2][2];
            for (int j = 0; j < nw; ++j) {
                const uint4* src = reinterpret_cast<const uint4*>(w_sm + (size_t)(s * 2 + j) * kWStageBytes + row * 32);
                pk[j][0] = src[0];
                pk[j][1] = src[1];
            }
            mbar_arrive(&bars->empty[s]);
            bool ok = true;
            for (int j = 0; j < nw; ++j, ++ai) {
                const int a = ai % kAStages;
                const uint32_t aph = (uint32_t)(ai / kAStages) & 1u;
                if (!mbar_wait(&bars->aempty[a], aph ^ 1u)) { ok = false; break; }
                const uint32_t w[8] = {pk[j][0].x, pk[j][0].y, pk[j][0].z, pk[j][0].w,
                                       pk[j][1].x, pk[j][1].y, pk[j][1].z, pk[j][1].w};
                uint32_t out[32];
#pragma unroll
                for (int g = 0; g < 4; ++g)
#pragma unroll
                    for (int p = 0; p < 8; ++p) out[8 * g + p] = decode_plane(w[p], g);
                tmem_st_32x32b_x32(lane_base + (uint32_t)(a * 32), out);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(&bars->afull[a]);
            }
            if (!ok) { *abort_flag = 1; break; }
        }
        // ------------------------------------------------------------------ epilogue (warps 0-3)
        if (!*abort_flag && mbar_wait(&bars->accfull, 0)) {
            tc_fence_after();
            const int n = n0 + row;
            for (int c = 0; c < bn / 16; ++c) {
                uint32_t a0[16], a1[16];
                tmem_ld_32x32b_x16(lane_base + kAccCol + (uint32_t)(c * 16), a0);
                if (mode == 1) tmem_ld_32x32b_x16(lane_base + kAccCol + acc_stride + (uint32_t)(c * 16), a1);
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = c * 16 + j, m = m0 + t;
                    float v = __fmul_rn((float)(int32_t)a0[j], rfac[t]);
                    if (mode == 1) {
                        const float u = __fmul_rn((float)(int32_t)a1[j], rfac[256 + t]);
                        const float r = v > 0.0f ? v : 0.0f;
                        v = __fmul_rn(__fmul_rn(r, r), u);
                    }
                    if (m < M && n < N) y[(int64_t)m * ldy + n] = v;
                }
            }
        } else {
            *abort_flag = 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

cudaError_t launch_gemm_i2s_tc(const TcGemmArgs& a, cudaStream_t st) {
    static bool attr_set = false;  // per process; the attribute is per function, device-independent
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i2s_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc::kSmemBytes);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    dim3 grid((unsigned)ceil_div(a.N, 128), (unsigned)ceil_div(a.M, a.bn));
    gemm_i2s_tc_kernel<<<grid, tc::kThreads, tc::kSmemBytes, st>>>(a.tmap_w0, a.tmap_w1, a.tmap_q, a.w0_scale,
                                                                     a.w1_scale, a.s, a.y, a.ldy, a.M, a.N, a.Kp,
                                                                     a.bn, a.mode);
    return cudaGetLastError();
}

}  // namespace b2s
