// gemm_i2s_tc.cu -- prefill-size i2_s x int8 GEMM on the sm_100a tensor cores (tcgen05 kind::i8).
//
// A CTA owns 128 weight rows and T tokens (T <= 320, as one or two MMA sub-tiles of bn_sub tokens).
// The weights are the MMA's A operand and live in tensor memory; the activations are the B operand in
// shared memory:
//   * warp 4 (producer) TMA-loads, per 128-wide K step, the packed weight tile (128 rows x 32 bytes from
//     local HBM, no multicast) and the int8 activation tile(s) (bn_sub rows x 128 bytes, 128B swizzle)
//     into a 4-stage shared-memory ring, weights and activations on separate barriers. The weight tiles
//     of the first ring round are requested before the kernel waits for its producer kernel
//     (programmatic dependent launch), so their HBM latency and their unpacking overlap the end of the
//     preceding kernel;
//   * warps 0-3 (converters) each own 32 TMEM lanes. A thread reads one weight row's 32 packed bytes and
//     extracts the unsigned 2-bit codes {0,1,2} of each bit-plane with one shift and one mask per 4
//     weights, then stores the 128 codes with one tcgen05.st.32x32b.x32 into the TMEM A stage that
//     pairs with the shared-memory stage: the unpacked weights never touch shared memory;
//   * warp 5 (MMA) issues, per 32-wide K slice and sub-tile, tcgen05.mma.cta_group::1.kind::i8 with
//     A = unsigned codes from TMEM and B = signed int8 activations (K-major SW128 descriptor), M=128,
//     N=bn_sub, int32 accumulators in TMEM. Since code = t + 1, acc = sum_k t_k q_k + sum_k q_k; the
//     epilogue subtracts the per-token activation sum (the method of the fork's ggml_vec_dot_i2_i8_s);
//   * warps 0-3 read the accumulators back (tcgen05.ld, two 16-token chunks per wait) and write fp32
//     y = (float)(acc - sum_q[m]) * (w_scale / s[m]) with coalesced stores.
// Mode 1 (FFN gate/up): in every converter warp, lanes 0-15 hold 16 gate rows and lanes 16-31 the 16 up
// rows of the same output columns, so one accumulator set holds both, and the epilogue writes
// p = relu(g)^2 * u (the squared-ReLU gate product fused into the GEMM). Without split-K it reads gate and
// up of the same output into one thread with 16x64b TMEM loads, stages the fp32 tile in the drained
// shared-memory ring and writes it with TMA tile stores; with split-K (or an output TMA cannot address)
// it pairs the 32x32b-loaded rows with one warp shuffle and stores directly.
//
// Split-K across a thread-block cluster: when the output tiles alone cannot fill the GPU, the grid's
// z dimension splits the K loop over the S CTAs of a cluster (1 x 1 x S). Each CTA stores its int32
// partial tile from TMEM into its own shared memory; after a cluster barrier, CTA z reduces every S-th
// 16-token chunk by reading the S partials through distributed shared memory (each rank's 16 loads in
// flight at once, two ranks at a time). When the caller provides a split-K workspace in global memory the
// partials go through L2 instead (stored coalesced, read back with L1-bypassing loads after the cluster
// barrier), which the cluster network's bandwidth makes about twice as fast. The int32 sum is exact, so the
// result is bit-identical to the unsplit loop.
//
// All mbarrier waits are bounded (about one second); on a timeout the kernel records the error in
// g_device_error, drains what it issued (bounded), still takes part in the cluster barriers, frees its
// TMEM and returns.
#include <atomic>
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

namespace tc {
constexpr int kStages = 4;             // shared-memory ring (TMA) = TMEM A ring
constexpr int kBK = 128;               // K per stage: one 128-byte swizzle row of int8
constexpr int kMaxT = 320;             // tokens per CTA
constexpr int kActStageBytes = kMaxT * 128;
constexpr int kWStageBytes = 128 * 32;
constexpr int kThreads = 320;  // warps 0-3 converters+epilogue, 4 TMA, 5 MMA, 6-9 set-up+epilogue
constexpr uint32_t kTmemCols = 512;

// One ring index s serves the shared-memory stage and the TMEM A stage of the same K step:
//   wfull[s]    the packed weight tile of stage s landed (expect_tx; producer arrives once). The weights
//               have their own barrier so that the converters can unpack them before the (larger,
//               later-requested) activation tile of the stage lands;
//   full[s]     the activation tile(s) of stage s landed (expect_tx; producer arrives once)
//   afull[s]    the converters wrote TMEM A stage s (one arrival per converter warp)
//   consumed[s] the MMAs of stage s completed (one tcgen05.commit): frees both the shared-memory
//               stage (producer may refill it) and the TMEM A stage (converters may overwrite it); the
//               converters read stage s's packed weights before arriving on afull[s], i.e. before
//               those MMAs were issued.
struct alignas(8) Bars {
    uint64_t wfull[kStages];
    uint64_t full[kStages];
    uint64_t afull[kStages];
    uint64_t consumed[kStages];
    uint64_t accfull;
    uint64_t drain;
    uint32_t tmem_slot;
    uint32_t abort;
};

constexpr size_t kSmemAct = (size_t)kStages * kActStageBytes;
constexpr size_t kSmemW = (size_t)kStages * kWStageBytes;
constexpr size_t kSmemBytes = 1024 /*align slack*/ + kSmemAct + kSmemW + 3 * kMaxT * sizeof(float) + sizeof(Bars);
static_assert((size_t)128 * kMaxT * 4 <= kSmemAct, "split-K partial tile must fit in the stage ring");
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

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// 16 int32 of CTA `rank`'s shared memory, 512 bytes apart (16 token columns of one row of the
// column-major partial tile), starting where `local_addr` points locally. All 16 loads are issued before
// any result is used; across the warp each load reads 32 consecutive rows = one 128-byte line.
__device__ __forceinline__ void dsmem_ld_col16(uint32_t local_addr, uint32_t rank, int32_t (&v)[16]) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    asm volatile(
        "ld.shared::cluster.b32 %0, [%16];\n\t"
        "ld.shared::cluster.b32 %1, [%16+512];\n\t"
        "ld.shared::cluster.b32 %2, [%16+1024];\n\t"
        "ld.shared::cluster.b32 %3, [%16+1536];\n\t"
        "ld.shared::cluster.b32 %4, [%16+2048];\n\t"
        "ld.shared::cluster.b32 %5, [%16+2560];\n\t"
        "ld.shared::cluster.b32 %6, [%16+3072];\n\t"
        "ld.shared::cluster.b32 %7, [%16+3584];\n\t"
        "ld.shared::cluster.b32 %8, [%16+4096];\n\t"
        "ld.shared::cluster.b32 %9, [%16+4608];\n\t"
        "ld.shared::cluster.b32 %10, [%16+5120];\n\t"
        "ld.shared::cluster.b32 %11, [%16+5632];\n\t"
        "ld.shared::cluster.b32 %12, [%16+6144];\n\t"
        "ld.shared::cluster.b32 %13, [%16+6656];\n\t"
        "ld.shared::cluster.b32 %14, [%16+7168];\n\t"
        "ld.shared::cluster.b32 %15, [%16+7680];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(remote)
        : "memory");
}

// Instruction descriptor, kind::i8: D s32, A unsigned 8-bit (weight codes), B signed 8-bit
// (activations), both K-major, shape 128 x N.
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Epilogue variants are compile-time (EPI bits: kEpiBias, kEpiGelu, kEpiResidual): with the optional steps
// as runtime branches inside the unrolled store loop the epilogue's code no longer fits the instruction
// cache and the store loop runs several times slower.
constexpr int kEpiBias = 1, kEpiGelu = 2, kEpiResidual = 4;

template <int MODE, int EPI>
__global__ void __launch_bounds__(tc::kThreads, 1)
gemm_i2s_tc_kernel(const __grid_constant__ CUtensorMap tmap_w0, const __grid_constant__ CUtensorMap tmap_w1,
                   const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_y,
                   const float* __restrict__ w0_scale, const float* __restrict__ w1_scale,
                   const float* __restrict__ s_act, const int32_t* __restrict__ sum_act, float* y, int64_t ldy,
                   int M, int N, int Kp, int T, int bn_sub, int nsub, const Epilogue epi,
                   int32_t* __restrict__ part_g, int y_tma) {
    using namespace tc;
    constexpr int mode = MODE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* act_sm = base;
    uint8_t* w_sm = base + kSmemAct;
    float* rfac = reinterpret_cast<float*>(w_sm + kSmemW);         // [2][kMaxT]
    int32_t* sumq = reinterpret_cast<int32_t*>(rfac + 2 * kMaxT);  // [kMaxT]
    Bars* bars = reinterpret_cast<Bars*>(sumq + kMaxT);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (int)gridDim.z;
    const int zr = (int)blockIdx.z;
    const int rows_per_w = (mode == 1) ? 64 : 128;          // weight rows of one matrix per CTA
    const int nb = blockIdx.x * rows_per_w;                 // first output column of this CTA
    const int m0 = blockIdx.y * T;
    const int nkt = Kp / kBK;
    const int kt0 = (int)((int64_t)nkt * zr / S), kt1 = (int)((int64_t)nkt * (zr + 1) / S);
    const int nk = kt1 - kt0;
    const int npre = nk < kStages ? nk : kStages;
    const uint32_t acc_stride = (uint32_t)((bn_sub + 31) / 32 * 32);
    const uint32_t a_col0 = acc_stride * (uint32_t)nsub;    // TMEM A ring after the accumulators (<= 320)
    const uint32_t tx = (uint32_t)T * 128u;

    auto load_w = [&](int s, int kt) {
        uint8_t* wst = w_sm + (size_t)s * kWStageBytes;
        mbar_arrive_expect_tx(&bars->wfull[s], (uint32_t)kWStageBytes);
        if (mode == 1) {
            tma_load_2d(wst, &tmap_w0, &bars->wfull[s], kt * 32, nb);
            tma_load_2d(wst + 64 * 32, &tmap_w1, &bars->wfull[s], kt * 32, nb);
        } else {
            tma_load_2d(wst, &tmap_w0, &bars->wfull[s], kt * 32, nb);
        }
    };

    if (threadIdx.x == 128) {  // producer thread: barriers, descriptors, weights of the first ring round
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&bars->wfull[i], 1);
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->afull[i], 4);  // one arrival per converter warp
            mbar_init(&bars->consumed[i], 1);
        }
        mbar_init(&bars->accfull, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_w0);
        if (mode == 1) tma_prefetch_desc(&tmap_w1);
        for (int i = 0; i < npre; ++i) load_w(i, kt0 + i);  // weights do not depend on the preceding kernel
    }
    if (warp == 0) {
        tmem_alloc(&bars->tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_slot;
    volatile uint32_t* abort_flag = &bars->abort;

    if (warp >= 6) {
        // ------------------------------------------------------------------ epilogue group B: set-up
        // Per-token rescale factors w_scale / s[m] (one IEEE division per token and matrix) and the
        // activation sums, computed while the main loop runs.
        griddep_wait();  // scales and sums come from the preceding kernel
        const int nmat = (mode == 1) ? 2 : 1;
        const int tid = threadIdx.x - 192;
        // The staged mode-1 epilogue reads the factors of the even tokens of a 16-token chunk, then the odd
        // ones (the column order of a 16x64b TMEM load), so they are stored in that order.
        const bool perm = (mode == 1) && S == 1 && y_tma;
        auto pos = [&](int t) { return perm ? (t & ~15) + ((t & 1) << 3) + ((t & 15) >> 1) : t; };
        for (int i = tid; i < nmat * T; i += 128) {
            const int j = i / T, t = i - j * T, m = m0 + t;
            const float ws = __ldg(j == 0 ? w0_scale + (epi.scale_rows ? nb / epi.scale_rows : 0) : w1_scale);
            rfac[j * kMaxT + pos(t)] = (m < M) ? __fdiv_rn(ws, s_act[m]) : 0.0f;
        }
        for (int t = tid; t < T; t += 128) sumq[pos(t)] = (m0 + t < M) ? sum_act[m0 + t] : 0;
        int good = 1;
        if (lane == 0) good = mbar_wait(&bars->accfull, 0);
        if (!__shfl_sync(0xffffffffu, good, 0) && lane == 0) *abort_flag = 1;
        __syncwarp();
        tc_fence_after();
    } else if (warp == 4) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            griddep_wait();  // the activation tiles are written by the preceding kernel
            int issued = 0;
            int s = 0;
            uint32_t ph = 0;
            for (int it = 0; it < nk; ++it) {
                const int kt = kt0 + it;
                if (it >= kStages) {  // first-round weights were requested before the setup barrier
                    if (!mbar_wait(&bars->consumed[s], ph ^ 1u) || *abort_flag) { *abort_flag = 1; break; }
                    load_w(s, kt);
                }
                mbar_arrive_expect_tx(&bars->full[s], tx);
                uint8_t* act = act_sm + (size_t)s * kActStageBytes;
                for (int u = 0; u < nsub; ++u)
                    tma_load_2d(act + (size_t)u * bn_sub * 128, &tmap_q, &bars->full[s], kt * kBK, m0 + u * bn_sub);
                ++issued;
                if (++s == kStages) { s = 0; ph ^= 1u; }
            }
            if (*abort_flag) {  // drain copies still in flight before the CTA's shared memory goes away
                for (int it = (issued > kStages ? issued - kStages : 0); it < issued; ++it)
                    mbar_wait(&bars->full[it % kStages], (uint32_t)(it / kStages) & 1u, 2u);
                const int wissued = issued > npre ? issued : npre;  // first-round weights went out at start
                for (int it = (wissued > kStages ? wissued - kStages : 0); it < wissued; ++it)
                    mbar_wait(&bars->wfull[it % kStages], (uint32_t)(it / kStages) & 1u, 2u);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_u8s8(128, bn_sub);
            const uint32_t act_base = smem_u32(act_sm);
            const uint32_t sub_bytes = (uint32_t)bn_sub * 128u;
            bool issued_any = false;
            uint32_t acc_flag = 0;  // first MMA of each accumulator overwrites it
            int s = 0;
            uint32_t ph = 0;
            for (int it = 0; it < nk; ++it) {
                // afull[s]: the unpacked weights of the stage are in TMEM; full[s]: its activation tile
                // landed (the wait also makes those TMA-written bytes visible to this thread's MMAs).
                if (!mbar_wait(&bars->afull[s], ph) || !mbar_wait(&bars->full[s], ph)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t b_base = act_base + (uint32_t)s * kActStageBytes;
                const uint32_t a_base = tmem_base + a_col0 + (uint32_t)s * 32u;
#pragma unroll
                for (int kk = 0; kk < kBK / 32; ++kk) {
                    tc_mma_i8_ts(tmem_base, a_base + kk * 8, umma_desc_k_sw128(b_base + kk * 32), idesc, acc_flag);
                    if (nsub == 2)
                        tc_mma_i8_ts(tmem_base + acc_stride, a_base + kk * 8,
                                     umma_desc_k_sw128(b_base + sub_bytes + kk * 32), idesc, acc_flag);
                    acc_flag = 1;
                }
                issued_any = true;
                tc_commit(&bars->consumed[s]);
                if (++s == kStages) { s = 0; ph ^= 1u; }
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
        // TMEM lane L = threadIdx.x holds weight row r_sm of the stage: in mode 1, lanes 0-15 of each warp
        // take gate rows 16w..16w+15 (stage rows 0-63) and lanes 16-31 the up rows of the same output
        // columns (stage rows 64-127).
        const int r_sm = (mode == 1) ? ((lane < 16) ? (16 * warp + lane) : (64 + 16 * warp + lane - 16))
                                     : (int)threadIdx.x;
        const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
        // Lane 0 waits on the barriers and the warp follows (a timed-out wait is broadcast with
        // __shfl_sync), so control flow stays warp-uniform for the .sync.aligned tcgen05.st.
        bool ok = true;
        int s = 0;
        uint32_t ph = 0;
        for (int it = 0; it < nk; ++it) {
            int good = 1;
            if (lane == 0) good = (*abort_flag == 0) && mbar_wait(&bars->wfull[s], ph);
            if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
            // Every lane acquires the completed phase itself before reading the TMA-written bytes (the
            // phase cannot advance: stage s is refilled only after this warp arrives on afull[s]).
            (void)mbar_try_wait(&bars->wfull[s], ph);
            // 32-byte swizzle: rows 4-7 of every 8 have their 16-byte halves swapped (TMA SWIZZLE_32B)
            const uint8_t* rowp = w_sm + (size_t)s * kWStageBytes + r_sm * 32;
            const int sw = (r_sm >> 2) & 1;
            const uint4 p0 = *reinterpret_cast<const uint4*>(rowp + 16 * sw);
            const uint4 p1 = *reinterpret_cast<const uint4*>(rowp + 16 * (1 - sw));
            if (lane == 0) good = mbar_wait(&bars->consumed[s], ph ^ 1u);  // TMEM A stage s is free
            if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
            const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            uint32_t out[32];
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                out[p] = (w[p] >> 6) & 0x03030303u;       // k = 4p..4p+3
                out[8 + p] = (w[p] >> 4) & 0x03030303u;   // k = 32+4p..
                out[16 + p] = (w[p] >> 2) & 0x03030303u;  // k = 64+4p..
                out[24 + p] = w[p] & 0x03030303u;         // k = 96+4p..
            }
            tmem_st_32x32b_x32(lane_base + a_col0 + (uint32_t)(s * 32), out);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->afull[s]);
            if (++s == kStages) { s = 0; ph ^= 1u; }
        }
        if (!ok && lane == 0) *abort_flag = 1;
        int good = ok ? 1 : 0;
        if (lane == 0 && good) good = mbar_wait(&bars->accfull, 0);
        if (!__shfl_sync(0xffffffffu, good, 0) && lane == 0) *abort_flag = 1;
        __syncwarp();
        tc_fence_after();
    }
    griddep_launch();  // the next kernel may start its prologue while this one writes its outputs

    // ---------------------------------------------------------------------- epilogue
    // Two epilogue groups: warps 0-3 (group 0) and warps 6-9 (group 1). Warp w reads TMEM lane quadrant
    // w % 4, so each quadrant has one warp per group; the groups take alternate token chunk pairs.
    const bool split = S > 1;
    const int nchunk = T / 16;
    const bool is_epi = (warp < 4) || (warp >= 6);
    const int egrp = (warp < 4) ? 0 : 1;
    const int q = warp & 3;                                                  // TMEM lane quadrant
    const int row = 32 * q + lane;                                           // TMEM lane
    int32_t* part = reinterpret_cast<int32_t*>(act_sm);  // [T tokens][128 rows] int32 (column-major)
    // With a global split-K workspace the partial of CTA rank r of this tile lives at part_g + part_off(r)
    // (same [T][128] layout) and is read back through L2 instead of distributed shared memory.
    const size_t tile_lin = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
    auto part_off = [&](int r) -> size_t { return (tile_lin * (size_t)S + (size_t)r) * (size_t)T * 128u; };
    auto chunk_col = [&](int ch) -> uint32_t {           // TMEM column of 16-token chunk ch
        const int t0 = ch * 16, u = t0 / bn_sub;
        return (uint32_t)u * acc_stride + (uint32_t)(t0 - u * bn_sub);
    };
    // Loads the raw accumulators of chunks ch and ch+1 (if hb) for this thread's TMEM lane.
    auto load_pair = [&](int ch, bool hb, bool good, int32_t (&ra)[16], int32_t (&rb)[16]) {
        uint32_t a[16], b[16];
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        if (good) {
            tmem_ld_32x32b_x16(lane_base + chunk_col(ch), a);
            if (hb) tmem_ld_32x32b_x16(lane_base + chunk_col(ch + 1), b);
            tc_wait_ld();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            ra[j] = good ? (int32_t)a[j] : 0;
            rb[j] = (good && hb) ? (int32_t)b[j] : 0;
        }
    };

    if (split) {
        __syncthreads();  // every role has left the main loop: the rings are free; rfac/sumq are ready
        if (is_epi) {
            const bool good = __all_sync(0xffffffffu, *abort_flag == 0);
            for (int ch = 2 * egrp; ch < nchunk; ch += 4) {
                int32_t ra[16], rb[16];
                const bool hb = ch + 1 < nchunk;
                load_pair(ch, hb, good, ra, rb);
                int32_t* dst = (part_g ? part_g + part_off(zr) : part) + (ch * 16) * 128 + row;
#pragma unroll
                for (int j = 0; j < 16; ++j) dst[j * 128] = ra[j];
                if (hb) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) dst[(16 + j) * 128] = rb[j];
                }
            }
        }
        if (part_g) __threadfence();  // the partials in global memory are visible before the barrier
        cluster_sync_all();
    } else if (is_epi) {
        named_bar_sync(2, 256);  // group 1's rfac/sumq are visible to group 0
    }

    if constexpr (MODE == 1) {
        if (!split && y_tma && is_epi) {
            // Staged FFN epilogue. Per 16-token chunk, each warp loads its quadrant's 16 gate lanes and the
            // 16 up lanes of the same output columns with two 16x64b loads, so thread i holds gate and up of
            // output column 16q + (i >> 2) + 8 (i & 1) for the tokens (i >> 1) & 1 + 2j, j = 0..7: the
            // product needs no shuffle. Results go to shared memory as a [T][64] fp32 tile (the drained
            // stage ring); once the group's four warps have written a chunk pair, one thread stores it with
            // TMA (box 64 x 16), which also drops the rows past M.
            const bool good = __all_sync(0xffffffffu, *abort_flag == 0);
            const int col = 16 * q + (lane >> 2) + 8 * (lane & 1);  // output column within the CTA's 64
            const int par = (lane >> 1) & 1;                           // token parity within the chunk
            float* stage = reinterpret_cast<float*>(act_sm);           // [T][64] fp32
            const uint32_t lane_g = tmem_base + ((uint32_t)(q * 32) << 16);
            const uint32_t lane_u = tmem_base + ((uint32_t)(q * 32 + 16) << 16);
            const bool issuer = (q == 0) && lane == 0;
            auto finish16 = [&](int ch, const uint32_t (&g)[8], const uint32_t (&u)[8]) {
                const int t0 = ch * 16, f = t0 + 8 * par;
                const int4 sq0 = *reinterpret_cast<const int4*>(sumq + f);
                const int4 sq1 = *reinterpret_cast<const int4*>(sumq + f + 4);
                const float4 rg0 = *reinterpret_cast<const float4*>(rfac + f);
                const float4 rg1 = *reinterpret_cast<const float4*>(rfac + f + 4);
                const float4 ru0 = *reinterpret_cast<const float4*>(rfac + kMaxT + f);
                const float4 ru1 = *reinterpret_cast<const float4*>(rfac + kMaxT + f + 4);
                const int sq[8] = {sq0.x, sq0.y, sq0.z, sq0.w, sq1.x, sq1.y, sq1.z, sq1.w};
                const float rg[8] = {rg0.x, rg0.y, rg0.z, rg0.w, rg1.x, rg1.y, rg1.z, rg1.w};
                const float ru[8] = {ru0.x, ru0.y, ru0.z, ru0.w, ru1.x, ru1.y, ru1.z, ru1.w};
                float* dst = stage + (t0 + par) * 64 + col;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float gv = __fmul_rn((float)((int32_t)g[j] - sq[j]), rg[j]);
                    const float uv = __fmul_rn((float)((int32_t)u[j] - sq[j]), ru[j]);
                    const float rgv = gv > 0.0f ? gv : 0.0f;
                    dst[j * 128] = __fmul_rn(__fmul_rn(rgv, rgv), uv);
                }
            };
            for (int ch = 2 * egrp; ch < nchunk; ch += 4) {
                const bool hb = ch + 1 < nchunk;
                uint32_t g0[8], u0[8], g1[8], u1[8];
                if (good) {
                    tmem_ld_16x64b_x8(lane_g + chunk_col(ch), g0);
                    tmem_ld_16x64b_x8(lane_u + chunk_col(ch), u0);
                    if (hb) {
                        tmem_ld_16x64b_x8(lane_g + chunk_col(ch + 1), g1);
                        tmem_ld_16x64b_x8(lane_u + chunk_col(ch + 1), u1);
                    }
                    tc_wait_ld();
                    finish16(ch, g0, u0);
                    if (hb) finish16(ch + 1, g1, u1);
                }
                fence_proxy_async_smem();
                named_bar_sync(3 + egrp, 128);  // the group's four quadrants of the chunk pair are staged
                if (issuer && good) {
                    tma_store_2d(&tmap_y, stage + ch * 16 * 64, nb, m0 + ch * 16);
                    if (hb) tma_store_2d(&tmap_y, stage + (ch + 1) * 16 * 64, nb, m0 + ch * 16 + 16);
                    bulk_commit();
                }
            }
            if (issuer) bulk_wait_all();  // the staged tile is read and written before the CTA exits
        }
    }
    if (is_epi && !(MODE == 1 && !split && y_tma)) {
        const bool good = __all_sync(0xffffffffu, *abort_flag == 0);
        const int gu = (mode == 1) ? (lane >> 4) : 0;                     // 0 gate / 1 up lane (mode 1)
        const int n = (mode == 1) ? nb + 16 * q + (lane & 15) : nb + row;  // output column

        // Mode 0: the bias of this thread's output column is loaded once; residual values are fetched
        // for a whole chunk pair before the pair's accumulators are read (load_res), so their latency
        // is paid once per pair and overlaps the TMEM loads, not once per output.
        const float bias_n = ((EPI & kEpiBias) && n < N) ? epi.bias[n] : 0.0f;
        auto load_res = [&](int ch, float (&r)[16]) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = m0 + ch * 16 + j;
                r[j] = ((EPI & kEpiResidual) && ch < nchunk && m < M && n < N)
                           ? epi.residual[(int64_t)m * epi.ld_res + n]
                           : 0.0f;
            }
        };
        auto finish = [&](int ch, const int32_t (&raw)[16], const float (&res)[16]) {
            const int t0 = ch * 16;
            if (mode == 0) {
                // all 16 values first (independent chains that interleave), then the guarded stores
                float val[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + j;
                    float v = __fmul_rn((float)(raw[j] - sumq[t]), rfac[t]);
                    if (EPI & kEpiBias) v = __fadd_rn(v, bias_n);
                    if (EPI & kEpiGelu) v = gelu_tanh(v);
                    if (EPI & kEpiResidual) v = __fadd_rn(res[j], v);
                    val[j] = v;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + t0 + j;
                    if (good && m < M && n < N) y[(int64_t)m * ldy + n] = val[j];
                }
            } else {
                float p[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + j;
                    const float v = __fmul_rn((float)(raw[j] - sumq[t]), rfac[gu * kMaxT + t]);
                    const float o = __shfl_xor_sync(0xffffffffu, v, 16);
                    const float g = gu ? o : v, u = gu ? v : o;
                    const float rg = g > 0.0f ? g : 0.0f;
                    p[j] = __fmul_rn(__fmul_rn(rg, rg), u);
                }
                // gate lanes store tokens 0-7 of the chunk, up lanes tokens 8-15 (same 16 columns)
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const float v = gu ? p[8 + jj] : p[jj];
                    const int m = m0 + t0 + gu * 8 + jj;
                    if (good && m < M && n < N) y[(int64_t)m * ldy + n] = v;
                }
            }
        };

        if (split) {
            const int rank = (int)cluster_ctarank();
            int i = 0;
            for (int ch = rank; ch < nchunk; ch += S, ++i) {
                if ((i & 1) != egrp) continue;
                int32_t raw[16];
                float res[16];
                load_res(ch, res);
#pragma unroll
                for (int j = 0; j < 16; ++j) raw[j] = 0;
                if (part_g) {
                    for (int r0 = 0; r0 < S; r0 += 4) {  // four ranks' loads in flight (L2, bypassing L1)
                        int32_t pv[4][16];
#pragma unroll
                        for (int r = 0; r < 4; ++r)
                            if (good && r0 + r < S) {
                                const int32_t* src = part_g + part_off(r0 + r) + (ch * 16) * 128 + row;
#pragma unroll
                                for (int j = 0; j < 16; ++j) pv[r][j] = __ldcg(src + j * 128);
                            }
#pragma unroll
                        for (int r = 0; r < 4; ++r)
                            if (good && r0 + r < S) {
#pragma unroll
                                for (int j = 0; j < 16; ++j) raw[j] += pv[r][j];
                            }
                    }
                } else {
                    const uint32_t addr = smem_u32(part + (ch * 16) * 128 + row);
                    for (int r = 0; r < S; r += 2) {
                        int32_t a[16], b[16];
                        if (good) dsmem_ld_col16(addr, (uint32_t)r, a);
                        if (good && r + 1 < S) dsmem_ld_col16(addr, (uint32_t)(r + 1), b);
#pragma unroll
                        for (int j = 0; j < 16; ++j) raw[j] += (good ? a[j] : 0) + ((good && r + 1 < S) ? b[j] : 0);
                    }
                }
                finish(ch, raw, res);
            }
        } else {
            for (int ch = 2 * egrp; ch < nchunk; ch += 4) {
                int32_t ra[16], rb[16];
                float sa[16], sb[16];
                const bool hb = ch + 1 < nchunk;
                load_res(ch, sa);
                load_res(ch + 1, sb);
                load_pair(ch, hb, good, ra, rb);
                finish(ch, ra, sa);
                if (hb) finish(ch + 1, rb, sb);
            }
        }
    }

    if (split) cluster_sync_all();  // partials stay readable until every CTA of the cluster is done
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <int MODE, int EPI>
static cudaError_t launch_variant(const TcGemmArgs& a, cudaStream_t st) {
    auto kfn = gemm_i2s_tc_kernel<MODE, EPI>;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), tc::kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.n_tiles, (unsigned)a.m_tiles, (unsigned)a.splits);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)a.splits;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kfn, a.tmap_w0, a.tmap_w1, a.tmap_q, a.tmap_y, a.w0_scale, a.w1_scale, a.s,
                              a.sums, a.y, a.ldy, a.M, a.N, a.Kp, a.T, a.bn_sub, a.nsub, a.epi, a.part,
                              (MODE == 1 && a.y_tma) ? 1 : 0);
}

// Clusters of `size` CTAs of this kernel that can be resident at once on the current device (a cluster
// must fit inside one GPC, so e.g. 7-CTA clusters leave SMs of every GPC idle). Cached per device/size.
int tc_max_active_clusters(int size) {
    static std::atomic<int> cache[64][9];
    int dev = 0;
    if (size < 1 || size > 8 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev][size]) return cache[dev][size];
    auto kfn = gemm_i2s_tc_kernel<0, 0>;
    if (ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), tc::kSmemBytes) != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)size);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)size;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    cache[dev][size] = n > 0 ? n : -1;
    return cache[dev][size];
}

cudaError_t launch_gemm_i2s_tc(const TcGemmArgs& a, cudaStream_t st) {
    if (a.mode == 1) return launch_variant<1, 0>(a, st);
    const int epi = (a.epi.bias ? kEpiBias : 0) | (a.epi.act == 1 ? kEpiGelu : 0) |
                    (a.epi.residual ? kEpiResidual : 0);
    switch (epi) {
        case 0: return launch_variant<0, 0>(a, st);
        case kEpiBias: return launch_variant<0, kEpiBias>(a, st);
        case kEpiBias | kEpiGelu: return launch_variant<0, kEpiBias | kEpiGelu>(a, st);
        case kEpiGelu: return launch_variant<0, kEpiGelu>(a, st);
        case kEpiResidual: return launch_variant<0, kEpiResidual>(a, st);
        case kEpiBias | kEpiResidual: return launch_variant<0, kEpiBias | kEpiResidual>(a, st);
        case kEpiGelu | kEpiResidual: return launch_variant<0, kEpiGelu | kEpiResidual>(a, st);
        default: return launch_variant<0, kEpiBias | kEpiGelu | kEpiResidual>(a, st);
    }
}

}  // namespace b2s
