// gemm_i2s_tcp.cu -- persistent i2_s x int8 GEMM on the sm_100a tensor cores (tcgen05 kind::i8), for
// outputs with at least one tile per SM.
//
// One CTA per SM walks the output tiles (128 weight rows x T tokens, T <= 192; in the gate/up mode 64 gate
// and 64 up rows) in the order blockIdx.x, blockIdx.x + gridDim.x, ... Work moves between the roles in
// stages of two 128-wide K steps: a stage's barrier waits, arrivals, fences and commits cost about as much
// as a step's MMAs at these tile sizes (time per tile, measured over token tiles of 64..192, is ~3/4 a
// fixed per-handoff cost), so each handoff carries twice the work. Per stage:
//   * warp 4 (producer) TMA-loads, for each of its two K steps, the packed weight tile (128 rows x 32 bytes,
//     local HBM, no multicast) and the int8 activation tile (T rows x 128 bytes, 128B swizzle) into a
//     4-stage shared-memory ring; past Kp (an odd step count) the boxes read zeros, which add nothing;
//   * warps 0-3 (converters, one per TMEM lane quadrant) turn each row's 2 x 32 packed bytes into 2 x 128
//     unsigned 2-bit codes {0,1,2} and store them with tcgen05.st into a 2-stage TMEM ring (the MMA's A
//     operand), one store wait and one arrival per stage;
//   * warp 5 (MMA) issues eight tcgen05.mma.kind::i8 (M=128, N=T, K=32): A = codes from TMEM, B = signed
//     int8 activations from shared memory (descriptors derived from one precomputed ring descriptor),
//     int32 accumulators in one of two TMEM buffers;
//   * warps 6.. (epilogue, two per quadrant, three for the plain and +bias forms at K <= 2560) read the
//     finished buffer (tcgen05.ld) and write
//     y = (float)(acc - sum_q[m]) * (w_scale / s[m]) (+ bias, GELU, + residual), while the MMAs of the
//     next tile already fill the other buffer. The output writes of one tile therefore overlap the
//     main loop of the next instead of stalling every SM at the end of a wave.
// TMEM: columns [0,128) A ring, [128,320) and [320,512) accumulators. Every mbarrier wait is bounded (about
// one second); on a timeout the kernel records the error in g_device_error, stops issuing, drains what it
// issued (bounded), frees its TMEM and returns. The int32 accumulation is exact and the fp32 epilogue is
// the same operation sequence as gemm_i2s_tc.cu, so both kernels give bit-identical outputs.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

namespace tcp {
constexpr int kKS = 2;       // 128-wide K steps per stage and per handoff between the roles
constexpr int kStages = 4;   // shared-memory ring (stages of kKS K steps)
constexpr int kAStages = 2;  // TMEM ring of converted codes (stages of kKS x 32 columns)
constexpr int kMaxT = 192;
constexpr int kActSubBytes = kMaxT * 128;             // one K step's activation tile (24 KB, SW128 atoms)
constexpr int kActStageBytes = kKS * kActSubBytes;
constexpr int kWSubBytes = 128 * 32;                  // one K step's packed weight tile
constexpr int kWStageBytes = kKS * kWSubBytes;
// warps 0-3 converters, 4 TMA producer, 5 MMA, 6.. epilogue (G per TMEM quadrant, see tcp_threads)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol0 = kAStages * kKS * 32;  // accumulator buffer b at kAccCol0 + b * kMaxT
static_assert(kAccCol0 + 2 * kMaxT <= kTmemCols, "TMEM budget");

struct alignas(8) Bars {
    uint64_t full[kStages];     // TMA bytes of smem stage landed
    uint64_t sfree[kStages];    // MMAs reading smem stage done (commit)
    uint64_t afull[kAStages];   // converters wrote TMEM A stage (4 arrivals)
    uint64_t afree[kAStages];   // MMAs reading TMEM A stage done (commit)
    uint64_t accfull[2];        // accumulator buffer complete (commit)
    uint64_t accfree[2];        // epilogue drained accumulator buffer (one arrival per epilogue warp)
    uint64_t drain;
    uint32_t tmem_slot;
    uint32_t abort;
};
constexpr size_t kSmemBytes = 1024 + (size_t)kStages * (kActStageBytes + kWStageBytes) + sizeof(Bars);
static_assert(kSmemBytes <= 227 * 1024, "dynamic shared memory per CTA");
}  // namespace tcp

// Instruction descriptor, kind::i8: D s32, A unsigned 8-bit (codes), B signed 8-bit, K-major, 128 x N.
__host__ __device__ constexpr uint32_t idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

constexpr int kPEpiBias = 1, kPEpiGelu = 2, kPEpiResidual = 4;

// Epilogue warps per TMEM lane quadrant (template parameter G). A tile's epilogue runs latency-bound at
// two warps per scheduler; where the K loop is short (K <= 2560: 1152 has five stages per tile) that
// took longer than the next tile's K loop, so the plain and +bias forms there take three warps per
// quadrant (2048 x 1152 -> 4304: 25.6 -> 21.2 µs; 16384 x 1152 -> 4304: 0.35 -> 0.45 of the int8 peak).
// At K = 6912, where the epilogue hides behind a long K loop, three measured no better (16384 x 6912 ->
// 2560: 238 µs against 226-235 µs with two in other runs), so long K keeps two, as do the residual forms
// (128 registers) and the gate/up form.
__host__ __device__ constexpr int tcp_threads(int groups) { return 32 * (6 + 4 * groups); }

template <int MODE, int EPI, int G>
__global__ void __launch_bounds__(tcp_threads(G), 1)
gemm_i2s_tcp_kernel(const __grid_constant__ CUtensorMap tmap_w0, const __grid_constant__ CUtensorMap tmap_w1,
                    const __grid_constant__ CUtensorMap tmap_q, const float* __restrict__ w0_scale,
                    const float* __restrict__ w1_scale, const float* __restrict__ s_act,
                    const int32_t* __restrict__ sum_act, float* y, int64_t ldy, int M, int N, int Kp, int T,
                    int n_tiles, int m_tiles, const Epilogue epi) {
    using namespace tcp;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* act_sm = base;                                       // kStages x kActStageBytes
    uint8_t* w_sm = base + (size_t)kStages * kActStageBytes;      // kStages x kWStageBytes
    Bars* bars = reinterpret_cast<Bars*>(w_sm + (size_t)kStages * kWStageBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int rows_per_w = (MODE == 1) ? 64 : 128;
    const int nkt = Kp / 128;
    const int nks = (nkt + kKS - 1) / kKS;  // stages per tile (past Kp the boxes read zeros, which add 0)
    const int total = n_tiles * m_tiles;
    const uint32_t tx = (uint32_t)kKS * ((uint32_t)T * 128u + (uint32_t)kWSubBytes);

    if (threadIdx.x == 128) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->sfree[i], 1);
        }
        for (int i = 0; i < kAStages; ++i) {
            mbar_init(&bars->afull[i], 4);
            mbar_init(&bars->afree[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->accfull[i], 1);
            mbar_init(&bars->accfree[i], 4 * G);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_w0);
        if (MODE == 1) tma_prefetch_desc(&tmap_w1);
    }
    if (warp == 4) {
        tmem_alloc(&bars->tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_slot;
    volatile uint32_t* abort_flag = &bars->abort;

    if (warp == 4) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            griddep_wait();  // activations, scales and sums come from the preceding kernel
            uint32_t g = 0;
            bool stop = false;
            for (int t = blockIdx.x; t < total && !stop; t += gridDim.x) {
                const int nb = (t % n_tiles) * rows_per_w, m0 = (t / n_tiles) * T;
                for (int ks = 0; ks < nks; ++ks, ++g) {
                    const uint32_t s = g % kStages, u = g / kStages;
                    if (u > 0 && (!mbar_wait(&bars->sfree[s], (u - 1) & 1u) || *abort_flag)) {
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&bars->full[s], tx);
#pragma unroll
                    for (int j = 0; j < kKS; ++j) {
                        const int kt = kKS * ks + j;
                        uint8_t* wst = w_sm + (size_t)s * kWStageBytes + (size_t)j * kWSubBytes;
                        tma_load_2d(wst, &tmap_w0, &bars->full[s], kt * 32, nb);
                        if (MODE == 1) tma_load_2d(wst + 64 * 32, &tmap_w1, &bars->full[s], kt * 32, nb);
                        tma_load_2d(act_sm + (size_t)s * kActStageBytes + (size_t)j * kActSubBytes, &tmap_q,
                                    &bars->full[s], kt * 128, m0);
                    }
                }
            }
            // Copies still in flight must land before the CTA's shared memory goes away: wait for the
            // last use of every stage that was armed.
            for (uint32_t k = (g > kStages ? g - kStages : 0); k < g; ++k)
                mbar_wait(&bars->full[k % kStages], (k / kStages) & 1u, 2u);
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_u8s8(128, T);
            // B descriptors: the ring's first one, computed once; stage s and K slice kk add their byte offset
            // / 16 to the start-address field (exact: shared addresses stay below 2^18 bytes).
            const uint64_t desc0 = umma_desc_k_sw128(smem_u32(act_sm));
            uint32_t g = 0, i = 0;
            bool issued_any = false, stop = false;
            for (int t = blockIdx.x; t < total && !stop; t += gridDim.x, ++i) {
                const uint32_t b = i & 1u, v = i >> 1;
                if (v > 0 && !mbar_wait(&bars->accfree[b], (v - 1) & 1u)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + kAccCol0 + b * (uint32_t)kMaxT;
                for (int ks = 0; ks < nks; ++ks, ++g) {
                    const uint32_t s = g % kStages, a = g % kAStages;
                    if (!mbar_wait(&bars->afull[a], (g / kAStages) & 1u) ||
                        !mbar_wait(&bars->full[s], (g / kStages) & 1u) || *abort_flag) {
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int j = 0; j < kKS; ++j) {
                        const uint64_t bd =
                            desc0 + (uint64_t)((s * (uint32_t)kActStageBytes + j * (uint32_t)kActSubBytes) >> 4);
                        const uint32_t a_base = tmem_base + a * (uint32_t)(kKS * 32) + j * 32u;
                        tc_mma_i8_ts(d_tmem, a_base, bd, idesc, (ks > 0 || j > 0) ? 1u : 0u);
                        tc_mma_i8_ts_acc(d_tmem, a_base + 8, bd + 2, idesc);
                        tc_mma_i8_ts_acc(d_tmem, a_base + 16, bd + 4, idesc);
                        tc_mma_i8_ts_acc(d_tmem, a_base + 24, bd + 6, idesc);
                    }
                    issued_any = true;
                    tc_commit(&bars->sfree[s]);
                    tc_commit(&bars->afree[a]);
                }
                if (stop) break;
                tc_commit(&bars->accfull[b]);
            }
            if (*abort_flag && issued_any) {  // let issued MMAs finish before TMEM is released
                tc_commit(&bars->drain);
                mbar_wait(&bars->drain, 0, 2u);
            }
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------------ converters
        // TMEM lane L = 32 warp + lane holds stage row r_sm: in the gate/up mode lanes 0-15 of each
        // warp take gate rows 16w..16w+15 (stage rows 0-63) and lanes 16-31 the up rows of the same
        // output columns (stage rows 64-127).
        const int q = warp;
        const int r_sm = (MODE == 1) ? ((lane < 16) ? (16 * q + lane) : (64 + 16 * q + lane - 16)) : (32 * q + lane);
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        uint32_t g = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
            for (int ks = 0; ks < nks; ++ks, ++g) {
                const uint32_t s = g % kStages, a = g % kAStages, ua = g / kAStages;
                int good = 1;
                if (lane == 0) good = (*abort_flag == 0) && mbar_wait(&bars->full[s], (g / kStages) & 1u);
                if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
                (void)mbar_try_wait(&bars->full[s], (g / kStages) & 1u);  // each lane acquires the phase
                // 32-byte swizzle: rows 4-7 of every 8 have their 16-byte halves swapped (TMA SWIZZLE_32B)
                const int sw = (r_sm >> 2) & 1;
                uint4 p0[kKS], p1[kKS];
#pragma unroll
                for (int j = 0; j < kKS; ++j) {
                    const uint8_t* rowp = w_sm + (size_t)s * kWStageBytes + (size_t)j * kWSubBytes + r_sm * 32;
                    p0[j] = *reinterpret_cast<const uint4*>(rowp + 16 * sw);
                    p1[j] = *reinterpret_cast<const uint4*>(rowp + 16 * (1 - sw));
                }
                if (lane == 0 && ua > 0) good = mbar_wait(&bars->afree[a], (ua - 1) & 1u);
                if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
#pragma unroll
                for (int j = 0; j < kKS; ++j) {
                    const uint32_t w[8] = {p0[j].x, p0[j].y, p0[j].z, p0[j].w, p1[j].x, p1[j].y, p1[j].z, p1[j].w};
                    uint32_t out[32];
#pragma unroll
                    for (int p = 0; p < 8; ++p) {
                        out[p] = (w[p] >> 6) & 0x03030303u;
                        out[8 + p] = (w[p] >> 4) & 0x03030303u;
                        out[16 + p] = (w[p] >> 2) & 0x03030303u;
                        out[24 + p] = w[p] & 0x03030303u;
                    }
                    tmem_st_32x32b_x32(lane_base + a * (uint32_t)(kKS * 32) + j * 32u, out);
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->afull[a]);
            }
        }
        if (!ok && lane == 0) *abort_flag = 1;
    } else {
        // ------------------------------------------------------------------ epilogue (warps 6..)
        // The G warps of a quadrant take every G-th 16-token chunk pair. Before a tile's accumulators
        // are waited for, each lane fetches the scales (w_scale / s[m], one IEEE division) and code sums of
        // the tokens its warp will write, so no global-memory latency sits between accumulator and store.
        const int q = warp & 3;             // TMEM lane quadrant
        const int grp = (warp - 6) >> 2;  // 0 .. G-1 (G epilogue warps per quadrant)
        const int row = 32 * q + lane;
        const int gu = (MODE == 1) ? (lane >> 4) : 0;
        const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
        const int nchunk = T / 16;
        constexpr int kPairs = (kMaxT / 16 + 2 * G - 1) / (2 * G);  // chunk pairs per warp
        griddep_wait();  // scales, sums and residual come from the preceding kernels
        uint32_t i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
            const uint32_t b = i & 1u, v = i >> 1;
            const int nt = t % n_tiles, m0 = (t / n_tiles) * T;
            const int nb = nt * rows_per_w;
            const int n = (MODE == 1) ? nb + 16 * q + (lane & 15) : nb + row;
            const float ws0 = __ldg(w0_scale + ((MODE == 0 && epi.scale_rows) ? nb / epi.scale_rows : 0));
            const float ws1 = (MODE == 1) ? __ldg(w1_scale) : ws0;
            const float wsl = (MODE == 1 && lane >= 16) ? ws1 : ws0;
            const float bias_n = ((EPI & kPEpiBias) && n < N) ? epi.bias[n] : 0.0f;
            // chunk pair p of this warp: chunks 2 (G p + grp) and 2 (G p + grp) + 1; lane l holds token l & 15
            float rf[2 * kPairs];
            int sm[2 * kPairs];
#pragma unroll
            for (int c = 0; c < 2 * kPairs; ++c) {
                const int ch = 2 * (G * (c >> 1) + grp) + (c & 1);
                const int mj = m0 + 16 * ch + (lane & 15);
                const bool ok = ch < nchunk && mj < M;
                sm[c] = ok ? sum_act[mj] : 0;
                rf[c] = ok ? __fdiv_rn(wsl, s_act[mj]) : 0.0f;
            }
            auto load_res = [&](int ch, float (&r)[16]) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + 16 * ch + j;
                    r[j] = ((EPI & kPEpiResidual) && ch < nchunk && m < M && n < N)
                               ? epi.residual[(int64_t)m * epi.ld_res + n]
                               : 0.0f;
                }
            };
            // residual rows run one chunk ahead of the stores: the first chunk's are fetched before the wait
            float resa[16], resb[16];
            load_res(2 * grp, resa);
            int good = 1;
            if (lane == 0) good = (*abort_flag == 0) && mbar_wait(&bars->accfull[b], v & 1u);
            if (!__shfl_sync(0xffffffffu, good, 0)) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t acc = lane_base + kAccCol0 + b * (uint32_t)kMaxT;
            auto finish = [&](int ch, const uint32_t (&raw)[16], float rfc, int smc, const float (&res)[16]) {
                const int t0 = 16 * ch;
                if (MODE == 0) {
                    // all 16 values first (independent chains that interleave), then the guarded stores
                    float val[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float rfj = __shfl_sync(0xffffffffu, rfc, j);
                        const int smj = __shfl_sync(0xffffffffu, smc, j);
                        float v = __fmul_rn((float)((int32_t)raw[j] - smj), rfj);
                        if (EPI & kPEpiBias) v = __fadd_rn(v, bias_n);
                        if (EPI & kPEpiGelu) v = gelu_tanh(v);
                        if (EPI & kPEpiResidual) v = __fadd_rn(res[j], v);
                        val[j] = v;
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int m = m0 + t0 + j;
                        if (m < M && n < N) y[(int64_t)m * ldy + n] = val[j];
                    }
                } else {
                    float p[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float rfj = __shfl_sync(0xffffffffu, rfc, gu * 16 + j);
                        const int smj = __shfl_sync(0xffffffffu, smc, j);
                        const float val = __fmul_rn((float)((int32_t)raw[j] - smj), rfj);
                        const float o = __shfl_xor_sync(0xffffffffu, val, 16);
                        const float gv = gu ? o : val, uv = gu ? val : o;
                        const float rg = gv > 0.0f ? gv : 0.0f;
                        p[j] = __fmul_rn(__fmul_rn(rg, rg), uv);
                    }
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const float val = gu ? p[8 + jj] : p[jj];
                        const int m = m0 + t0 + gu * 8 + jj;
                        if (m < M && n < N) y[(int64_t)m * ldy + n] = val;
                    }
                }
            };
#pragma unroll
            for (int pp = 0; pp < kPairs; ++pp) {
                const int ch = 2 * (G * pp + grp);
                if (ch >= nchunk) break;
                const bool hb = ch + 1 < nchunk;
                uint32_t xa[16], xb[16];
                tmem_ld_x16(acc + (uint32_t)(16 * ch), xa);
                if (hb) tmem_ld_x16(acc + (uint32_t)(16 * ch + 16), xb);
                tc_wait_ld();
                if (hb) load_res(ch + 1, resb);
                finish(ch, xa, rf[2 * pp], sm[2 * pp], resa);
                if (ch + 2 * G < nchunk) load_res(ch + 2 * G, resa);
                if (hb) finish(ch + 1, xb, rf[2 * pp + 1], sm[2 * pp + 1], resb);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->accfree[b]);
        }
    }

    griddep_launch();
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

template <int MODE, int EPI, int G>
static cudaError_t launch_tcp_groups(const TcGemmArgs& a, int grid, cudaStream_t st) {
    auto kfn = gemm_i2s_tcp_kernel<MODE, EPI, G>;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), tcp::kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(tcp_threads(G));
    cfg.dynamicSmemBytes = tcp::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, a.tmap_w0, a.tmap_w1, a.tmap_q, a.w0_scale, a.w1_scale, a.s, a.sums, a.y,
                              a.ldy, a.M, a.N, a.Kp, a.T, a.n_tiles, a.m_tiles, a.epi);
}

template <int MODE, int EPI>
static cudaError_t launch_tcp_variant(const TcGemmArgs& a, int grid, cudaStream_t st) {
    if constexpr (MODE == 0 && !(EPI & kPEpiResidual)) {
        if (a.Kp <= 2560) return launch_tcp_groups<MODE, EPI, 3>(a, grid, st);
    }
    return launch_tcp_groups<MODE, EPI, 2>(a, grid, st);
}

int tcp_max_tokens() { return tcp::kMaxT; }

cudaError_t launch_gemm_i2s_tcp(const TcGemmArgs& a, int grid, cudaStream_t st) {
    if (a.T <= 0 || a.T > tcp::kMaxT || a.T % 16 != 0) return cudaErrorInvalidValue;
    if (a.mode == 1) return launch_tcp_variant<1, 0>(a, grid, st);
    const int epi = (a.epi.bias ? kPEpiBias : 0) | (a.epi.act == 1 ? kPEpiGelu : 0) |
                    (a.epi.residual ? kPEpiResidual : 0);
    switch (epi) {
        case 0: return launch_tcp_variant<0, 0>(a, grid, st);
        case kPEpiBias: return launch_tcp_variant<0, kPEpiBias>(a, grid, st);
        case kPEpiBias | kPEpiGelu: return launch_tcp_variant<0, kPEpiBias | kPEpiGelu>(a, grid, st);
        case kPEpiGelu: return launch_tcp_variant<0, kPEpiGelu>(a, grid, st);
        case kPEpiResidual: return launch_tcp_variant<0, kPEpiResidual>(a, grid, st);
        case kPEpiBias | kPEpiResidual: return launch_tcp_variant<0, kPEpiBias | kPEpiResidual>(a, grid, st);
        case kPEpiGelu | kPEpiResidual: return launch_tcp_variant<0, kPEpiGelu | kPEpiResidual>(a, grid, st);
        default: return launch_tcp_variant<0, kPEpiBias | kPEpiGelu | kPEpiResidual>(a, grid, st);
    }
}

}  // namespace b2s
