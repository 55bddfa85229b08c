// gemv_i2s.cu -- decode-size (M <= 16) i2_s x int8 GEMV: dp4a for one token, warp int8 MMAs for 2..16.
//
// Streams the packed 2-bit weights once from HBM with 128-bit loads and decodes them in registers:
// a 16-byte half of a 32-byte i2_s block holds, for each of its 4 bit-planes g, 16 consecutive
// weights k = 128b + 32g + 16h + [0,16); (word >> (6-2g)) & 0x03030303 yields four unsigned codes
// {0,1,2} ready for dp4a.u32.s32 against four int8 activations. The code offset is removed once per
// output with the per-token activation sum: sum_k (t_k+1) q_k - sum_k q_k = sum_k t_k q_k
// (the method of ggml_vec_dot_i2_i8_s in the BitNet fork).
//
// Mapping: a CTA owns 16 weight rows; in each warp, lane pair (2r, 2r+1) reads row r, one 32-byte
// block per step (16 rows x 32 B = 16 full sectors per load instruction). The CTA's warps split the
// row's blocks into contiguous ranges and reduce through shared memory. The int8 activations of all
// M tokens sit in shared memory and are read as broadcasts (every row of the warp reads the same
// 32 bytes per bit-plane).
//
// Launches with many rows (batched decode problems, ggml ne[2]) use streaming forms instead: for one
// token a TMA-fed kernel (per-warp shared-memory rings of 64-row x 128-byte stages, one persistent wave)
// or, where its requirements do not hold, a register-ring kernel; for 2..16 tokens a register-ring MMA
// kernel. A bit-plane may also be masked in place (byte & (3 << (6-2g))): its dot product then comes
// out scaled by 4^(3-g), exactly, and is shifted back once per row.
//
// Weight loads for the first range are issued before griddepcontrol.wait, so when launched with
// programmatic stream serialization the weight stream overlaps the tail of the kernel that produces
// the activations.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

constexpr int kGemvRows = 16;   // rows per CTA
constexpr int kGemvWarps = 8;   // warps per CTA (split K)
constexpr int kGemvUnroll = 8;  // 16-byte loads in flight per lane
constexpr int kS1R = 4, kS1D = 2;  // one-token streaming kernel: rows per lane, register ring depth

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
// 16-byte asynchronous global -> shared copy; bytes past src_bytes (0..16) are zero-filled.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int MT>
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_i2s_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ wscale, int N, int Kp,
                const int8_t* __restrict__ q, int64_t ldq, int K, int mrows, const float* __restrict__ s,
                const int32_t* __restrict__ sums, float* y, int64_t ldy, const Epilogue epi, const GemvBatch bt) {
    extern __shared__ __align__(16) uint8_t q_sm[];  // MT x Kp int8, zero beyond K and beyond mrows
    __shared__ int red[kGemvWarps][kGemvRows][MT];
    codes += (int64_t)blockIdx.y * bt.w_stride;  // problem blockIdx.y of a batched launch
    q += (int64_t)blockIdx.y * bt.q_stride;
    s += (int64_t)blockIdx.y * bt.a_stride;
    sums += (int64_t)blockIdx.y * bt.a_stride;
    y += (int64_t)blockIdx.y * bt.y_stride;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 1, h = lane & 1;
    const int row = blockIdx.x * kGemvRows + r;
    const bool row_ok = row < N;
    const int nblk = Kp / kQK;
    const int per = (nblk + kGemvWarps - 1) / kGemvWarps;
    const int b0 = min(nblk, warp * per), b1 = min(nblk, b0 + per);
    const uint8_t* wr = codes + (int64_t)(row_ok ? row : 0) * (Kp / 4) + 16 * h;

    uint4 wv[kGemvUnroll];
    int b = b0;
    int cnt = min(kGemvUnroll, b1 - b);
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
        if (u < cnt && row_ok) wv[u] = ld_stream_v4(wr + 32 * (b + u));

    griddep_launch();  // the next kernel may start streaming its own weights now
    griddep_wait();    // activations are produced by the preceding kernel

    // Stage q (MT rows of K int8) into shared memory, zero-filling [K, Kp) and token rows past M. With a
    // 16-byte aligned q and 4+ tokens every chunk is one cp.async, all in flight at once (a loop of
    // load -> store round trips serialized 20 L2 latencies per thread at 16 tokens); otherwise plain
    // 16-byte loads, or a byte-wise copy for unaligned q.
    const int cpr = Kp / 16;  // 16-byte chunks per token row
    const bool q_vec = ((ldq & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 15) == 0) && (K % 16 == 0);
    if (q_vec && MT < 4) {  // a few chunks per thread: plain 16-byte loads
        for (int i = threadIdx.x; i < MT * cpr; i += blockDim.x) {
            const int m = i / cpr, k0 = (i - m * cpr) * 16;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m < mrows && k0 < K) v = *reinterpret_cast<const uint4*>(q + (int64_t)m * ldq + k0);
            reinterpret_cast<uint4*>(q_sm)[i] = v;
        }
    } else if (q_vec) {
        for (int i = threadIdx.x; i < MT * cpr; i += blockDim.x) {
            const int m = i / cpr, k0 = (i - m * cpr) * 16;
            const bool live = m < mrows && k0 < K;
            cp_async_16(q_sm + 16 * i, live ? (const void*)(q + (int64_t)m * ldq + k0) : (const void*)q,
                        live ? 16u : 0u);
        }
        cp_async_wait_all();
    } else {
        for (int i = threadIdx.x; i < MT * cpr; i += blockDim.x) {
            const int m = i / cpr, k0 = (i - m * cpr) * 16;
            uint8_t tmp[16];
            const int8_t* src = q + (int64_t)m * ldq + k0;
#pragma unroll
            for (int j = 0; j < 16; ++j) tmp[j] = (m < mrows && k0 + j < K) ? (uint8_t)src[j] : 0;
            reinterpret_cast<uint4*>(q_sm)[i] = *reinterpret_cast<uint4*>(tmp);
        }
    }
    __syncthreads();

    int acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0;
    const uint4* q4 = reinterpret_cast<const uint4*>(q_sm);

    while (cnt > 0) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            if (u < cnt) {
                const int bb = b + u;
                const uint32_t w[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t c[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) c[i] = (w[i] >> (6 - 2 * g)) & 0x03030303u;
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        // words [32bb + 8g + 4h, +4) of token m -> one 16-byte broadcast load
                        const uint4 qv = q4[m * cpr + 8 * bb + 2 * g + h];
                        int a = acc[m];
                        a = dp4a_us(c[0], (int)qv.x, a);
                        a = dp4a_us(c[1], (int)qv.y, a);
                        a = dp4a_us(c[2], (int)qv.z, a);
                        a = dp4a_us(c[3], (int)qv.w, a);
                        acc[m] = a;
                    }
                }
            }
        }
        b += cnt;
        cnt = min(kGemvUnroll, b1 - b);
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u)
            if (u < cnt && row_ok) wv[u] = ld_stream_v4(wr + 32 * (b + u));
    }

#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int v = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 1);
        if (h == 0) red[warp][r][m] = v;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < kGemvRows * MT; t += blockDim.x) {
        const int rr = t / MT, m = t - rr * MT;
        const int n = blockIdx.x * kGemvRows + rr;
        if (n < N && m < mrows) {
            int tot = 0;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) tot += red[w][rr][m];
            const float rs = __fdiv_rn(__ldg(wscale + (epi.scale_rows ? n / epi.scale_rows : 0)), s[m]);
            float v = __fmul_rn((float)(tot - sums[m]), rs);
            if (epi.bias) v = __fadd_rn(v, epi.bias[n]);
            if (epi.act == 1) v = gelu_tanh(v);
            if (epi.residual) v = __fadd_rn(epi.residual[(int64_t)m * epi.ld_res + n], v);
            y[(int64_t)m * ldy + n] = v;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// 2..16 tokens: warp-level int8 MMAs (mma.sync m16n8k32, A = unsigned codes, B = int8 activations).
// At these token counts the dp4a loop above is bound by its instruction rate (each weight code is
// multiplied M times); the MMA does 16 rows x 8 tokens x 32 k per instruction at 2048 MAC/cycle/SM, so
// the kernel is bound by the weight stream instead. The codes go from the loaded registers straight into
// the MMA; the tcgen05 path would stage 128-row weight tiles through tensor memory for 16 tokens.
//
// A warp owns 16 weight rows (one MMA row tile); thread (g = lane / 4, t = lane % 4) loads 8 bytes
// (words 2t, 2t+1) of each 32-byte i2_s block of rows g and g + 8, so a warp load instruction reads 8 full
// 32-byte sectors. For bit-plane p of the block, word 2t gives the codes of k = 32p + 8t + [0,4) and word
// 2t+1 those of k = 32p + 8t + [4,8); they are the A fragment's k = 4t + [0,4) and 16 + 4t + [0,4), and
// the B fragment reads the activations of exactly those k (one 8-byte shared-memory load per token):
// the MMA's k order is a permutation of the true order, which an exact int32 sum does not see.
// A CTA holds ROWT row tiles (16 ROWT rows); the 8 / ROWT warps of a row tile split its blocks and
// reduce through shared memory. Every CTA stages all M x K activations, so more rows per CTA means
// less of that (L2-resident, but read by every CTA at once) traffic per weight byte. The epilogue is
// the dp4a kernel's.
constexpr int kMmaQPad = 32;  // bytes added to each token row in shared memory (conflict-free 8-byte loads)

__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

template <int NT, int ROWT>  // NT n-tiles of 8 tokens; ROWT row tiles of 16 rows per CTA
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_i2s_mma_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ wscale, int N, int Kp,
                    const int8_t* __restrict__ q, int64_t ldq, int K, int mrows, const float* __restrict__ s,
                    const int32_t* __restrict__ sums, float* y, int64_t ldy, const Epilogue epi, const GemvBatch bt) {
    constexpr int MT = 8 * NT, WPT = kGemvWarps / ROWT;  // warps per row tile
    extern __shared__ __align__(16) uint8_t q_sm[];  // MT rows of (Kp + kMmaQPad) int8, zero past K / mrows
    __shared__ int red[kGemvWarps][kGemvRows][MT];
    codes += (int64_t)blockIdx.y * bt.w_stride;  // problem blockIdx.y of a batched launch
    q += (int64_t)blockIdx.y * bt.q_stride;
    s += (int64_t)blockIdx.y * bt.a_stride;
    sums += (int64_t)blockIdx.y * bt.a_stride;
    y += (int64_t)blockIdx.y * bt.y_stride;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt = warp / WPT, ws = warp - rt * WPT;  // row tile, K share within it
    const int g = lane >> 2, t = lane & 3;
    const int row_a = (blockIdx.x * ROWT + rt) * kGemvRows + g, row_b = row_a + 8;
    const bool ok_a = row_a < N, ok_b = row_b < N;
    const int nblk = Kp / kQK;
    const int per = (nblk + WPT - 1) / WPT;
    const int b0 = min(nblk, ws * per), b1 = min(nblk, b0 + per);
    const int64_t rbytes = Kp / 4;
    const uint8_t* wa = codes + (int64_t)(ok_a ? row_a : 0) * rbytes + 8 * t;
    const uint8_t* wb = codes + (int64_t)(ok_b ? row_b : 0) * rbytes + 8 * t;

    uint2 va[kGemvUnroll], vb[kGemvUnroll];
    int b = b0;
    int cnt = min(kGemvUnroll, b1 - b);
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
        if (u < cnt) {
            va[u] = ok_a ? ld_stream_v2(wa + 32 * (b + u)) : make_uint2(0x55555555u, 0x55555555u);
            vb[u] = ok_b ? ld_stream_v2(wb + 32 * (b + u)) : make_uint2(0x55555555u, 0x55555555u);
        }
    }

    griddep_launch();  // the next kernel may start streaming its own weights now
    griddep_wait();    // activations are produced by the preceding kernel

    // Stage the activations of this warp's K share only: the mrows token rows x [128 b0, 128 b1) bytes at a
    // row stride of Kp + kMmaQPad, zero past K (token rows past mrows are not staged: their B fragments are
    // zero). The ROWT warps that share the K range split the copy and meet at a named barrier; no
    // CTA-wide barrier stands between a warp and its MMAs.
    const int qstride = Kp + kMmaQPad;  // bytes
    const int c0 = 8 * b0, nck = 8 * (b1 - b0);  // 16-byte chunks of the share (8 per block)
    const bool q_vec = ((ldq & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 15) == 0) && (K % 16 == 0);
    if (q_vec) {
        for (int i = lane + 32 * rt; i < mrows * nck; i += 32 * ROWT) {
            const int m = i / nck, k0 = 16 * (c0 + i - m * nck);
            const bool live = k0 < K;
            cp_async_16(q_sm + (size_t)m * qstride + k0, live ? (const void*)(q + (int64_t)m * ldq + k0) : (const void*)q,
                        live ? 16u : 0u);
        }
        cp_async_wait_all();
    } else {
        for (int i = lane + 32 * rt; i < mrows * nck; i += 32 * ROWT) {
            const int m = i / nck, k0 = 16 * (c0 + i - m * nck);
            uint8_t tmp[16];
            const int8_t* src = q + (int64_t)m * ldq + k0;
#pragma unroll
            for (int j = 0; j < 16; ++j) tmp[j] = (k0 + j < K) ? (uint8_t)src[j] : 0;
            *reinterpret_cast<uint4*>(q_sm + (size_t)m * qstride + k0) = *reinterpret_cast<uint4*>(tmp);
        }
    }
    if (ROWT == 1) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + ws), "r"(32 * ROWT) : "memory");

    int acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[n][i] = 0;
    // token g of n-tile n reads its activations at q_sm + (8n + g) * qstride + 128 bb + 32 p + 8 t
    const uint8_t* qg = q_sm + (size_t)g * qstride + 8 * t;

    while (cnt > 0) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            if (u < cnt) {
                const int bb = b + u;
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const int sh = 6 - 2 * p;
                    const uint32_t a0 = (va[u].x >> sh) & 0x03030303u, a2 = (va[u].y >> sh) & 0x03030303u;
                    const uint32_t a1 = (vb[u].x >> sh) & 0x03030303u, a3 = (vb[u].y >> sh) & 0x03030303u;
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const uint2 bv = (8 * n + g < mrows)
                            ? *reinterpret_cast<const uint2*>(qg + (size_t)(8 * n) * qstride + 128 * bb + 32 * p)
                            : make_uint2(0u, 0u);
                        mma_u8s8_16832(acc[n], a0, a1, a2, a3, bv.x, bv.y);
                    }
                }
            }
        }
        b += cnt;
        cnt = min(kGemvUnroll, b1 - b);
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            if (u < cnt) {
                va[u] = ok_a ? ld_stream_v2(wa + 32 * (b + u)) : make_uint2(0x55555555u, 0x55555555u);
                vb[u] = ok_b ? ld_stream_v2(wb + 32 * (b + u)) : make_uint2(0x55555555u, 0x55555555u);
            }
        }
    }

    // D fragment: acc[n][0..1] = row g, tokens 8n + 2t + {0,1}; acc[n][2..3] = row g + 8, same tokens.
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        red[warp][g][8 * n + 2 * t] = acc[n][0];
        red[warp][g][8 * n + 2 * t + 1] = acc[n][1];
        red[warp][g + 8][8 * n + 2 * t] = acc[n][2];
        red[warp][g + 8][8 * n + 2 * t + 1] = acc[n][3];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ROWT * kGemvRows * MT; i += blockDim.x) {
        const int rr = i / MT, m = i - rr * MT;             // rr: row within the CTA
        const int rti = rr / kGemvRows, r16 = rr - rti * kGemvRows;
        const int n = blockIdx.x * ROWT * kGemvRows + rr;
        if (n < N && m < mrows) {
            int tot = 0;
#pragma unroll
            for (int w = 0; w < WPT; ++w) tot += red[rti * WPT + w][r16][m];
            const float rs = __fdiv_rn(__ldg(wscale + (epi.scale_rows ? n / epi.scale_rows : 0)), s[m]);
            float v = __fmul_rn((float)(tot - sums[m]), rs);
            if (epi.bias) v = __fadd_rn(v, epi.bias[n]);
            if (epi.act == 1) v = gelu_tanh(v);
            if (epi.residual) v = __fadd_rn(epi.residual[(int64_t)m * epi.ld_res + n], v);
            y[(int64_t)m * ldy + n] = v;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// 2..16 tokens, streaming form for launches with many rows (batched problems): the warp MMA arithmetic of
// gemv_i2s_mma_kernel, but every warp owns one 16-row tile over the full K and loops over row tiles
// (tile i = blockIdx.x * 8 + warp + i * 8 * gridDim.x), issuing the next tile's first weight loads before it
// writes the current tile's outputs. All token rows are staged once per CTA; no K split, no shared-memory
// reduction.
template <int NT>
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_mma_stream_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ wscale, int N, int Kp,
                       const int8_t* __restrict__ q, int64_t ldq, int K, int mrows, const float* __restrict__ s,
                       const int32_t* __restrict__ sums, float* y, int64_t ldy, const Epilogue epi,
                       const GemvBatch bt) {
    extern __shared__ __align__(16) uint8_t qs_sm[];  // mrows rows of (Kp + kMmaQPad) int8, zero past K
    __shared__ float s_sm[8 * NT];
    __shared__ int32_t u_sm[8 * NT];
    codes += (int64_t)blockIdx.y * bt.w_stride;
    q += (int64_t)blockIdx.y * bt.q_stride;
    s += (int64_t)blockIdx.y * bt.a_stride;
    sums += (int64_t)blockIdx.y * bt.a_stride;
    y += (int64_t)blockIdx.y * bt.y_stride;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nblk = Kp / kQK;
    const int64_t rbytes = Kp / 4;
    const int ntiles = (N + kGemvRows - 1) / kGemvRows;
    const int tstride = (int)gridDim.x * kGemvWarps;
    // The warp's blocks form one stream (tile tile0 blocks 0..nblk-1, then tile tile0 + tstride, ...); slot
    // u of the rings va / vb holds item i with i % 8 == u and is refilled with item i + 8 as soon as item i
    // is consumed, so eight loads per lane and row stay in flight across tile boundaries. Rows past N read
    // row 0 (their outputs are not stored).
    int tile = (int)blockIdx.x * kGemvWarps + warp, b = 0;  // next item to consume
    int lt = tile, lb = 0;                                  // next item to load
    const uint8_t *la, *lbp;
    auto rows_of = [&](int tt) {
        const int ra = tt * kGemvRows + g, rb = ra + 8;
        la = codes + (int64_t)(ra < N ? ra : 0) * rbytes + 8 * t;
        lbp = codes + (int64_t)(rb < N ? rb : 0) * rbytes + 8 * t;
    };
    rows_of(lt < ntiles ? lt : 0);
    uint2 va[kGemvUnroll], vb[kGemvUnroll];
    auto load_next = [&](int u) {
        va[u] = ld_stream_v2(la + 32 * lb);
        vb[u] = ld_stream_v2(lbp + 32 * lb);
        if (++lb == nblk) {
            lb = 0;
            lt += tstride;
            rows_of(lt < ntiles ? lt : 0);
        }
    };
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
        if (lt < ntiles) load_next(u);
    griddep_launch();
    griddep_wait();  // activations, scales and sums come from the preceding kernel
    const int qstride = Kp + kMmaQPad;
    const int cpr = Kp / 16;
    const bool q_vec = ((ldq & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 15) == 0) && (K % 16 == 0);
    for (int i = threadIdx.x; i < mrows * cpr; i += blockDim.x) {
        const int m = i / cpr, k0 = 16 * (i - m * cpr);
        if (q_vec) {
            const bool in = k0 < K;
            cp_async_16(qs_sm + (size_t)m * qstride + k0, in ? (const void*)(q + (int64_t)m * ldq + k0) : (const void*)q,
                        in ? 16u : 0u);
        } else {
            uint8_t tmp[16];
            const int8_t* src = q + (int64_t)m * ldq + k0;
#pragma unroll
            for (int j = 0; j < 16; ++j) tmp[j] = (k0 + j < K) ? (uint8_t)src[j] : 0;
            *reinterpret_cast<uint4*>(qs_sm + (size_t)m * qstride + k0) = *reinterpret_cast<uint4*>(tmp);
        }
    }
    if (threadIdx.x < 8 * NT) {
        s_sm[threadIdx.x] = threadIdx.x < mrows ? s[threadIdx.x] : 1.0f;
        u_sm[threadIdx.x] = threadIdx.x < mrows ? sums[threadIdx.x] : 0;
    }
    cp_async_wait_all();
    __syncthreads();
    const uint8_t* qg = qs_sm + (size_t)g * qstride + 8 * t;
    int acc[2][NT][4];  // two MMA chains per n-tile (even / odd bit-planes), summed when a tile is done
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[c][n][i] = 0;
    while (tile < ntiles) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            if (tile < ntiles) {
                const uint2 xa = va[u], xb = vb[u];
                if (lt < ntiles) load_next(u);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const int sh = 6 - 2 * p;
                    const uint32_t a0 = (xa.x >> sh) & 0x03030303u, a2 = (xa.y >> sh) & 0x03030303u;
                    const uint32_t a1 = (xb.x >> sh) & 0x03030303u, a3 = (xb.y >> sh) & 0x03030303u;
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const uint2 bv = (8 * n + g < mrows)
                            ? *reinterpret_cast<const uint2*>(qg + (size_t)(8 * n) * qstride + 128 * b + 32 * p)
                            : make_uint2(0u, 0u);
                        mma_u8s8_16832(acc[p & 1][n], a0, a1, a2, a3, bv.x, bv.y);
                    }
                }
                if (++b == nblk) {  // tile done: write its outputs
                    const int row_a = tile * kGemvRows + g;
                    // D fragment: acc[n][0..1] = row g, tokens 8n + 2t + {0,1}; acc[n][2..3] = row g + 8.
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int m = 8 * n + 2 * t + (i & 1), row = row_a + 8 * (i >> 1);
                            if (m < mrows && row < N) {
                                const float rs =
                                    __fdiv_rn(__ldg(wscale + (epi.scale_rows ? row / epi.scale_rows : 0)), s_sm[m]);
                                float v = __fmul_rn((float)(acc[0][n][i] + acc[1][n][i] - u_sm[m]), rs);
                                if (epi.bias) v = __fadd_rn(v, epi.bias[row]);
                                if (epi.act == 1) v = gelu_tanh(v);
                                if (epi.residual) v = __fadd_rn(epi.residual[(int64_t)m * epi.ld_res + row], v);
                                y[(int64_t)m * ldy + row] = v;
                            }
                            acc[0][n][i] = acc[1][n][i] = 0;
                        }
                    b = 0;
                    tile += tstride;
                }
            }
        }
    }
}

template <int NT>
static cudaError_t launch_mma_stream(const I2sWeight& w, const int8_t* q, int64_t ldq, int mrows, const float* s,
                                     const int32_t* sums, float* y, int64_t ldy, const Epilogue& epi,
                                     const GemvBatch& bt, cudaStream_t st) {
    const size_t smem = (size_t)mrows * (size_t)(w.Kp + kMmaQPad);
    auto kfn = gemv_mma_stream_kernel<NT>;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), smem);
        if (e != cudaSuccess) return e;
    }
    const int64_t ntiles = ceil_div(w.N, kGemvRows);
    const int64_t total = ntiles * bt.count;
    int64_t tpw = total / (148 * 8 * 8);
    tpw = tpw < 1 ? 1 : (tpw > 8 ? 8 : tpw);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(ntiles, kGemvWarps * tpw), (unsigned)bt.count);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, w.codes, w.scale, (int)w.N, (int)w.Kp, q, ldq, (int)w.K, mrows, s, sums, y,
                              ldy, epi, bt);
}

template <int NT, int ROWT>
static cudaError_t launch_mma_nt(const I2sWeight& w, const int8_t* q, int64_t ldq, int mrows, const float* s,
                                 const int32_t* sums, float* y, int64_t ldy, const Epilogue& epi, const GemvBatch& bt,
                                 cudaStream_t st) {
    const size_t smem = (size_t)(8 * NT) * (size_t)(w.Kp + kMmaQPad);
    auto kfn = gemv_i2s_mma_kernel<NT, ROWT>;
    if (smem + sizeof(int) * kGemvWarps * kGemvRows * 8 * NT > 48 * 1024) {
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(w.N, ROWT * kGemvRows), (unsigned)bt.count);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, w.codes, w.scale, (int)w.N, (int)w.Kp, q, ldq, (int)w.K, mrows, s, sums, y,
                              ldy, epi, bt);
}

// Row tiles per CTA for the MMA GEMV: enough CTAs to keep about one per SM streaming weights, and as few
// as that allows, so the activations (staged by every CTA) are re-read as little as possible.
static int mma_row_tiles(int64_t N, int count) {
    const int64_t tiles = ceil_div(N, kGemvRows) * count;
    if (tiles >= 4 * 148) return 4;
    if (tiles >= 2 * 148) return 2;
    return 1;
}

template <int NT>
static cudaError_t launch_mma(const I2sWeight& w, const int8_t* q, int64_t ldq, int mrows, const float* s,
                              const int32_t* sums, float* y, int64_t ldy, const Epilogue& epi, const GemvBatch& bt,
                              cudaStream_t st) {
    switch (mma_row_tiles(w.N, bt.count)) {
        case 4: return launch_mma_nt<NT, 4>(w, q, ldq, mrows, s, sums, y, ldy, epi, bt, st);
        case 2: return launch_mma_nt<NT, 2>(w, q, ldq, mrows, s, sums, y, ldy, epi, bt, st);
        default: return launch_mma_nt<NT, 1>(w, q, ldq, mrows, s, sums, y, ldy, epi, bt, st);
    }
}

// ------------------------------------------------------------------------------------------------
// One token, register-streaming form for launches with many rows that the TMA-fed kernel does not take
// (problems not back to back, K % 16 != 0, unaligned activations): every warp owns 64 weight rows at a
// time over the full K (lane (r, h) reads 16 bytes of each 32-byte block of rows r, r + 16, r + 32 and
// r + 48), with the warp's blocks streamed through a two-item register ring (eight 16-byte loads in
// flight per lane, refilled across group boundaries), and walks groups g = blockIdx.x * 8 + warp + i * 8 *
// gridDim.x. The token's codes are staged once per CTA; there is no K split across warps and no
// shared-memory reduction. The integer sums are exact, so results equal gemv_i2s_kernel's bit for bit.
template <int R, int D>  // R rows per lane (a warp group is 16 R rows); ring depth D (items of R 16-byte loads)
__global__ void __launch_bounds__(kGemvWarps * 32, 3)
gemv1_stream_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ wscale, int N, int Kp,
                    const int8_t* __restrict__ q, int K, const float* __restrict__ s, const int32_t* __restrict__ sums,
                    float* y, const Epilogue epi, const GemvBatch bt) {
    extern __shared__ __align__(16) uint8_t q1_sm[];  // Kp int8, zero beyond K
    codes += (int64_t)blockIdx.y * bt.w_stride;
    q += (int64_t)blockIdx.y * bt.q_stride;
    s += (int64_t)blockIdx.y * bt.a_stride;
    sums += (int64_t)blockIdx.y * bt.a_stride;
    y += (int64_t)blockIdx.y * bt.y_stride;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 1, h = lane & 1;
    const int nblk = Kp / kQK;
    const int64_t rbytes = Kp / 4;
    constexpr int GR = 16 * R;  // rows per warp group
    const int ngroups = (N + GR - 1) / GR;
    const int gstride = (int)gridDim.x * kGemvWarps;
    // Lane (r, h) owns rows r, r + 16, ..., r + 16 (R-1) of the warp's group: one activation load per
    // bit-plane serves R rows. Rows past N read the group's first row (their outputs are not stored).
    auto group_ptr = [&](int gg) { return codes + ((int64_t)gg * GR + r) * rbytes + 16 * h; };
    auto row_ok = [&](int gg, int j) { return gg * GR + r + 16 * j < N; };
    // The warp's blocks form one stream: group g0 blocks 0..nblk-1, then group g0 + gstride, ... Item i
    // (one block of the R rows) sits in slot i % D of the ring wv; consuming it reloads the slot with
    // item i + D, so R D 16-byte loads per lane stay in flight across group boundaries.
    int g = (int)blockIdx.x * kGemvWarps + warp, b = 0;  // next item to consume
    int lg = g, lb = 0;                                  // next item to load
    const uint8_t* lp;
    int lstep[R];  // byte offsets of the R rows from lp (Kp <= 48 K keeps 48 rows within int range)
    auto set_group = [&](int gg) {
        const int gc = gg < ngroups ? gg : 0;
        lp = group_ptr(gc);
#pragma unroll
        for (int j = 0; j < R; ++j) lstep[j] = row_ok(gc, j) ? 16 * j * (int)rbytes : -r * (int)rbytes;
    };
    set_group(lg);
    uint4 wv[D][R];
    auto load_next = [&](int slot) {
#pragma unroll
        for (int j = 0; j < R; ++j) wv[slot][j] = ld_stream_v4(lp + lstep[j] + 32 * lb);
        if (++lb == nblk) {
            lb = 0;
            lg += gstride;
            set_group(lg);
        }
    };
#pragma unroll
    for (int u = 0; u < D; ++u)
        if (lg < ngroups) load_next(u);
    griddep_launch();
    griddep_wait();  // the token's codes come from the preceding kernel
    const bool q_vec = ((reinterpret_cast<uintptr_t>(q) & 15) == 0) && (K % 16 == 0);
    for (int i = threadIdx.x; i < Kp / 16; i += blockDim.x) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (q_vec) {
            if (16 * i < K) v = *reinterpret_cast<const uint4*>(q + 16 * i);
        } else {
            uint8_t tmp[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) tmp[j] = (16 * i + j < K) ? (uint8_t)q[16 * i + j] : 0;
            v = *reinterpret_cast<uint4*>(tmp);
        }
        reinterpret_cast<uint4*>(q1_sm)[i] = v;
    }
    const float s0 = s[0];
    const int32_t sum0 = sums[0];
    __syncthreads();
    const uint4* q4 = reinterpret_cast<const uint4*>(q1_sm) + h;
    // Bit-plane gp is masked in place (byte & (3 << (6 - 2gp))), so its chain accumulates 4^(3-gp) times
    // the plane's exact integer dot product; the planes are shifted back when the rows are done.
    int acc[R][4];  // [row j][plane]
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[j][p] = 0;
    while (g < ngroups) {
#pragma unroll
        for (int u = 0; u < D; ++u) {
            if (g < ngroups) {
                uint4 cur[R];
#pragma unroll
                for (int j = 0; j < R; ++j) cur[j] = wv[u][j];
                if (lg < ngroups) load_next(u);
#pragma unroll
                for (int gp = 0; gp < 4; ++gp) {
                    const uint32_t m = 0x03030303u << (6 - 2 * gp);
                    const uint4 qv = q4[8 * b + 2 * gp];
#pragma unroll
                    for (int j = 0; j < R; ++j) {
                        int a = acc[j][gp];
                        a = dp4a_us(cur[j].x & m, (int)qv.x, a);
                        a = dp4a_us(cur[j].y & m, (int)qv.y, a);
                        a = dp4a_us(cur[j].z & m, (int)qv.z, a);
                        a = dp4a_us(cur[j].w & m, (int)qv.w, a);
                        acc[j][gp] = a;
                    }
                }
                if (++b == nblk) {  // group done: reduce and store its rows
                    const float ws0 = epi.scale_rows ? 0.0f : __ldg(wscale);
#pragma unroll
                    for (int j = 0; j < R; ++j) {
                        const int part = ((acc[j][0] >> 6) + (acc[j][1] >> 4)) + ((acc[j][2] >> 2) + acc[j][3]);
                        const int tot = part + __shfl_xor_sync(0xffffffffu, part, 1);
                        const int row = g * GR + r + 16 * j;
                        if (h == 0 && row < N) {
                            const float wsr = epi.scale_rows ? __ldg(wscale + row / epi.scale_rows) : ws0;
                            const float rs = __fdiv_rn(wsr, s0);
                            float v = __fmul_rn((float)(tot - sum0), rs);
                            if (epi.bias) v = __fadd_rn(v, epi.bias[row]);
                            if (epi.act == 1) v = gelu_tanh(v);
                            if (epi.residual) v = __fadd_rn(epi.residual[row], v);
                            y[row] = v;
                        }
#pragma unroll
                        for (int p = 0; p < 4; ++p) acc[j][p] = 0;
                    }
                    b = 0;
                    g += gstride;
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// One token, TMA-fed form for launches with many rows: batched decode problems stored back to back (one
// 2D tensor of count * N rows x Kp/4 bytes). The weight stream bypasses registers: every warp owns a
// ring of `nst` shared-memory stages, each one 64 rows x 128 bytes (four 32-byte blocks of each row)
// brought in by a single tiled TMA load with 128-byte swizzle, and keeps the next nst - 1 stages in flight
// while it computes one. The grid is one persistent wave (one 8-warp CTA per SM); warp w walks the
// contiguous range [w G / W, (w + 1) G / W) of the G = count * ceil(N / 64) row groups (problem-major), so
// it changes problem rarely; on a change it reloads its own copy of the problem's int8 activations with
// one bulk copy. Lane (r, h) = (lane % 16, lane / 16) reads the 16-byte half h of each block of rows
// r + 16 j, j = 0..3; with the swizzle (16-byte chunk index XOR row % 8) the eight lanes of each
// shared-memory phase hit eight different bank groups, and the activation loads are broadcasts. Same
// integer arithmetic as the other one-token kernels (bit-plane masks, exact sums), same epilogue.
// Every mbarrier wait is bounded; after a timeout the warp records it in the device error word, waits
// (bounded) for its copies still in flight and returns.
constexpr int kT1Warps = 8;                     // warps per CTA (one CTA per SM)
constexpr int kT1Rows = 64;                     // rows per group
constexpr int kT1Box = 128;                     // bytes of each row per stage
constexpr int kT1Stage = kT1Rows * kT1Box;      // 8 KB

__global__ void __launch_bounds__(kT1Warps * 32, 1)
gemv1_tma_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ wscale, int N, int Kp,
                 const int8_t* __restrict__ q, int K, const float* __restrict__ s, const int32_t* __restrict__ sums,
                 float* y, const Epilogue epi, const GemvBatch bt, int nst) {
    extern __shared__ __align__(16) uint8_t t1_sm[];  // aligned to 1024 by hand below
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane & 15, h = lane >> 4;
    // stages 1024-byte aligned (the swizzle pattern follows shared-memory address bits 7..9)
    const uint32_t a0 = smem_u32(t1_sm), a1 = (a0 + 1023u) & ~1023u;
    uint8_t* base = t1_sm + (a1 - a0);
    const int kpa = (Kp + 127) & ~127;
    uint8_t* ring = base + (size_t)warp * nst * kT1Stage;
    uint8_t* act = base + (size_t)kT1Warps * nst * kT1Stage + (size_t)warp * kpa;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + (size_t)kT1Warps * nst * kT1Stage + (size_t)kT1Warps * kpa) +
                     warp * (nst + 1);
    uint64_t* abar = bars + nst;
    const int nblk = Kp / kQK, rbytes = Kp / 4;
    const int nchunk = (rbytes + kT1Box - 1) / kT1Box;
    const int ngroups = (N + kT1Rows - 1) / kT1Rows;
    const int64_t G = (int64_t)ngroups * bt.count;
    const int64_t nw = (int64_t)gridDim.x * kT1Warps, gw = (int64_t)blockIdx.x * kT1Warps + warp;
    const int64_t gbeg = gw * G / nw, gend = (gw + 1) * G / nw;
    const int nstages = (int)(gend - gbeg) * nchunk;

    if (lane == 0) {
        for (int i = 0; i <= nst; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    auto issue = [&](int k) {  // lane 0
        const int64_t gi = gbeg + k / nchunk;
        const int p = (int)(gi / ngroups), g = (int)(gi - (int64_t)p * ngroups);
        uint64_t* bar = &bars[k % nst];
        mbar_arrive_expect_tx(bar, kT1Stage);
        tma_load_2d(ring + (size_t)(k % nst) * kT1Stage, &tmap, bar, kT1Box * (k % nchunk), p * N + g * kT1Rows);
    };
    int issued = min(nst, nstages);
    if (lane == 0)
        for (int k = 0; k < issued; ++k) issue(k);
    griddep_launch();
    griddep_wait();  // the tokens' codes come from the preceding kernel
    for (int i = K + 16 * lane; i < kpa; i += 16 * 32) *reinterpret_cast<uint4*>(act + i) = make_uint4(0, 0, 0, 0);

    int acc[4][4];  // [row j][bit-plane], plane gp scaled by 4^(3-gp) (masked in place)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[j][p] = 0;
    int cur_p = -1;
    uint32_t aphase = 0;
    bool act_pending = false;
    float s0 = 1.0f;
    int32_t sum0 = 0;
    bool ok = true;
    int k = 0;
    for (; k < nstages; ++k) {
        const int c = k % nchunk;
        const int64_t gi = gbeg + k / nchunk;
        const int p = (int)(gi / ngroups), g = (int)(gi - (int64_t)p * ngroups);
        if (p != cur_p) {  // new problem: this warp's activation copy
            __syncwarp();
            fence_proxy_async_smem();
            if (lane == 0) {
                mbar_arrive_expect_tx(abar, (uint32_t)K);
                bulk_load(act, q + (int64_t)p * bt.q_stride, (uint32_t)K, abar);
            }
            act_pending = true;
            if (!mbar_wait(abar, aphase)) {
                ok = false;
                break;
            }
            act_pending = false;
            aphase ^= 1u;
            s0 = s[(int64_t)p * bt.a_stride];
            sum0 = sums[(int64_t)p * bt.a_stride];
            cur_p = p;
        }
        const int slot = k % nst;
        if (!mbar_wait(&bars[slot], (uint32_t)((k / nst) & 1))) {
            ok = false;
            break;
        }
        const uint8_t* st = ring + (size_t)slot * kT1Stage;
        const int nb = min(4, nblk - 4 * c);
        const uint4* q4 = reinterpret_cast<const uint4*>(act) + 32 * c + h;
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            if (bb < nb) {
                uint4 wv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    wv[j] = *reinterpret_cast<const uint4*>(st + (r + 16 * j) * kT1Box + 16 * ((2 * bb + h) ^ (r & 7)));
#pragma unroll
                for (int gp = 0; gp < 4; ++gp) {
                    const uint32_t m = 0x03030303u << (6 - 2 * gp);
                    const uint4 qv = q4[8 * bb + 2 * gp];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        int a = acc[j][gp];
                        a = dp4a_us(wv[j].x & m, (int)qv.x, a);
                        a = dp4a_us(wv[j].y & m, (int)qv.y, a);
                        a = dp4a_us(wv[j].z & m, (int)qv.z, a);
                        a = dp4a_us(wv[j].w & m, (int)qv.w, a);
                        acc[j][gp] = a;
                    }
                }
            }
        }
        __syncwarp();              // every lane is done reading the slot
        fence_proxy_async_smem();  // order those reads before the TMA load that refills it
        if (k + nst < nstages) {
            if (lane == 0) issue(k + nst);
            issued = k + nst + 1;
        }
        if (c == nchunk - 1) {  // group done: reduce and store its 64 rows
            float* yp = y + (int64_t)p * bt.y_stride;
            const float ws0 = epi.scale_rows ? 0.0f : __ldg(wscale);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int part = ((acc[j][0] >> 6) + (acc[j][1] >> 4)) + ((acc[j][2] >> 2) + acc[j][3]);
                const int tot = part + __shfl_xor_sync(0xffffffffu, part, 16);
                const int row = g * kT1Rows + r + 16 * j;
                if (h == 0 && row < N) {
                    const float wsr = epi.scale_rows ? __ldg(wscale + row / epi.scale_rows) : ws0;
                    const float rs = __fdiv_rn(wsr, s0);
                    float v = __fmul_rn((float)(tot - sum0), rs);
                    if (epi.bias) v = __fadd_rn(v, epi.bias[row]);
                    if (epi.act == 1) v = gelu_tanh(v);
                    if (epi.residual) v = __fadd_rn(epi.residual[row], v);
                    yp[row] = v;
                }
#pragma unroll
                for (int p2 = 0; p2 < 4; ++p2) acc[j][p2] = 0;
            }
        }
    }
    if (!ok) {  // drain this warp's copies still in flight before the CTA can exit
        if (act_pending) mbar_wait(abar, aphase, 2u);
        for (int kk = k; kk < issued; ++kk) mbar_wait(&bars[kk % nst], (uint32_t)((kk / nst) & 1), 2u);
    }
}

// Shared memory of gemv1_tma_kernel for a ring of nst stages per warp.
static size_t tma1_smem(int nst, int64_t Kp) {
    const size_t kpa = (size_t)((Kp + 127) / 128 * 128);
    return 1024 + (size_t)kT1Warps * nst * kT1Stage + (size_t)kT1Warps * kpa + (size_t)kT1Warps * (nst + 1) * 8;
}

// The TMA-fed kernel when its requirements hold (weights of all problems back to back and 16-byte
// aligned, K % 16 == 0, aligned activations, a ring of at least two stages per warp); returns false to
// let the caller use the register-streaming kernel.
static bool try_launch_tma1(const I2sWeight& w, const int8_t* q, const float* s, const int32_t* sums, float* y,
                            const Epilogue& epi, const GemvBatch& bt, cudaStream_t st, cudaError_t* err) {
    const int64_t rbytes = w.Kp / 4;
    if (w.K % 16 != 0 || (reinterpret_cast<uintptr_t>(q) & 15) != 0) return false;
    if (bt.count > 1 && (bt.w_stride != w.N * rbytes || bt.q_stride % 16 != 0)) return false;
    if (w.N * bt.count >= (int64_t)1 << 31) return false;
    int nst = 0;
    for (int d = 4; d >= 2 && !nst; --d)
        if (tma1_smem(d, w.Kp) <= 227 * 1024) nst = d;
    if (!nst) return false;
    CUtensorMap tm;
    if (!tmap_u8_2d(&tm, w.codes, (uint64_t)rbytes, (uint64_t)(w.N * bt.count), (uint64_t)rbytes, kT1Box, kT1Rows,
                    CU_TENSOR_MAP_SWIZZLE_128B))
        return false;
    const size_t smem = tma1_smem(nst, w.Kp);
    *err = ensure_dynamic_smem(reinterpret_cast<const void*>(gemv1_tma_kernel), smem);
    if (*err != cudaSuccess) return true;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t G = ceil_div(w.N, kT1Rows) * bt.count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(G < (int64_t)sms * kT1Warps ? ceil_div(G, kT1Warps) : sms));
    cfg.blockDim = dim3(kT1Warps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    *err = cudaLaunchKernelEx(&cfg, gemv1_tma_kernel, tm, w.scale, (int)w.N, (int)w.Kp, q, (int)w.K, s, sums, y, epi,
                              bt, nst);
    return true;
}

// 16-row tiles: the streaming kernels (TMA-fed or register ring for one token, MMA ring for 2..16) serve
// launches with at least this many tiles in total; smaller launches use the K-split kernels, which spread
// few rows over more warps.
constexpr int64_t kStreamMinGroups = 148 * 8 * 2;

static cudaError_t launch_stream1(const I2sWeight& w, const int8_t* q, const float* s, const int32_t* sums, float* y,
                                  const Epilogue& epi, const GemvBatch& bt, cudaStream_t st) {
    const int64_t ngroups = ceil_div(w.N, (int64_t)16 * kS1R);
    const int64_t total = ngroups * bt.count;
    // Groups per warp: as few CTAs as one wave needs (each warp then streams its groups without a CTA
    // boundary in between).
    int64_t gpw = ceil_div(total, (int64_t)148 * 3 * kGemvWarps);
    gpw = gpw < 1 ? 1 : gpw;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(ngroups, kGemvWarps * gpw), (unsigned)bt.count);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = (size_t)w.Kp;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv1_stream_kernel<kS1R, kS1D>, w.codes, w.scale, (int)w.N, (int)w.Kp, q, (int)w.K, s, sums, y, epi, bt);
}

template <int MT>
static cudaError_t launch_mt(const I2sWeight& w, const int8_t* q, int64_t ldq, int mrows, const float* s,
                             const int32_t* sums, float* y, int64_t ldy, const Epilogue& epi, const GemvBatch& bt,
                             cudaStream_t st) {
    const size_t smem = (size_t)MT * (size_t)w.Kp;
    auto kfn = gemv_i2s_kernel<MT>;
    // Dynamic + static shared memory above 48 KB needs the opt-in attribute.
    if (smem + sizeof(int) * kGemvWarps * kGemvRows * MT > 48 * 1024) {
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kfn), smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(w.N, kGemvRows), (unsigned)bt.count);
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, w.codes, w.scale, (int)w.N, (int)w.Kp, q, ldq, (int)w.K, mrows, s, sums, y,
                              ldy, epi, bt);
}

cudaError_t launch_gemv_i2s(const I2sWeight& w, const Q8Act& a, float* y, int64_t ldy, const Epilogue& epi,
                            cudaStream_t st, const GemvBatch& bt) {
    // Token groups of up to 16, each one pass over the weights; a group of m tokens runs the smallest
    // power-of-two variant >= m with the extra token rows zero. A batched call (bt.count problems) runs each
    // token group of every problem in the same launch.
    for (int64_t m0 = 0; m0 < a.M; m0 += 16) {
        const int mt = (int)((a.M - m0) < 16 ? (a.M - m0) : 16);
        const int8_t* q = a.q + m0 * a.ldq;
        const float* s = a.s + m0;
        const int32_t* sums = a.sums + m0;
        float* yy = y + m0 * ldy;
        Epilogue ep = epi;  // the residual rows move with the token group
        if (ep.residual) ep.residual += m0 * ep.ld_res;
        cudaError_t e = cudaSuccess;
        const bool many = ceil_div(w.N, kGemvRows) * bt.count >= kStreamMinGroups;
        if (mt == 1 && many && try_launch_tma1(w, q, s, sums, yy, ep, bt, st, &e)) {
        } else if (mt == 1 && many && w.Kp <= 48 * 1024)
            e = launch_stream1(w, q, s, sums, yy, ep, bt, st);
        else if (mt == 1) e = launch_mt<1>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, bt, st);
        else if (many && (size_t)mt * (size_t)(w.Kp + kMmaQPad) <= 200 * 1024)
            e = (mt <= 8) ? launch_mma_stream<1>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, bt, st)
                          : launch_mma_stream<2>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, bt, st);
        else if (mt <= 8) e = launch_mma<1>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, bt, st);
        else e = launch_mma<2>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, bt, st);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

}  // namespace b2s
