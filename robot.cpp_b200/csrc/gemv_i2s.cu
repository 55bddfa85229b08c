// gemv_i2s.cu -- decode-size (M <= 16) i2_s x int8 GEMV with dp4a.
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
// Weight loads for the first range are issued before griddepcontrol.wait, so when launched with
// programmatic stream serialization the weight stream overlaps the tail of the kernel that produces
// the activations.
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace b2s {

constexpr int kGemvRows = 16;   // rows per CTA
constexpr int kGemvWarps = 8;   // warps per CTA (split K)
constexpr int kGemvUnroll = 8;  // 16-byte loads in flight per lane

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
                const int32_t* __restrict__ sums, float* y, int64_t ldy, const Epilogue epi) {
    extern __shared__ __align__(16) uint8_t q_sm[];  // MT x Kp int8, zero beyond K and beyond mrows
    __shared__ int red[kGemvWarps][kGemvRows][MT];

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

template <int MT>
static cudaError_t launch_mt(const I2sWeight& w, const int8_t* q, int64_t ldq, int mrows, const float* s,
                             const int32_t* sums, float* y, int64_t ldy, const Epilogue& epi, cudaStream_t st) {
    const size_t smem = (size_t)MT * (size_t)w.Kp;
    auto kfn = gemv_i2s_kernel<MT>;
    // Dynamic + static shared memory above 48 KB needs the opt-in attribute (raised once per size).
    static int opted_in = 0;
    if (smem + sizeof(int) * kGemvWarps * kGemvRows * MT > 48 * 1024 && (int)smem > opted_in) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        opted_in = (int)smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(w.N, kGemvRows));
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, w.codes, w.scale, (int)w.N, (int)w.Kp, q, ldq, (int)w.K, mrows, s, sums, y,
                              ldy, epi);
}

cudaError_t launch_gemv_i2s(const I2sWeight& w, const Q8Act& a, float* y, int64_t ldy, const Epilogue& epi,
                            cudaStream_t st) {
    // Token groups of up to 16, each one pass over the weights; a group of m tokens runs the smallest
    // power-of-two variant >= m with the extra token rows zero.
    for (int64_t m0 = 0; m0 < a.M; m0 += 16) {
        const int mt = (int)((a.M - m0) < 16 ? (a.M - m0) : 16);
        const int8_t* q = a.q + m0 * a.ldq;
        const float* s = a.s + m0;
        const int32_t* sums = a.sums + m0;
        float* yy = y + m0 * ldy;
        Epilogue ep = epi;  // the residual rows move with the token group
        if (ep.residual) ep.residual += m0 * ep.ld_res;
        cudaError_t e;
        if (mt == 1) e = launch_mt<1>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, st);
        else if (mt == 2) e = launch_mt<2>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, st);
        else if (mt <= 4) e = launch_mt<4>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, st);
        else if (mt <= 8) e = launch_mt<8>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, st);
        else e = launch_mt<16>(w, q, a.ldq, mt, s, sums, yy, ldy, ep, st);
        if (e != cudaSuccess) return e;
    }
    return cudaGetLastError();
}

}  // namespace b2s
