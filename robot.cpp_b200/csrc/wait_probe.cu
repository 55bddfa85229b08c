// wait_probe.cu -- b2s_debug_wait_timeout: runs the failure path of the pipelined kernels' bounded waits.
//
// Every mbarrier wait in the tensor-core GEMMs is bounded (mbar_wait, b2s_common.cuh). When one runs out the
// kernel sets bit 0 of the device error word, stops issuing work, waits (bounded again) for the copies and
// MMAs it already issued, frees its tensor memory and returns, so the CUDA context stays usable and the host
// reads the failure with b2s_device_error. This entry point makes that sequence happen on purpose, in one
// small CTA with the same resources held: 32 TMEM columns allocated, one bulk copy in flight into shared
// memory, then a wait on an mbarrier that nothing arrives at, bounded by the caller's limit. No wait here is
// unbounded and nothing faults: the wait simply gives up.
#include <cuda_runtime.h>

#include "b2s.h"
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace {

constexpr uint32_t kProbeBytes = 4096;

__global__ void __launch_bounds__(64, 1) wait_probe_kernel(const uint8_t* __restrict__ src, uint32_t bytes,
                                                           uint64_t limit_ns) {
    __shared__ __align__(128) uint8_t buf[kProbeBytes];
    __shared__ __align__(8) uint64_t landed, never;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        b2s::mbar_init(&landed, 1);
        b2s::mbar_init(&never, 1);  // its one arrival never comes
        b2s::fence_mbar_init();
    }
    if (warp == 0) {
        b2s::tmem_alloc(&tmem_slot, 32);
        b2s::tmem_relinquish();
    }
    b2s::tc_fence_before();
    __syncthreads();
    b2s::tc_fence_after();
    if (warp == 0 && lane == 0) {  // the "producer": one copy in flight
        b2s::mbar_arrive_expect_tx(&landed, bytes);
        b2s::bulk_load(buf, src, bytes, &landed);
    }
    if (warp == 1 && lane == 0) {  // the "consumer": a wait that runs out and records bit 0
        (void)b2s::mbar_wait(&never, 0, 1u, limit_ns);
    }
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // Drain: the copy must land before this CTA's shared memory goes away (bounded, bit 1 on failure).
        b2s::mbar_wait(&landed, 0, 2u);
    }
    b2s::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        b2s::tc_fence_after();
        b2s::tmem_dealloc(tmem_slot, 32);
    }
}

}  // namespace

extern "C" int b2s_debug_wait_timeout(const void* src, size_t bytes, uint64_t wait_limit_ns, void* stream) {
    int rc = b2s_device_check();
    if (rc) return rc;
    if (!src || bytes == 0 || bytes > kProbeBytes || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src) & 15) != 0)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG,
                                   "debug_wait_timeout: src must be 16-byte aligned, 16..4096 bytes, a multiple of 16");
    if (wait_limit_ns == 0 || wait_limit_ns > 1000000000ull)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "debug_wait_timeout: wait limit must be in (0, 1 s]");
    wait_probe_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(src),
                                                                       (uint32_t)bytes, wait_limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return b2s::set_last_error(B2S_ERR_CUDA, cudaGetErrorString(e));
    return B2S_OK;
}
