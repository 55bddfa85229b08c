// peer.cu -- host side of the N-split MUL_MAT over several GPUs (C ABI in include/b2s.h).
//
// A very large-M MUL_MAT is split over the output rows of W: rank r of g owns weight rows [n0_r, n1_r),
// a contiguous byte range of the i2_s tensor because rows are K/4 (or Kp/4 when row-padded) bytes each.
// The activations are replicated; each rank computes its column slice Y[:, n0_r:n1_r) and its GEMM
// epilogue stores that slice straight into the root GPU's output over NVLink: the root exports its
// output buffer (a CUDA IPC handle of the enclosing allocation plus the buffer's offset in it), the other
// ranks open it and pass `peer_ptr + n0_r` (row stride N) as the kernel's output. The stores are plain
// peer stores issued by the epilogue; there is no gather kernel, no collective and no multicast. How the 72 handle bytes travel between processes (a process
// group broadcast, a socket) is the caller's choice.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "b2s.h"
#include "b2s_common.cuh"
#include "b2s_internal.h"

namespace {

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return B2S_OK;
    (void)cudaGetLastError();
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return b2s::set_last_error(B2S_ERR_CUDA, buf);
}

// A CUDA IPC handle names a whole allocation, while callers pass pointers that an allocator (a caching
// allocator such as torch's) may have carved out of a larger cudaMalloc block. The exported bytes are the
// handle of the enclosing allocation followed by the pointer's byte offset inside it.
using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn get_range_fn() {
    static GetRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetRangeFn>(p);
    });
    return fn;
}

std::mutex g_open_mu;
std::map<void*, void*> g_open_base;  // pointer returned by b2s_peer_open -> mapped allocation base

}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(uint64_t) == B2S_PEER_HANDLE_BYTES, "peer handle size");

extern "C" {

int b2s_nsplit_range(int64_t n_rows, int world, int rank, int64_t* n0, int64_t* n1) {
    if (n_rows < 0 || world <= 0 || rank < 0 || rank >= world || !n0 || !n1)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "nsplit_range: need n_rows >= 0 and 0 <= rank < world");
    const int64_t base = n_rows / world, extra = n_rows % world;
    *n0 = rank * base + (rank < extra ? rank : extra);
    *n1 = *n0 + base + (rank < extra ? 1 : 0);
    return B2S_OK;
}

size_t b2s_i2s_shard_rows(const void* src, int32_t type, int64_t nrow, int64_t n_per_row, int64_t r0, int64_t r1,
                          void* dst) {
    if (!src || !dst || nrow <= 0 || n_per_row <= 0 || r0 < 0 || r1 <= r0 || r1 > nrow) {
        b2s::set_last_error(B2S_ERR_INVALID_ARG, "i2s_shard_rows: need 0 <= r0 < r1 <= nrow and non-NULL buffers");
        return 0;
    }
    int64_t row_bytes;
    if (type == B2S_TYPE_I2_S) {
        if (n_per_row % b2s::kQK != 0) {
            b2s::set_last_error(B2S_ERR_UNSUPPORTED,
                                "i2s_shard_rows: flattened i2_s rows are separable only when n_per_row % 128 == 0; "
                                "repack to I2_S_R first");
            return 0;
        }
        row_bytes = n_per_row / 4;
    } else if (type == B2S_TYPE_I2_S_R) {
        row_bytes = b2s::round_up(n_per_row, b2s::kQK) / 4;
    } else {
        b2s::set_last_error(B2S_ERR_UNSUPPORTED, "i2s_shard_rows: type must be I2_S or I2_S_R");
        return 0;
    }
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint8_t* d = static_cast<uint8_t*>(dst);
    const size_t body = (size_t)((r1 - r0) * row_bytes);
    memcpy(d, s + r0 * row_bytes, body);
    memcpy(d + body, s + nrow * row_bytes, 32);  // the 32-byte trailer holding the fp32 tensor scale
    return body + 32;
}

int b2s_peer_export(const void* dev_ptr, void* handle, size_t handle_bytes) {
    if (!dev_ptr || !handle || handle_bytes < B2S_PEER_HANDLE_BYTES)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "peer_export: need a device pointer and B2S_PEER_HANDLE_BYTES handle bytes");
    int rc = b2s_device_check();
    if (rc) return rc;
    GetRangeFn range = get_range_fn();
    if (!range) return b2s::set_last_error(B2S_ERR_CUDA, "peer_export: cuMemGetAddressRange is not available");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS || base == 0)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "peer_export: not a device allocation of this context");
    cudaIpcMemHandle_t h;
    rc = cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
    if (rc) return rc;
    const uint64_t off = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
    memcpy(handle, &h, sizeof(h));
    memcpy(static_cast<uint8_t*>(handle) + sizeof(h), &off, sizeof(off));
    return B2S_OK;
}

int b2s_peer_open(const void* handle, size_t handle_bytes, void** dev_ptr) {
    if (!handle || !dev_ptr || handle_bytes < B2S_PEER_HANDLE_BYTES)
        return b2s::set_last_error(B2S_ERR_INVALID_ARG, "peer_open: need B2S_PEER_HANDLE_BYTES handle bytes and an output pointer");
    *dev_ptr = nullptr;
    int rc = b2s_device_check();
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    uint64_t off = 0;
    memcpy(&h, handle, sizeof(h));
    memcpy(&off, static_cast<const uint8_t*>(handle) + sizeof(h), sizeof(off));
    void* p = nullptr;
    rc = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    if (rc) return rc;
    void* user = static_cast<uint8_t*>(p) + off;
    {
        std::lock_guard<std::mutex> lk(g_open_mu);
        g_open_base[user] = p;
    }
    *dev_ptr = user;
    return B2S_OK;
}

int b2s_peer_close(void* dev_ptr) {
    if (!dev_ptr) return b2s::set_last_error(B2S_ERR_INVALID_ARG, "peer_close: NULL pointer");
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_open_mu);
        auto it = g_open_base.find(dev_ptr);
        if (it == g_open_base.end())
            return b2s::set_last_error(B2S_ERR_INVALID_ARG, "peer_close: pointer was not returned by b2s_peer_open");
        base = it->second;
        g_open_base.erase(it);
    }
    return cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
}

}  // extern "C"
