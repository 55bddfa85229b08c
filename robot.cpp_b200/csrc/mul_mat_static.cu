// mul_mat_static.cu -- b2s_mul_mat_static: the MUL_MAT node without any caller workspace.
//
// Who needs it: callers that hold no device workspace and may not allocate while they run. A ggml
// backend executes a graph after its scheduler has sized and allocated every buffer, and an op there
// gets no allocator; a robot control loop that has finished start-up must not call cudaMalloc, which
// can synchronize the whole device and adds latency jitter to every control period. For them the int8
// activations, per-token scales and sums that b2s_mul_mat keeps in the caller's workspace live here in
// one file-scope device array instead.
//
// Rules of this entry point:
//   * Capacity: kStaticScratchBytes (4 MiB) per device, held by every GPU that loads the library until the
//     process exits. The call's scratch need is its activation layout: a256(M * roundup(K,16)) bytes of
//     int8 codes + a256(4*M) of scales + a256(4*M) of sums (a256 = rounded up to 256 bytes), e.g. M <= 300
//     tokens at K = 6912 or M <= 1600 at K = 2560. A call that needs more returns B2S_ERR_WORKSPACE with a
//     message and launches nothing. Whatever the activations leave free holds split-K partials, as the
//     workspace of b2s_mul_mat does, so both entry points pick the same kernels.
//   * Nothing here allocates: no cudaMalloc, no cudaFree, no allocating library routine.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that
//     device current) and caches it for the life of the process; make that first call before any stream
//     capture begins, and do not reset the device (cudaDeviceReset) after it: a new context reloads the
//     module and the cached address would no longer name this array.
//   * Every call on a device shares the one array, and the array keeps the previous call's contents.
//     Calls whose work overlaps on the GPU (other streams, other host threads) race on it: serialize
//     them, e.g. on one stream. Nothing in the array needs to start at zero: each call writes every
//     byte it later reads (the codes of all K columns of its M rows, their scales and sums).
#include <cstdio>
#include <mutex>

#include "b2s.h"
#include "b2s_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

void* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_static_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return b2s::set_last_error(B2S_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return b2s::set_last_error(B2S_ERR_DEVICE, "device index out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p) {
            (void)cudaGetLastError();
            return b2s::set_last_error(B2S_ERR_CUDA, "cudaGetSymbolAddress of the static scratch array failed");
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return B2S_OK;
}

}  // namespace

extern "C" int b2s_mul_mat_static(const b2s_tensor* W, const b2s_tensor* X, b2s_tensor* Y, void* stream) {
    int rc = b2s_device_check();
    if (rc) return rc;
    size_t need = 0;
    if ((rc = b2s::mul_mat_scratch_bytes(W, X, &need))) return rc;  // the status b2s_mul_mat gives
    if (need > kStaticScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof(msg),
                 "b2s_mul_mat_static: this call needs %zu scratch bytes, above the %zu-byte static limit; "
                 "use b2s_mul_mat with a workspace",
                 need, kStaticScratchBytes);
        return b2s::set_last_error(B2S_ERR_WORKSPACE, msg);
    }
    void* scratch = nullptr;
    if ((rc = scratch_address(&scratch))) return rc;
    return b2s::mul_mat_into_scratch(W, X, Y, scratch, kStaticScratchBytes, static_cast<cudaStream_t>(stream));
}
