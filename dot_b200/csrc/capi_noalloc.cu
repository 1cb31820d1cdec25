// dot_sinkhorn_fwd_noalloc: the Sinkhorn forward for callers that cannot
// allocate device memory.  Its scratch space is a fixed file-scope device
// array instead of a caller-provided workspace.
#include <mutex>
#include <string>

#include "internal.h"

namespace {

// 16 MiB of scratch, held by every GPU that loads this library until the
// process exits.  Enough for e.g. B=256 x 512 x 512 or B=4096 x 128 x 128.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  The host-side
// name of the array is only a stand-in; the address is looked up once per
// device, with that device current, and cached for the life of the process
// (a primary context destroyed by cudaDeviceReset leaves the entry stale; the
// header tells callers not to use this entry point after one).
int scratch_on_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return dotb::fail(DOT_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return dotb::fail(DOT_ERR_UNSUPPORTED, "device index out of range");
    std::lock_guard<std::mutex> g(g_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return dotb::fail(DOT_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return DOT_OK;
}

}  // namespace

extern "C" int dot_sinkhorn_fwd_noalloc(const float* X, float score_sign, const float* log_a,
                                        const float* log_b, int64_t B, int64_t n, int64_t m, float tau,
                                        int n_iters, float tol, int out_mode, float* out, float* cost,
                                        float* pot_u, float* pot_v, int32_t* status, void* stream) {
    dotb::clear_error();
    if (B > 0 && n > 0 && m > 0) {
        const size_t need = dot_sinkhorn_fwd_workspace_bytes(B, n, m, n_iters, tol, cost != nullptr);
        if (need > kNoAllocScratchBytes)
            return dotb::fail(DOT_ERR_WORKSPACE,
                              "problem needs " + std::to_string(need) + " bytes of scratch; the no-allocation "
                              "entry point has a fixed 16 MiB (16777216 bytes); use dot_sinkhorn_fwd with a "
                              "caller-provided workspace");
    }
    void* scratch = nullptr;
    int rc = scratch_on_current_device(&scratch);
    if (rc != DOT_OK) return rc;
    return dot_sinkhorn_fwd(X, score_sign, log_a, log_b, B, n, m, tau, n_iters, tol, out_mode, out, cost, pot_u,
                            pot_v, status, scratch, kNoAllocScratchBytes, stream);
}
