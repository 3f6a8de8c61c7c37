// noalloc.cu -- a forward entry point that allocates no device memory.
//
// Some callers cannot allocate device memory at the point where they run the attention
// forward: code that executes inside a custom allocator's or framework's memory-pressure
// callback, real-time / inference servers whose memory plan is fixed at start-up and
// forbid any cudaMalloc afterwards, and embedders whose host language has no binding to
// an allocator at all.  For them morpho_sm100_forward_noalloc keeps its scratch in a
// fixed device array that is part of this library, so the caller passes only the inputs
// and outputs.
//
// The scratch array (kNoAllocScratchBytes, 32 MiB) is a file-scope __device__ object: every
// GPU that loads it holds it until the process exits.  Its device address is looked up once
// per device with cudaGetSymbolAddress, the first time this entry point runs on that device
// (with that device current).  Under CUDA's lazy module loading (the default since CUDA
// 12.2; CUDA_MODULE_LOADING=EAGER turns it off) that first call is also the moment the
// array and the forward's kernel modules are placed on the device, so it does reserve
// device memory: make it at start-up, before the code that must not allocate runs, and
// outside any CUDA stream capture.  Later calls reserve nothing.  The cached address
// belongs to the device's current context; after cudaDeviceReset this entry point must
// not be called again in the same process.  All calls share the one array, so two calls
// whose work overlaps on the GPU (different streams, or different host threads without
// ordering) race on it; calls issued in order on one stream are safe.  The forward
// overwrites every scratch byte it later reads (the soft-morphology range flag is cleared
// by the forward itself), so nothing needs clearing between calls.
#include <mutex>

#include "host_common.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cudaGetLastError();  // do not leave the failure for the next launch check to report
        return morpho::set_error(MORPHO_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= kMaxDevices)
        return morpho::set_error(MORPHO_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            cudaGetLastError();  // as above: the error is returned here, not left pending
            return morpho::set_error(MORPHO_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s",
                                     cudaGetErrorString(e));
        }
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return MORPHO_OK;
}

}  // namespace

extern "C" {

size_t morpho_sm100_forward_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

int morpho_sm100_forward_noalloc(const morpho_problem_t* p, const void* X, const void* W_phi, const void* gate_q,
                                 const void* gate_k, const void* W_V, void* out, float* lse, void* stream) {
    const size_t need = morpho_sm100_forward_workspace_size(p);
    if (need == 0) return MORPHO_ERR_INVALID;  // message already set by the size query
    if (need > kNoAllocScratchBytes)
        return morpho::set_error(MORPHO_ERR_WORKSPACE,
                                 "morpho_sm100_forward_noalloc: this problem needs %zu bytes of scratch, more than the "
                                 "%zu bytes built into the library; call morpho_sm100_forward with a workspace instead",
                                 need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != MORPHO_OK) return rc;
    return morpho_sm100_forward(p, X, W_phi, gate_q, gate_k, W_V, out, lse, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
