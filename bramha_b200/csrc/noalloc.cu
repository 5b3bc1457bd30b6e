// noalloc.cu -- the fixed device scratch behind bramha_cuda_gemm_noalloc_dev.
//
// The prefill GEMM normally takes its scratch (per-token activation sums for
// the log4 correction) from the stream-ordered memory pool.  Callers that must
// not allocate device memory during a call use the allocation-free entry point
// instead, which works out of this fixed array.  Its size caps the number of
// tokens per call at kNoAllocMaxTokens (64 KiB of floats); every GPU that loads
// this library holds the array until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace bramha {

namespace {
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) float g_noalloc_rowsum[kNoAllocMaxTokens];

// Device address of g_noalloc_rowsum on the current device.  On the host the
// array's name only stands in for the symbol (a kernel handed that name would
// read the wrong memory or fault), so the real address is looked up with
// cudaGetSymbolAddress -- once per device, with that device current -- and
// cached.  The first call on a device therefore does this set-up.
cudaError_t noalloc_rowsum_scratch(int device, float** out) {
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    if (addr[device] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_rowsum);
        if (e != cudaSuccess) return e;
        addr[device] = static_cast<float*>(p);
    }
    *out = addr[device];
    return cudaSuccess;
}

}  // namespace bramha
