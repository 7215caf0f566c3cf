// Scratch memory for the allocation-free search entry point
// (vesper_ivfpq_search_batch_device_noalloc).
//
// Some callers cannot let a library call cudaMalloc/cudaFree: applications that hand
// all device memory to their own arena or to a framework's caching allocator (so a
// fresh allocation may fail or fragment their pool), and latency-critical serving
// loops where an allocation -- which can synchronize the whole device -- is not
// acceptable.  For them the search's temporary buffers (query-centroid distance rows,
// probe lists, rotated queries, per-query lookup tables) live in one file-scope device
// array of fixed size instead of being allocated.
//
// Properties of the array, as a user of this library should know them:
//   * Size: kNoAllocScratchBytes (64 MiB).  Every GPU on which the library's code is
//     loaded holds it until the process exits.
//   * In host code `g_noalloc_scratch` names a host-side stand-in, not a device
//     address; a kernel must never be handed it.  Its device address is looked up
//     once per device with cudaGetSymbolAddress (with that device current) by the
//     first allocation-free call on that device, and cached.  Make that first call
//     before any stream capture.  The cached address belongs to the device's primary
//     context: once cudaDeviceReset has destroyed that context, the entry point must
//     not be called again on the device in the same process.
//   * Every call on a device shares the array and it keeps the last call's contents.
//     Nothing in it has to start at zero: every byte a call reads is written earlier
//     in the same call.  Calls that overlapped on the GPU would race on it, so the
//     entry point holds a process-wide lock until its GPU work has finished.
#include <mutex>

#include "common.cuh"
#include "noalloc_search.hpp"

namespace vgpu {

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_addr_mu;
void* g_addr[256] = {};
std::mutex g_call_mu;
}  // namespace

void* noalloc_scratch_device_address(int device) {
    if (device < 0 || device >= 256) throw CudaError("noalloc scratch: device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_addr_mu);
    if (!g_addr[device]) {
        int cur = -1;
        check(cudaGetDevice(&cur), "cudaGetDevice");
        if (cur != device) throw CudaError("noalloc scratch: the device must be current when its address is looked up");
        void* p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (rc != cudaSuccess || p == nullptr)
            throw CudaError(std::string("cudaGetSymbolAddress(noalloc scratch): ") + cudaGetErrorString(rc));
        g_addr[device] = p;
    }
    return g_addr[device];
}

std::mutex& noalloc_call_mutex() { return g_call_mu; }

}  // namespace vgpu
