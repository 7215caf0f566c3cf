// Fixed device scratch for the allocation-free search entry point
// (definitions and the rules for its use in noalloc_search.cu).
#pragma once

#include <cstddef>
#include <mutex>

namespace vgpu {

// Size of the file-scope device array every allocation-free call uses.
constexpr std::size_t kNoAllocScratchBytes = std::size_t(64) << 20;

// Device address of the array on `device`, which must be the current device.  The
// first call per device performs the lookup (cudaGetSymbolAddress) and caches it;
// throws CudaError when the lookup fails.
void* noalloc_scratch_device_address(int device);

// Held for the whole of each allocation-free call, so calls never overlap on the GPU.
std::mutex& noalloc_call_mutex();

}  // namespace vgpu
