// The inverted-list section of the reference's index files (src/index/ivf_pq.cpp:4393-4404,
// 4466-4478): [lists_count u32] then per list [size u64][size x (id u64, m code bytes)],
// little-endian, unaligned.  These kernels convert between that byte stream (in device
// memory) and the index's CSR arrays, so a load uploads the section once and a save
// downloads it once, instead of copying entry by entry on the host.
#include "kernels.cuh"

namespace vgpu {

// One CTA per list; list_byte[l] = offset of list l's size field in `raw`.  Bytes are
// moved one per thread so that no access depends on the stream's alignment.
__global__ void unpack_lists_kernel(const uint8_t* __restrict__ raw, const uint64_t* __restrict__ list_byte,
                                    const uint64_t* __restrict__ offs, int m, uint64_t* __restrict__ ids,
                                    uint8_t* __restrict__ codes) {
    const int l = blockIdx.x;
    const uint64_t e0 = offs[l], n = offs[l + 1] - e0;
    const uint8_t* src = raw + list_byte[l] + 8;
    const uint64_t rec = 8 + (uint64_t)m;
    const uint64_t total = n * rec;
    for (uint64_t t = threadIdx.x; t < total; t += blockDim.x) {
        const uint64_t i = t / rec, b = t % rec;
        const uint8_t v = src[t];
        if (b < 8) reinterpret_cast<uint8_t*>(ids + e0 + i)[b] = v;
        else codes[(e0 + i) * m + (b - 8)] = v;
    }
}

__global__ void pack_lists_kernel(const uint64_t* __restrict__ ids, const uint8_t* __restrict__ codes,
                                  const uint64_t* __restrict__ offs, int m, const uint64_t* __restrict__ list_byte,
                                  uint8_t* __restrict__ raw) {
    const int l = blockIdx.x;
    const uint64_t e0 = offs[l], n = offs[l + 1] - e0;
    uint8_t* dst = raw + list_byte[l];
    if (threadIdx.x < 8) dst[threadIdx.x] = reinterpret_cast<const uint8_t*>(&n)[threadIdx.x];
    dst += 8;
    const uint64_t rec = 8 + (uint64_t)m;
    const uint64_t total = n * rec;
    for (uint64_t t = threadIdx.x; t < total; t += blockDim.x) {
        const uint64_t i = t / rec, b = t % rec;
        dst[t] = b < 8 ? reinterpret_cast<const uint8_t*>(ids + e0 + i)[b] : codes[(e0 + i) * m + (b - 8)];
    }
}

void launch_unpack_lists(const uint8_t* raw, const uint64_t* list_byte, const uint64_t* offs, int nlist, int m,
                         uint64_t* ids, uint8_t* codes, cudaStream_t st) {
    if (nlist <= 0) return;
    unpack_lists_kernel<<<nlist, 256, 0, st>>>(raw, list_byte, offs, m, ids, codes);
    VGPU_LAUNCH("unpack_lists_kernel");
}

void launch_pack_lists(const uint64_t* ids, const uint8_t* codes, const uint64_t* offs, int nlist, int m,
                       const uint64_t* list_byte, uint8_t* raw, cudaStream_t st) {
    if (nlist <= 0) return;
    pack_lists_kernel<<<nlist, 256, 0, st>>>(ids, codes, offs, m, list_byte, raw);
    VGPU_LAUNCH("pack_lists_kernel");
}

}  // namespace vgpu
