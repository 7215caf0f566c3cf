// Merge of per-shard top-k results for a database split across GPUs.
//
// Every shard returns, per query, up to k (id, distance) pairs sorted by distance, with
// the reference's padding past its count (vesper_c_api.cpp:243-253: id 0, the last real
// distance).  After an all-gather the parts sit side by side in one buffer; one thread
// per query walks the parts' sorted heads and keeps the k smallest, ties to the lower
// part and then the earlier slot -- the order a stable sort of the concatenation in part
// order gives -- and pads the same way.  No global memory beyond inputs and outputs.
#include "kernels.cuh"

namespace vgpu {

namespace {
constexpr int kMergeMaxParts = 64;

__global__ void __launch_bounds__(128) topk_merge_kernel(int parts, long long nq, int k,
                                                         const float* __restrict__ dist, long long dist_stride,
                                                         const uint64_t* __restrict__ ids, long long ids_stride,
                                                         const uint32_t* __restrict__ counts,
                                                         long long counts_stride, uint64_t* __restrict__ out_ids,
                                                         float* __restrict__ out_d, uint32_t* __restrict__ out_n) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq;
         q += (long long)gridDim.x * blockDim.x) {
        int head[kMergeMaxParts], lim[kMergeMaxParts];
        for (int p = 0; p < parts; ++p) {
            head[p] = 0;
            const uint32_t c = counts[p * counts_stride + q];
            lim[p] = c < (uint32_t)k ? (int)c : k;
        }
        int i = 0;
        float last = 0.0f;
        for (; i < k; ++i) {
            int best = -1;
            float bv = 0.0f;
            for (int p = 0; p < parts; ++p) {
                if (head[p] >= lim[p]) continue;
                const float v = dist[p * dist_stride + q * k + head[p]];
                if (best < 0 || v < bv) { best = p; bv = v; }
            }
            if (best < 0) break;
            out_ids[q * k + i] = ids[best * ids_stride + q * k + head[best]];
            out_d[q * k + i] = bv;
            last = bv;
            ++head[best];
        }
        if (out_n) out_n[q] = (uint32_t)i;
        for (int j = i; j < k; ++j) {
            out_ids[q * k + j] = 0;
            out_d[q * k + j] = last;
        }
    }
}
}  // namespace

void launch_topk_merge(int parts, long long nq, int k, const float* dist, long long dist_stride, const uint64_t* ids,
                       long long ids_stride, const uint32_t* counts, long long counts_stride, uint64_t* out_ids,
                       float* out_d, uint32_t* out_n, cudaStream_t st) {
    if (nq <= 0 || k <= 0) return;
    if (parts < 1 || parts > kMergeMaxParts) throw CudaError("topk_merge: between 1 and 64 parts");
    const int blocks = (int)std::min<long long>((nq + 127) / 128, 148LL * 16);
    topk_merge_kernel<<<blocks, 128, 0, st>>>(parts, nq, k, dist, dist_stride, ids, ids_stride, counts, counts_stride,
                                              out_ids, out_d, out_n);
    VGPU_LAUNCH("topk_merge_kernel");
}

}  // namespace vgpu
