// GPU k-means engine: nearest-centroid assignment, k-means++ and the two k-means
// loops of the reference (KmeansElkan::cluster and the Lloyd kmeans_cluster), on
// device-resident data.  Used by IvfPqIndex::train and by the vesper_kmeans_* C entry
// points.
#pragma once

#include <cstddef>
#include <cstdint>

#include "common.cuh"
#include "kernels_train.cuh"

namespace vgpu {

// Nearest-centroid search runs on the tensor cores (tcgen05 screen + exact refine)
// unless the shapes or the pointer alignment rule it out, or VGPU_COARSE=exact asks
// for the CUDA-core kernels; both give the same (exact) result.
bool use_tensor_cores(const float* x, const float* c, int d, uint32_t k);

struct KmeansResultGpu {
    uint32_t iterations = 0;
    float inertia = 0.0f;
};

class KmeansEngine {
public:
    explicit KmeansEngine(cudaStream_t st) : st_(st) {}
    KmeansEngine(const KmeansEngine&) = delete;
    KmeansEngine& operator=(const KmeansEngine&) = delete;
    ~KmeansEngine();

    // Exact nearest centroid of each row of x [n x d] among c [k x d] (reference lane
    // order, lowest index on ties; keep -> the current assignment wins a tie).  Uses
    // the tensor-core screen + exact refine when the shapes allow it.  d_mind may be null.
    void assign(const float* d_x, size_t n, int d, const float* d_c, uint32_t k, uint32_t* d_assign, float* d_mind,
                bool keep);

    // kmeans_plusplus_init (src/index/kmeans.cpp:45-89): k rows of x copied into d_c.
    void kmeanspp(const float* d_x, size_t n, int d, uint32_t k, uint32_t seed, float* d_c);

    // KmeansElkan::cluster (src/index/kmeans_elkan.cpp:293-430) when elkan, else the
    // Lloyd loop of kmeans_cluster (src/index/kmeans.cpp:137-252, one run).
    KmeansResultGpu fit(const float* d_x, size_t n, int d, uint32_t k, uint32_t max_iter, float eps, uint32_t seed,
                        bool elkan, float* d_c, uint32_t* d_assign);

    // Sum of a device float array in index order, in fp64.
    double ordered_sum(const float* d, size_t n);

private:
    cudaStream_t st_;
    DeviceBuffer<float> D_, xn_, cn_, mind_, kpp_;
    DeviceBuffer<int> err_;
    DeviceBuffer<uint32_t> order_, seg_;
    GroupWork gw_;
    void* pin_ = nullptr;
    size_t pin_bytes_ = 0;
    float* pinned(size_t n);
};

}  // namespace vgpu
