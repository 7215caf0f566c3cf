// GPU k-means engine: nearest-centroid assignment, k-means++ and the two k-means
// loops of the reference (KmeansElkan::cluster and the Lloyd kmeans_cluster), on
// device-resident data.  Used by IvfPqIndex::train and by the vesper_kmeans_* C entry
// points.
#pragma once

#include <cstddef>
#include <cstdint>
#include <random>
#include <vector>

#include "common.cuh"
#include "kernels_tc.cuh"
#include "kernels_train.cuh"

namespace vgpu {

// Nearest-centroid search runs on the tensor cores (tcgen05 screen + exact refine)
// unless the shapes or the pointer alignment rule it out, or VGPU_COARSE=exact asks
// for the CUDA-core kernels; both give the same (exact) result.
bool use_tensor_cores(const float* x, const float* c, int d, uint32_t k);

// Whether the tensor-core nearest-centroid search screens every (row, centroid) pair
// into a distance matrix (VGPU_NEAREST=screen) instead of the sampled-threshold filter.
bool screen_all_columns();

// Whether k-means++ for n points and k centroids draws on the device (see kmeans_gpu.cpp).
bool kmeanspp_on_device(size_t n, uint32_t k);

// The draws of kmeans_plusplus_init (src/index/kmeans.cpp:45-89) on the host: the
// reference's std::mt19937(seed), uniform_int_distribution<size_t> for the first row,
// then per further centroid an fp64 running prefix sum of the D^2 vector in point
// order, one uniform_real_distribution<double>(0, total) draw and lower_bound.
class KmeansPPSampler {
public:
    KmeansPPSampler(uint32_t seed, size_t n);
    size_t first() const { return first_; }
    // d2: the current D^2 value of every point (host, n floats, point order).
    size_t next(const float* d2);

private:
    std::mt19937 gen_;
    size_t n_, first_;
    std::vector<double> cum_;
};

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
    // The same draws with the D^2 prefix sums and the lower_bound on the device.
    void kmeanspp_device(const float* d_x, size_t n, int d, uint32_t k, uint32_t seed, float* d_c);

    // KmeansElkan::cluster (src/index/kmeans_elkan.cpp:293-430) when elkan, else the
    // Lloyd loop of kmeans_cluster (src/index/kmeans.cpp:137-252, one run).
    KmeansResultGpu fit(const float* d_x, size_t n, int d, uint32_t k, uint32_t max_iter, float eps, uint32_t seed,
                        bool elkan, float* d_c, uint32_t* d_assign);

    // Sum of a device float array in index order, in fp64.
    double ordered_sum(const float* d, size_t n);

    // One shard's part of the M-step (launch_segment_accumulate): the points of x
    // [n x d] grouped by d_assign, sums continued from (sum, comp), sizes added to count.
    void accumulate(const float* d_x, size_t n, int d, const uint32_t* d_assign, uint32_t k, bool kahan,
                    double* sum, double* comp, unsigned long long* count);
    void finish_means(const double* sum, const unsigned long long* count, uint32_t k, int d, bool kahan,
                      float* d_c);
    void pp_update(const float* d_x, size_t n, int d, const float* d_crow, float* d_mind);
    // *total (host) continued by kmeans_cluster's final float running inertia over the
    // points of x in order (launch_ordered_sq_sum).
    void running_inertia(const float* d_x, size_t n, int d, const float* d_c, const uint32_t* d_assign, float* total);
    void sync();
    // Rows the last fused arg-min left to the filter path (candidate-list overflow).
    uint32_t last_overflow() const { return last_overflow_; }

private:
    cudaStream_t st_;
    DeviceBuffer<float> D_, xn_, cn_, cs_, cmax_, mind_, kpp_, ox_, oval_, caug_;
    DeviceBuffer<uint32_t> over_, oidx_, okeep_;
    uint32_t last_overflow_ = 0;
    DeviceBuffer<double> kpp_bsum_, kpp_u_;
    DeviceBuffer<int> err_;
    DeviceBuffer<uint32_t> order_, seg_, keep_;
    GroupWork gw_;
    FlatWork flat_;
    void* pin_ = nullptr;
    size_t pin_bytes_ = 0;
    float* pinned(size_t n);
};

}  // namespace vgpu
