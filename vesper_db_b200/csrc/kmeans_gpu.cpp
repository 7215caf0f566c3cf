// GPU k-means engine (see kmeans_gpu.hpp).
#include "kmeans_gpu.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <limits>
#include <random>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "kernels_tc.cuh"

namespace vgpu {

namespace {
constexpr size_t kDistBudget = size_t(512) << 20;  // bytes per distance-matrix chunk
}  // namespace

bool use_tensor_cores(const float* x, const float* c, int d, uint32_t k) {
    static const bool off = [] {
        const char* v = std::getenv("VGPU_COARSE");
        return v && std::string(v) == "exact";
    }();
    return !off && k >= 64 && tc_screen_supported(d) &&
           ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(c)) & 15) == 0;
}

// VGPU_NEAREST=screen: the one-pass screen of every (row, centroid) pair plus
// screen_select (the distance matrix in 512 MiB chunks) instead of the filter path.
bool screen_all_columns() {
    static const bool on = [] {
        const char* v = std::getenv("VGPU_NEAREST");
        return v && std::string(v) == "screen";
    }();
    return on;
}

KmeansEngine::~KmeansEngine() {
    if (pin_) cudaFreeHost(pin_);
}

float* KmeansEngine::pinned(size_t n) {
    if (n * sizeof(float) > pin_bytes_) {
        if (pin_) cudaFreeHost(pin_);
        check(cudaMallocHost(&pin_, n * sizeof(float)), "cudaMallocHost");
        pin_bytes_ = n * sizeof(float);
    }
    return static_cast<float*>(pin_);
}

double KmeansEngine::ordered_sum(const float* d, size_t n) {
    float* h = pinned(n);
    check(cudaMemcpyAsync(h, d, n * sizeof(float), cudaMemcpyDeviceToHost, st_), "d2h");
    check(cudaStreamSynchronize(st_), "sync");
    double t = 0.0;
    for (size_t i = 0; i < n; ++i) t += h[i];
    return t;
}

void KmeansEngine::assign(const float* d_x, size_t n, int d, const float* d_c, uint32_t k, uint32_t* d_assign,
                          float* d_mind, bool keep) {
    const bool tc = use_tensor_cores(d_x, d_c, d, k);
    if (tc && !screen_all_columns()) {
        // Fused arg-min on the tensor cores (tc_argmin_kernel): no n x k matrix of
        // screen values; rows whose candidate list overflowed are redone through the
        // sampled-threshold filter path (launch_exact_nearest).
        if (!d_mind) {
            mind_.reserve(n);
            d_mind = mind_.data();
        }
        const uint32_t* kp = nullptr;
        if (keep) {
            keep_.reserve(n);
            check(cudaMemcpyAsync(keep_.data(), d_assign, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st_), "d2d");
            kp = keep_.data();
        }
        xn_.reserve(n);
        cn_.reserve(k);
        cs_.reserve(k);
        cmax_.reserve(2);
        err_.reserve(1);
        over_.reserve(n + 1);
        launch_row_norms(d_x, (long long)n, d, xn_.data(), st_);
        launch_row_norms(d_c, k, d, cn_.data(), st_);
        launch_sqrt(cn_.data(), k, cs_.data(), st_);
        launch_col_max(cn_.data(), cs_.data(), (int)k, cmax_.data(), st_);
        check(cudaMemsetAsync(err_.data(), 0, sizeof(int), st_), "memset err");
        check(cudaMemsetAsync(over_.data() + n, 0, sizeof(uint32_t), st_), "memset over");
        caug_.reserve((size_t)k * (size_t)aug_ld(d));
        launch_tc_argmin(d_x, (long long)n, d_c, (int)k, d, xn_.data(), cn_.data(), cs_.data(), cmax_.data(), kp,
                         d_assign, d_mind, over_.data(), over_.data() + n, caug_.data(), err_.data(), st_);
        int h[2] = {0, 0};
        check(cudaMemcpyAsync(&h[0], err_.data(), sizeof(int), cudaMemcpyDeviceToHost, st_), "d2h err");
        check(cudaMemcpyAsync(&h[1], over_.data() + n, sizeof(uint32_t), cudaMemcpyDeviceToHost, st_), "d2h over");
        check(cudaStreamSynchronize(st_), "sync");
        if (h[0]) throw CudaError("tensor-core arg-min: bounded wait expired (code " + std::to_string(h[0]) + ")");
        last_overflow_ = (uint32_t)h[1];
        if (h[1]) {
            const size_t no = (size_t)(uint32_t)h[1];
            ox_.reserve(no * d);
            oidx_.reserve(no);
            oval_.reserve(no);
            launch_gather_rows(d_x, d, over_.data(), (long long)no, ox_.data(), st_);
            const uint32_t* okp = nullptr;
            if (keep) {
                okeep_.reserve(no);
                launch_gather_u32(kp, over_.data(), (long long)no, okeep_.data(), st_);
                okp = okeep_.data();
            }
            launch_exact_nearest(ox_.data(), (long long)no, d_c, k, d, 1, okp, oidx_.data(), oval_.data(), flat_, st_);
            launch_scatter_top1(over_.data(), (int)no, oidx_.data(), oval_.data(), d_assign, d_mind, st_);
            check(cudaStreamSynchronize(st_), "sync");
        }
        return;
    }
    const size_t rows = std::max<size_t>(1, std::min<size_t>(n, kDistBudget / (sizeof(float) * k)));
    D_.reserve(rows * k);
    if (tc) {
        cn_.reserve(k);
        xn_.reserve(rows);
        err_.reserve(1);
        launch_row_norms(d_c, k, d, cn_.data(), st_);
        check(cudaMemsetAsync(err_.data(), 0, sizeof(int), st_), "memset err");
    }
    for (size_t r0 = 0; r0 < n; r0 += rows) {
        const size_t nr = std::min(rows, n - r0);
        const float* xr = d_x + r0 * (size_t)d;
        if (tc) {
            launch_row_norms(xr, (long long)nr, d, xn_.data(), st_);
            launch_tc_screen(xr, (long long)nr, d_c, (int)k, d, xn_.data(), cn_.data(), D_.data(), (long long)k,
                             err_.data(), st_);
            launch_screen_select(D_.data(), (long long)nr, (long long)k, (int)k, xr, d, d_c, xn_.data(), cn_.data(), 1,
                                 keep ? d_assign + r0 : nullptr, d_assign + r0, d_mind ? d_mind + r0 : nullptr,
                                 err_.data(), st_);
        } else {
            launch_l2_dist(xr, (long long)nr, d_c, (int)k, d, D_.data(), (long long)k, st_);
            launch_row_argmin(D_.data(), (long long)nr, (int)k, (long long)k, keep ? d_assign + r0 : nullptr,
                              d_assign + r0, d_mind ? d_mind + r0 : nullptr, st_);
        }
    }
    if (tc) {
        int e = 0;
        check(cudaMemcpyAsync(&e, err_.data(), sizeof(int), cudaMemcpyDeviceToHost, st_), "d2h err");
        check(cudaStreamSynchronize(st_), "sync");
        if (e) throw CudaError("tensor-core screen: bounded wait expired (code " + std::to_string(e) + ")");
    }
}

KmeansPPSampler::KmeansPPSampler(uint32_t seed, size_t n) : gen_(seed), n_(n), cum_(n) {
    std::uniform_int_distribution<size_t> first(0, n - 1);
    first_ = first(gen_);
}

size_t KmeansPPSampler::next(const float* d2) {
    cum_[0] = d2[0];
    for (size_t i = 1; i < n_; ++i) cum_[i] = cum_[i - 1] + d2[i];
    std::uniform_real_distribution<double> sd(0.0, cum_.back());
    const double target = sd(gen_);
    return (size_t)(std::lower_bound(cum_.begin(), cum_.end(), target) - cum_.begin());
}

// Where the draws run.  Host: the D^2 vector is copied back for every draw and the
// reference's prefix sum is recomputed in point order (KmeansPPSampler), O(n) host work
// per centroid.  Device: the same mt19937 stream (generate_canonical values drawn
// ahead) and the same D^2 values, with the prefix sums formed per block on the GPU
// (launch_kpp_update_sum / launch_kpp_pick).  Device from n * k >= 2^30 (where the
// host loop takes many seconds); VGPU_KPP=host|device forces either.
bool kmeanspp_on_device(size_t n, uint32_t k) {
    if (const char* v = std::getenv("VGPU_KPP")) {
        if (std::string(v) == "host") return false;
        if (std::string(v) == "device") return true;
    }
    return (double)n * (double)k >= 1073741824.0;
}

void KmeansEngine::kmeanspp_device(const float* d_x, size_t n, int d, uint32_t k, uint32_t seed, float* d_c) {
    std::mt19937 gen(seed);
    std::uniform_int_distribution<size_t> first(0, n - 1);
    const size_t idx = first(gen);
    std::vector<double> u(std::max<uint32_t>(k, 1), 0.0);
    for (uint32_t c = 1; c < k; ++c) u[c] = std::generate_canonical<double, std::numeric_limits<double>::digits>(gen);
    kpp_u_.reserve(u.size());
    check(cudaMemcpyAsync(kpp_u_.data(), u.data(), u.size() * sizeof(double), cudaMemcpyHostToDevice, st_), "h2d");
    check(cudaMemcpyAsync(d_c, d_x + idx * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, st_), "d2d");
    kpp_.reserve(n);
    kpp_bsum_.reserve((size_t)kpp_blocks((long long)n));
    launch_fill(kpp_.data(), (long long)n, std::numeric_limits<float>::max(), st_);
    for (uint32_t c = 1; c < k; ++c) {
        launch_kpp_update_sum(d_x, (long long)n, d, d_c + (size_t)(c - 1) * d, kpp_.data(), kpp_bsum_.data(), st_);
        launch_kpp_pick(d_x, (long long)n, d, kpp_.data(), kpp_bsum_.data(), kpp_u_.data(), (int)c, d_c, st_);
    }
    // u must outlive the copy
    check(cudaStreamSynchronize(st_), "sync");
}

// kmeans_plusplus_init: the D^2 vector comes from the GPU; the draws run on the host
// (KmeansPPSampler) or, for large n * k, on the device (kmeanspp_device).
void KmeansEngine::kmeanspp(const float* d_x, size_t n, int d, uint32_t k, uint32_t seed, float* d_c) {
    if (kmeanspp_on_device(n, k)) {
        kmeanspp_device(d_x, n, d, k, seed, d_c);
        return;
    }
    KmeansPPSampler sampler(seed, n);
    size_t idx = sampler.first();
    check(cudaMemcpyAsync(d_c, d_x + idx * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, st_), "d2d");
    kpp_.reserve(n);
    launch_fill(kpp_.data(), (long long)n, std::numeric_limits<float>::max(), st_);
    float* h = pinned(n);
    for (uint32_t c = 1; c < k; ++c) {
        launch_kpp_update(d_x, (long long)n, d, d_c + (size_t)(c - 1) * d, kpp_.data(), st_);
        check(cudaMemcpyAsync(h, kpp_.data(), n * sizeof(float), cudaMemcpyDeviceToHost, st_), "d2h");
        check(cudaStreamSynchronize(st_), "sync");
        idx = sampler.next(h);
        check(cudaMemcpyAsync(d_c + (size_t)c * d, d_x + idx * d, sizeof(float) * d, cudaMemcpyDeviceToDevice, st_),
              "d2d");
    }
}

void KmeansEngine::accumulate(const float* d_x, size_t n, int d, const uint32_t* d_assign, uint32_t k, bool kahan,
                              double* sum, double* comp, unsigned long long* count) {
    if (n == 0) return;
    order_.reserve(n);
    seg_.reserve(k + 1);
    group_by_key(d_assign, (long long)n, (int)k, order_.data(), seg_.data(), gw_, st_);
    launch_segment_accumulate(d_x, d, order_.data(), seg_.data(), (int)k, kahan ? 1 : 0, sum, comp, count, st_);
}

void KmeansEngine::finish_means(const double* sum, const unsigned long long* count, uint32_t k, int d, bool kahan,
                                float* d_c) {
    launch_finish_means(sum, count, (int)k, d, kahan ? 1 : 0, d_c, st_);
}

void KmeansEngine::pp_update(const float* d_x, size_t n, int d, const float* d_crow, float* d_mind) {
    launch_kpp_update(d_x, (long long)n, d, d_crow, d_mind, st_);
}

void KmeansEngine::running_inertia(const float* d_x, size_t n, int d, const float* d_c, const uint32_t* d_assign,
                                   float* total) {
    mind_.reserve(1);
    check(cudaMemcpyAsync(mind_.data(), total, sizeof(float), cudaMemcpyHostToDevice, st_), "h2d");
    launch_ordered_sq_sum(d_x, d_c, d_assign, (long long)n, d, mind_.data(), st_);
    check(cudaMemcpyAsync(total, mind_.data(), sizeof(float), cudaMemcpyDeviceToHost, st_), "d2h");
    check(cudaStreamSynchronize(st_), "sync");
}

void KmeansEngine::sync() { check(cudaStreamSynchronize(st_), "sync"); }

// Elkan (KmeansElkan::cluster): exact E-step with the keep-on-tie rule (Elkan prunes
// only provably farther centroids), convergence test on the fp64-summed inertia
// before the M-step, Kahan M-step in point order; returns the last converged-from
// inertia and the iteration count, as the reference does.
// Lloyd (kmeans_cluster): lowest-index E-step, the same test, fp64 sum / count
// M-step; after the loop one more M-step and the inertia of the final assignment as the
// reference's float running total over every term.
KmeansResultGpu KmeansEngine::fit(const float* d_x, size_t n, int d, uint32_t k, uint32_t max_iter, float eps,
                                  uint32_t seed, bool elkan, float* d_c, uint32_t* d_assign) {
    kmeanspp(d_x, n, d, k, seed, d_c);
    mind_.reserve(n);
    order_.reserve(n);
    seg_.reserve(k + 1);
    // The reference's assignment vector starts at 0 (std::vector<uint32_t>(n)); with
    // max_iter = 0 the final Lloyd update reads it as it is.
    check(cudaMemsetAsync(d_assign, 0, n * sizeof(uint32_t), st_), "memset assignments");
    if (elkan) assign(d_x, n, d, d_c, k, d_assign, mind_.data(), false);
    float prev = std::numeric_limits<float>::max();
    uint32_t it = 0;
    for (; it < max_iter; ++it) {
        if (!elkan || it > 0) assign(d_x, n, d, d_c, k, d_assign, mind_.data(), elkan);
        const float inertia = (float)ordered_sum(mind_.data(), n);
        const float change = std::fabs(prev - inertia) / (prev + 1e-10f);
        if (change < eps) break;
        prev = inertia;
        group_by_key(d_assign, (long long)n, (int)k, order_.data(), seg_.data(), gw_, st_);
        launch_segment_mean(d_x, d, order_.data(), seg_.data(), (int)k, elkan ? 1 : 0, d_c, st_);
    }
    KmeansResultGpu r;
    r.iterations = it;
    if (elkan) {
        r.inertia = prev;
    } else {
        group_by_key(d_assign, (long long)n, (int)k, order_.data(), seg_.data(), gw_, st_);
        launch_segment_mean(d_x, d, order_.data(), seg_.data(), (int)k, 0, d_c, st_);
        float total = 0.0f;
        running_inertia(d_x, n, d, d_c, d_assign, &total);
        r.inertia = total;
    }
    check(cudaStreamSynchronize(st_), "sync");
    return r;
}

}  // namespace vgpu
