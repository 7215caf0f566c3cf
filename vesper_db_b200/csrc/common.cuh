// Shared CUDA helpers for the B200 IVF-PQ engine: error handling, device buffers,
// and the reference-order distance arithmetic used by every exact kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace vgpu {

struct CudaError : std::runtime_error {
    explicit CudaError(const std::string& s) : std::runtime_error(s) {}
};

inline void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}
#define VGPU_CHECK(x) ::vgpu::check((x), #x)
// Kernels this host thread has launched (every launch site of the library ends with
// VGPU_LAUNCH, which counts it); a search reports the difference across the call.
// Library kernels queued by CUB's device-wide scans and sorts are not counted.
inline unsigned long long& thread_launches() {
    static thread_local unsigned long long n = 0;
    return n;
}
#define VGPU_LAUNCH(what) (++::vgpu::thread_launches(), ::vgpu::check(cudaGetLastError(), what))

// Owning device allocation (cudaMalloc/cudaFree), movable, never copied.
template <class T>
class DeviceBuffer {
public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(size_t n) { resize(n); }
    ~DeviceBuffer() { release(); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept {
        if (this != &o) { release(); p_ = o.p_; n_ = o.n_; o.p_ = nullptr; o.n_ = 0; }
        return *this;
    }
    void resize(size_t n) {
        if (n == n_) return;
        release();
        if (n) VGPU_CHECK(cudaMalloc(&p_, n * sizeof(T)));
        n_ = n;
    }
    // Grow-only: keeps the allocation when it is already large enough.
    void reserve(size_t n) { if (n > n_) resize(n); }
    void release() {
        if (p_) cudaFree(p_);
        p_ = nullptr; n_ = 0;
    }
    T* data() const { return p_; }
    size_t size() const { return n_; }
    size_t bytes() const { return n_ * sizeof(T); }

private:
    T* p_ = nullptr;
    size_t n_ = 0;
};

#ifdef __CUDACC__
// ---------------------------------------------------------------------------------
// Reference-order arithmetic (device side).
//
// The reference computes every squared L2 distance with its AVX2 kernel
// (include/vesper/kernels/backends/avx2.hpp:76-108): eight lane accumulators, lane l
// holding fma(a_i - b_i, a_i - b_i, acc_l) for i = l (mod 8) below floor(n/8)*8; then
// hsum_ps (:37-46) = ((acc0+acc4) + (acc1+acc5)) + ((acc2+acc6) + (acc3+acc7)); then a
// scalar tail `result += d*d` with a rounded product and a rounded add.  The __f*_rn
// intrinsics below stop nvcc from contracting any of those steps into other FMAs.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float hsum8(const float acc[8]) {
    const float s0 = __fadd_rn(acc[4], acc[0]);
    const float s1 = __fadd_rn(acc[5], acc[1]);
    const float s2 = __fadd_rn(acc[6], acc[2]);
    const float s3 = __fadd_rn(acc[7], acc[3]);
    return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// Squared L2 over n floats in reference order.  Generic n (any length, any alignment).
__device__ __forceinline__ float l2_ref(const float* a, const float* b, int n) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
    const int simd_end = n & ~7;
    int i = 0;
    for (; i < simd_end; i += 8) {
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float d = __fsub_rn(a[i + l], b[i + l]);
            acc[l] = __fmaf_rn(d, d, acc[l]);
        }
    }
    float r = hsum8(acc);
    for (; i < n; ++i) {
        const float d = __fsub_rn(a[i], b[i]);
        r = __fadd_rn(r, __fmul_rn(d, d));
    }
    return r;
}

// Inner product in reference order (avx2_inner_product, avx2.hpp:124-154).
__device__ __forceinline__ float ip_ref(const float* a, const float* b, int n) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
    const int simd_end = n & ~7;
    int i = 0;
    for (; i < simd_end; i += 8) {
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[l] = __fmaf_rn(a[i + l], b[i + l], acc[l]);
    }
    float r = hsum8(acc);
    for (; i < n; ++i) r = __fadd_rn(r, __fmul_rn(a[i], b[i]));
    return r;
}

// Order-preserving map from float to uint32 (total order, -0 < +0, NaN last).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

#endif  // __CUDACC__

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

}  // namespace vgpu
