// B200 kernels for k-means training (coarse quantizer and PQ sub-quantizers).
//
//   * kpp_update: the D^2 refresh of k-means++ (src/index/kmeans.cpp:61-67), one
//     reference-order distance per point.
//   * points are grouped by cluster with a stable sort (group_by_key in
//     train_kernels.cu), so the M-step sums points in the order the reference
//     gathers them (src/index/kmeans_elkan.cpp:354-356).
//   * segment_mean: the M-step as a segmented reduction.  One thread owns one
//     (cluster, dimension) pair and walks the cluster's points in order:
//       kahan = 1: Kahan-compensated fp64 sum times (1/count) (update_centroid,
//                  src/index/kmeans_elkan.cpp:31-56);
//       kahan = 0: plain fp64 sum divided by count (kmeans_update_centroids,
//                  src/index/kmeans.cpp:107-135).
//     Empty clusters keep their previous centroid in both.
#include <cfloat>

#include "kernels.cuh"

namespace vgpu {

__global__ void kpp_update_kernel(const float* __restrict__ x, long long n, int dim,
                                  const float* __restrict__ c, float* __restrict__ mind) {
    // One warp per point: lanes 0..7 hold the eight lane accumulators of a strided
    // walk; lane l accumulates elements l, l+8, l+16, ... in order, exactly as lane l
    // of the AVX2 kernel does.  Lanes 8..31 idle on the FMA chain (the chain length
    // is dim/8, so this stays memory-bound).
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    const int simd_end = dim & ~7;
    for (long long i = warp; i < n; i += nwarps) {
        const float* p = x + i * dim;
        float acc = 0.0f;
        if (lane < 8)
            for (int t = lane; t < simd_end; t += 8) {
                const float d = __fsub_rn(p[t], c[t]);
                acc = __fmaf_rn(d, d, acc);
            }
        // hsum8 over lanes 0..7: ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7))
        const float a4 = __shfl_down_sync(0xffffffffu, acc, 4);
        const float s = __fadd_rn(a4, acc);          // lanes 0..3: s_l = a_{l+4} + a_l
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1);
        const float s2 = __shfl_down_sync(0xffffffffu, s, 2);
        const float s3 = __shfl_down_sync(0xffffffffu, s, 3);
        if (lane == 0) {
            float r = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
            for (int t = simd_end; t < dim; ++t) {
                const float d = __fsub_rn(p[t], c[t]);
                r = __fadd_rn(r, __fmul_rn(d, d));
            }
            const float old = mind[i];
            mind[i] = r < old ? r : old;   // std::min(old, r)
        }
    }
}

void launch_kpp_update(const float* x, long long n, int dim, const float* c, float* mind,
                       cudaStream_t st) {
    if (n <= 0) return;
    const long long warps = n;
    const int blocks = (int)std::min<long long>((warps * 32 + 255) / 256, 148LL * 64);
    kpp_update_kernel<<<blocks, 256, 0, st>>>(x, n, dim, c, mind);
    VGPU_LAUNCH("kpp_update_kernel");
}

// ---------------------------------------------------------------------------------
// k-means++ draws on the device.  kmeans_plusplus_init (src/index/kmeans.cpp:45-89)
// draws the next centroid as lower_bound(cumsum, u * cumsum.back()) over the fp64
// running prefix sum of the D^2 vector, with u the next generate_canonical<double>
// value of its std::mt19937 (uniform_real_distribution(0, t) is u * t in libstdc++).
// The host draws every u ahead (the stream has no other consumer) and the device finds
// the index: per-block fp64 sums of the refreshed D^2 (kpp_update_sum_kernel), then one
// CTA scans the block sums, finds the block holding the target and scans inside it
// (kpp_pick_kernel).  The D^2 values are the reference's lane-order distances; only
// the association of the fp64 prefix sums differs, so an index can differ only when a
// target lies within the sums' rounding (~n * 2^-53 of the total) of a boundary.
// ---------------------------------------------------------------------------------
constexpr int KPP_PTS = 2048;   // points per block of the refresh (and of the in-block scan)
constexpr int KPP_PICK_NT = 1024;

__global__ void __launch_bounds__(256) kpp_update_sum_kernel(const float* __restrict__ x, long long n, int dim,
                                                              const float* __restrict__ c, float* __restrict__ mind,
                                                              double* __restrict__ block_sum) {
    // Eight lanes per point (lane l of a group of 8 accumulates elements l, l+8, ...
    // in order, as AVX2 lane l does), four points per warp, 32 per pass of the CTA.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 3, l = lane & 7;
    const long long p0 = (long long)blockIdx.x * KPP_PTS;
    const long long p1 = p0 + KPP_PTS < n ? p0 + KPP_PTS : n;
    const int simd_end = dim & ~7;
    double part = 0.0;
    for (long long base = p0 + warp * 4; base < p1; base += 32) {   // warp-uniform trip count
        const long long i = base + g;
        const bool act = i < p1;
        const float* p = x + (act ? i : p0) * (long long)dim;
        float acc = 0.0f;
        if (act)
            for (int t = l; t < simd_end; t += 8) {
                const float d = __fsub_rn(p[t], c[t]);
                acc = __fmaf_rn(d, d, acc);
            }
        const float a4 = __shfl_down_sync(0xffffffffu, acc, 4, 8);
        const float sv = __fadd_rn(a4, acc);          // l = 0..3: a_{l+4} + a_l
        const float s1 = __shfl_down_sync(0xffffffffu, sv, 1, 8);
        const float s2 = __shfl_down_sync(0xffffffffu, sv, 2, 8);
        const float s3 = __shfl_down_sync(0xffffffffu, sv, 3, 8);
        if (act && l == 0) {
            float r = __fadd_rn(__fadd_rn(sv, s1), __fadd_rn(s2, s3));
            for (int t = simd_end; t < dim; ++t) {
                const float d = __fsub_rn(p[t], c[t]);
                r = __fadd_rn(r, __fmul_rn(d, d));
            }
            const float old = mind[i];
            const float v = r < old ? r : old;   // std::min(old, r)
            mind[i] = v;
            part += (double)v;
        }
    }
    __shared__ double s_part[8];
    for (int o = 16; o > 0; o >>= 1) part += __shfl_down_sync(0xffffffffu, part, o);
    if (lane == 0) s_part[warp] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; ++w) t += s_part[w];
        block_sum[blockIdx.x] = t;
    }
}

// Exclusive prefix sum of v over the CTA (KPP_PICK_NT threads); *total gets the sum.
__device__ double kpp_block_exclusive_scan(double v, double* s_warp, double* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        double w = s_warp[lane];
        double wi = w;
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        s_warp[lane] = wi - w;       // exclusive prefix of the warp totals
        if (lane == 31) s_warp[32] = wi;
    }
    __syncthreads();
    const double r = s_warp[warp] + (inc - v);
    *total = s_warp[32];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(KPP_PICK_NT) kpp_pick_kernel(const float* __restrict__ x, long long n, int dim,
                                                               const float* __restrict__ mind,
                                                               const double* __restrict__ block_sum, int nb,
                                                               const double* __restrict__ u, int c,
                                                               float* __restrict__ centroids) {
    __shared__ double s_warp[33];
    __shared__ int s_blk;
    __shared__ double s_blk_excl;
    __shared__ unsigned long long s_idx;
    __shared__ unsigned long long s_last1;   // 1 + last index with weight, 0 = none
    const int t = threadIdx.x;
    if (t == 0) { s_blk = nb; s_idx = ~0ull; s_last1 = 0; }
    // 1) block sums: thread t owns blocks [t*per, (t+1)*per)
    const int per = (nb + KPP_PICK_NT - 1) / KPP_PICK_NT;
    const int b0 = t * per, b1 = min(nb, b0 + per);
    double mine = 0.0;
    for (int b = b0; b < b1; ++b) mine += block_sum[b];
    double total;
    const double excl = kpp_block_exclusive_scan(mine, s_warp, &total);
    const double target = __dmul_rn(u[c], total);
    {
        double run = excl;
        for (int b = b0; b < b1; ++b) {
            const double nx = run + block_sum[b];
            if (nx >= target && block_sum[b] > 0.0) {
                atomicMin(&s_blk, b);
                break;
            }
            run = nx;
        }
    }
    __syncthreads();
    int blk = s_blk;
    if (blk >= nb) {
        // the target exceeds every prefix (rounding): the last block with weight
        if (t == 0) {
            int b = nb - 1;
            while (b > 0 && !(block_sum[b] > 0.0)) --b;
            s_blk = b;
        }
        __syncthreads();
        blk = s_blk;
    }
    // exclusive prefix of the chosen block (its owner recomputes it the same way)
    if (blk >= b0 && blk < b1) {
        double run = excl;
        for (int b = b0; b < blk; ++b) run += block_sum[b];
        s_blk_excl = run;
    }
    __syncthreads();
    // 2) inside the block: thread t holds points p0 + 2t, p0 + 2t + 1
    const long long p0 = (long long)blk * KPP_PTS;
    const long long i0 = p0 + 2 * t, i1 = i0 + 1;
    const double v0 = i0 < n ? (double)mind[i0] : 0.0;
    const double v1 = i1 < n ? (double)mind[i1] : 0.0;
    double dummy;
    const double e = kpp_block_exclusive_scan(v0 + v1, s_warp, &dummy) + s_blk_excl;
    const double c0 = e + v0, c1 = c0 + v1;
    // lower_bound: the first point whose prefix reaches the target (a point of zero
    // weight never does first: its prefix equals its predecessor's)
    if (i0 < n && v0 > 0.0 && c0 >= target) atomicMin(&s_idx, (unsigned long long)i0);
    else if (i1 < n && v1 > 0.0 && c1 >= target) atomicMin(&s_idx, (unsigned long long)i1);
    if (i1 < n && v1 > 0.0) atomicMax(&s_last1, (unsigned long long)i1 + 1);
    else if (i0 < n && v0 > 0.0) atomicMax(&s_last1, (unsigned long long)i0 + 1);
    __syncthreads();
    long long idx = s_idx != ~0ull ? (long long)s_idx : (s_last1 ? (long long)s_last1 - 1 : p0);
    if (idx >= n) idx = n - 1;
    // 3) copy the point into centroid row c
    for (int j = t; j < dim; j += KPP_PICK_NT) centroids[(long long)c * dim + j] = x[idx * dim + j];
}

void launch_kpp_update_sum(const float* x, long long n, int dim, const float* c, float* mind, double* block_sum,
                           cudaStream_t st) {
    if (n <= 0) return;
    const long long nb = (n + KPP_PTS - 1) / KPP_PTS;
    kpp_update_sum_kernel<<<(unsigned)nb, 256, 0, st>>>(x, n, dim, c, mind, block_sum);
    VGPU_LAUNCH("kpp_update_sum_kernel");
}

void launch_kpp_pick(const float* x, long long n, int dim, const float* mind, const double* block_sum,
                     const double* u, int c, float* centroids, cudaStream_t st) {
    if (n <= 0) return;
    const long long nb = (n + KPP_PTS - 1) / KPP_PTS;
    kpp_pick_kernel<<<1, KPP_PICK_NT, 0, st>>>(x, n, dim, mind, block_sum, (int)nb, u, c, centroids);
    VGPU_LAUNCH("kpp_pick_kernel");
}

long long kpp_blocks(long long n) { return (n + KPP_PTS - 1) / KPP_PTS; }

__global__ void segment_mean_kernel(const float* __restrict__ x, int dim,
                                    const uint32_t* __restrict__ order,
                                    const uint32_t* __restrict__ seg, int kahan,
                                    float* __restrict__ centroids) {
    const int c = blockIdx.x;
    const uint32_t b = seg[c], e = seg[c + 1];
    if (b == e) return;  // empty cluster keeps its centroid
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        double sum = 0.0, comp = 0.0;
        if (kahan) {
            for (uint32_t j = b; j < e; ++j) {
                const double y = (double)x[(long long)order[j] * dim + d] - comp;
                const double t = sum + y;
                comp = (t - sum) - y;
                sum = t;
            }
            const double scale = 1.0 / (double)(e - b);
            centroids[(long long)c * dim + d] = (float)(sum * scale);
        } else {
            for (uint32_t j = b; j < e; ++j) sum += (double)x[(long long)order[j] * dim + d];
            centroids[(long long)c * dim + d] = (float)(sum / (double)(e - b));
        }
    }
}

void launch_segment_mean(const float* x, int dim, const uint32_t* order, const uint32_t* seg,
                         int k, int kahan, float* centroids, cudaStream_t st) {
    if (k <= 0) return;
    const int threads = dim >= 256 ? 256 : ((dim + 31) / 32) * 32;
    segment_mean_kernel<<<k, threads, 0, st>>>(x, dim, order, seg, kahan, centroids);
    VGPU_LAUNCH("segment_mean_kernel");
}

// One CTA per cluster, one thread per dimension: the loop of segment_mean_kernel,
// resumed from and saved to (sum, comp).
__global__ void segment_accumulate_kernel(const float* __restrict__ x, int dim, const uint32_t* __restrict__ order,
                                          const uint32_t* __restrict__ seg, int kahan, double* __restrict__ sum,
                                          double* __restrict__ comp, unsigned long long* __restrict__ count) {
    const int c = blockIdx.x;
    const uint32_t b = seg[c], e = seg[c + 1];
    if (b == e) return;
    if (threadIdx.x == 0) count[c] += e - b;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        const long long o = (long long)c * dim + d;
        double s = sum[o];
        if (kahan) {
            double cp = comp[o];
            for (uint32_t j = b; j < e; ++j) {
                const double y = (double)x[(long long)order[j] * dim + d] - cp;
                const double t = s + y;
                cp = (t - s) - y;
                s = t;
            }
            comp[o] = cp;
        } else {
            for (uint32_t j = b; j < e; ++j) s += (double)x[(long long)order[j] * dim + d];
        }
        sum[o] = s;
    }
}

__global__ void finish_means_kernel(const double* __restrict__ sum, const unsigned long long* __restrict__ count,
                                    long long total, int dim, int kahan, float* __restrict__ centroids) {
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const unsigned long long n = count[t / dim];
        if (n == 0) continue;  // empty cluster keeps its centroid
        centroids[t] = kahan ? (float)(sum[t] * (1.0 / (double)n)) : (float)(sum[t] / (double)n);
    }
}

void launch_segment_accumulate(const float* x, int dim, const uint32_t* order, const uint32_t* seg, int k,
                               int kahan, double* sum, double* comp, unsigned long long* count, cudaStream_t st) {
    if (k <= 0) return;
    const int threads = dim >= 256 ? 256 : ((dim + 31) / 32) * 32;
    segment_accumulate_kernel<<<k, threads, 0, st>>>(x, dim, order, seg, kahan, sum, comp, count);
    VGPU_LAUNCH("segment_accumulate_kernel");
}

void launch_finish_means(const double* sum, const unsigned long long* count, int k, int dim, int kahan,
                         float* centroids, cudaStream_t st) {
    const long long total = (long long)k * dim;
    if (total <= 0) return;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    finish_means_kernel<<<blocks, 256, 0, st>>>(sum, count, total, dim, kahan, centroids);
    VGPU_LAUNCH("finish_means_kernel");
}

}  // namespace vgpu

namespace vgpu {

// The final inertia of kmeans_cluster (src/index/kmeans.cpp:230-241): ONE float running
// total over every (point, dimension) term in point-major order, t += (x - c)^2 with the
// subtraction, the square and the add each rounded.  A running float sum has no
// reassociation, so one thread adds; the CTA's other threads compute the next chunk of
// terms into shared memory.  *total holds the starting value and receives the result.
constexpr int OSQ_CHUNK = 8192;
__global__ void __launch_bounds__(1024) ordered_sq_sum_kernel(const float* __restrict__ x, const float* __restrict__ c,
                                                              const uint32_t* __restrict__ assign, long long n,
                                                              int dim, float* __restrict__ total) {
    __shared__ float terms[OSQ_CHUNK];
    const long long count = n * dim;
    float acc = *total;
    for (long long t0 = 0; t0 < count; t0 += OSQ_CHUNK) {
        const int len = (int)(count - t0 < OSQ_CHUNK ? count - t0 : (long long)OSQ_CHUNK);
        for (int j = threadIdx.x; j < len; j += blockDim.x) {
            const long long t = t0 + j;
            const long long i = t / dim;
            const int d = (int)(t - i * dim);
            const float diff = __fsub_rn(x[t], c[(long long)assign[i] * dim + d]);
            terms[j] = __fmul_rn(diff, diff);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
#pragma unroll 16
            for (int j = 0; j < len; ++j) acc = __fadd_rn(acc, terms[j]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *total = acc;
}

void launch_ordered_sq_sum(const float* x, const float* c, const uint32_t* assign, long long n, int dim,
                           float* total, cudaStream_t st) {
    if (n <= 0) return;
    ordered_sq_sum_kernel<<<1, 1024, 0, st>>>(x, c, assign, n, dim, total);
    VGPU_LAUNCH("ordered_sq_sum_kernel");
}


}  // namespace vgpu
