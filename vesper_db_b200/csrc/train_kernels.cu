// B200 kernels for PQ training (m sub-space k-means runs batched in one launch) and
// for the training-time error passes.
//
// FastScanPq::train (src/index/pq_fastscan.cpp:15-76) runs one KmeansElkan per
// sub-space (k = 2^nbits, seed 42 + s).  Here all sub-spaces advance together; each
// keeps its own k-means++ stream and its own convergence test, and a converged
// sub-space stops changing (the `active` mask).
#include <cfloat>

#include <cub/device/device_radix_sort.cuh>

#include "kernels.cuh"
#include "kernels_train.cuh"

namespace vgpu {

__global__ void fill_f32_kernel(float* p, long long n, float v) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        p[i] = v;
}

void launch_fill(float* p, long long n, float v, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    fill_f32_kernel<<<blocks, 256, 0, st>>>(p, n, v);
    VGPU_LAUNCH("fill_f32_kernel");
}

// mind[s][i] = min(mind[s][i], l2(x_i[s], pick_s)) for every sub-space s.
__global__ void pq_kpp_update_kernel(const float* __restrict__ x, long long n, int dim, int m,
                                     int dsub, const float* __restrict__ picks,
                                     float* __restrict__ mind) {
    const long long total = n * m;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int s = (int)(e / n);
        const long long i = e % n;
        const float d = l2_ref(x + i * dim + (long long)s * dsub, picks + (long long)s * dsub, dsub);
        const float old = mind[e];
        mind[e] = d < old ? d : old;
    }
}

void launch_pq_kpp_update(const float* x, long long n, int dim, int m, int dsub,
                          const float* picks, float* mind, cudaStream_t st) {
    const long long total = n * m;
    if (total <= 0) return;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 32);
    pq_kpp_update_kernel<<<blocks, 256, 0, st>>>(x, n, dim, m, dsub, picks, mind);
    VGPU_LAUNCH("pq_kpp_update_kernel");
}

// picks[s] = x[idx[s]][s*dsub : (s+1)*dsub]; also written to cb[s][slot].
__global__ void pq_gather_picks_kernel(const float* __restrict__ x, int dim, int m, int dsub,
                                       const uint32_t* __restrict__ idx, int slot, int ksub,
                                       float* __restrict__ picks, float* __restrict__ cb) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= m * dsub) return;
    const int s = e / dsub, t = e % dsub;
    const float v = x[(long long)idx[s] * dim + (long long)s * dsub + t];
    picks[e] = v;
    cb[((long long)s * ksub + slot) * dsub + t] = v;
}

void launch_pq_gather_picks(const float* x, int dim, int m, int dsub, const uint32_t* idx, int slot,
                            int ksub, float* picks, float* cb, cudaStream_t st) {
    pq_gather_picks_kernel<<<ceil_div((long long)m * dsub, 256), 256, 0, st>>>(x, dim, m, dsub, idx, slot,
                                                                              ksub, picks, cb);
    VGPU_LAUNCH("pq_gather_picks_kernel");
}

// E-step of every sub-space k-means: codes[s][i] = arg-min_j l2(x_i[s], cb[s][j]) with
// a strict `<` scan (lowest j wins); with keep != 0 the current code is kept when it
// ties the minimum (assign_with_bounds, src/index/kmeans_elkan.cpp:183-262).
// Inactive sub-spaces are left untouched.  mind[s][i] receives the minimum.
template <int DS>
__global__ void __launch_bounds__(128) pq_assign_kernel(const float* __restrict__ x, long long n,
                                                        int dim, int ksub, int dsub_rt,
                                                        const float* __restrict__ cb,
                                                        uint32_t* __restrict__ codes,
                                                        float* __restrict__ mind, int keep,
                                                        const int* __restrict__ active) {
    extern __shared__ __align__(16) float ycb[];
    const int dsub = DS > 0 ? DS : dsub_rt;
    const int s = blockIdx.y;
    if (active && !active[s]) return;
    const float* y = cb + (long long)s * ksub * dsub;
    for (int e = threadIdx.x; e < ksub * dsub; e += blockDim.x) ycb[e] = y[e];
    __syncthreads();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* v = x + i * dim + (long long)s * dsub;
    float vr[DS > 0 ? DS : 64];
    const float* vp = v;
    if (DS > 0) {
#pragma unroll
        for (int t = 0; t < (DS > 0 ? DS : 1); ++t) vr[t] = v[t];
        vp = vr;
    }
    float best = FLT_MAX;
    uint32_t code = 0;
    for (int j = 0; j < ksub; ++j) {
        const float d = l2_ref(vp, ycb + j * dsub, dsub);
        if (d < best) { best = d; code = (uint32_t)j; }
    }
    const long long o = (long long)s * n + i;
    if (keep) {
        const uint32_t cur = codes[o];
        if (l2_ref(vp, ycb + cur * dsub, dsub) == best) code = cur;
    }
    codes[o] = code;
    mind[o] = best;
}

void launch_pq_assign(const float* x, long long n, int dim, int m, int ksub, int dsub,
                      const float* cb, uint32_t* codes, float* mind, int keep, const int* active,
                      cudaStream_t st) {
    if (n <= 0) return;
    const size_t smem = (size_t)ksub * dsub * sizeof(float);
    if (smem > 200 * 1024) throw CudaError("pq_assign: sub-space codebook too large for shared memory");
    dim3 grid(ceil_div(n, 128), m);
#define VGPU_PQA(DSV)                                                                             \
    do {                                                                                          \
        VGPU_CHECK(cudaFuncSetAttribute(pq_assign_kernel<DSV>,                                    \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        pq_assign_kernel<DSV><<<grid, 128, smem, st>>>(x, n, dim, ksub, dsub, cb, codes, mind,     \
                                                       keep, active);                             \
    } while (0)
    if (dsub == 4) VGPU_PQA(4);
    else if (dsub == 8) VGPU_PQA(8);
    else if (dsub == 16) VGPU_PQA(16);
    else VGPU_PQA(0);
#undef VGPU_PQA
    VGPU_LAUNCH("pq_assign_kernel");
}

// keys[s*n + i] = s*ksub + codes[s*n + i]
__global__ void pq_keys_kernel(const uint32_t* __restrict__ codes, long long n, int m, int ksub,
                               uint32_t* __restrict__ keys) {
    const long long total = n * m;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x)
        keys[e] = (uint32_t)(e / n) * (uint32_t)ksub + codes[e];
}

void launch_pq_keys(const uint32_t* codes, long long n, int m, int ksub, uint32_t* keys,
                    cudaStream_t st) {
    const long long total = n * m;
    if (total <= 0) return;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    pq_keys_kernel<<<blocks, 256, 0, st>>>(codes, n, m, ksub, keys);
    VGPU_LAUNCH("pq_keys_kernel");
}

// PQ M-step: cluster (s, j) = segment s*ksub + j of `order`, whose items are
// s*n + i.  Kahan fp64 in item (= point) order, times 1/count; empty -> unchanged.
__global__ void pq_segment_mean_kernel(const float* __restrict__ x, long long n, int dim,
                                       int dsub, int ksub, const uint32_t* __restrict__ order,
                                       const uint32_t* __restrict__ seg,
                                       const int* __restrict__ active, float* __restrict__ cb) {
    const int cid = blockIdx.x;
    const int s = cid / ksub;
    if (active && !active[s]) return;
    const uint32_t b = seg[cid], e = seg[cid + 1];
    if (b == e) return;
    for (int t = threadIdx.x; t < dsub; t += blockDim.x) {
        double sum = 0.0, comp = 0.0;
        for (uint32_t j = b; j < e; ++j) {
            const long long i = (long long)order[j] - (long long)s * n;
            const double y = (double)x[i * dim + (long long)s * dsub + t] - comp;
            const double tt = sum + y;
            comp = (tt - sum) - y;
            sum = tt;
        }
        const double scale = 1.0 / (double)(e - b);
        cb[(long long)cid * dsub + t] = (float)(sum * scale);
    }
}

void launch_pq_segment_mean(const float* x, long long n, int dim, int m, int dsub, int ksub,
                            const uint32_t* order, const uint32_t* seg, const int* active, float* cb,
                            cudaStream_t st) {
    const int threads = dsub >= 32 ? 32 * ((dsub + 31) / 32 > 8 ? 8 : (dsub + 31) / 32) : 32;
    pq_segment_mean_kernel<<<m * ksub, threads, 0, st>>>(x, n, dim, dsub, ksub, order, seg, active, cb);
    VGPU_LAUNCH("pq_segment_mean_kernel");
}

// Stable grouping of items by key: order = item indices sorted by key (stable radix
// sort keeps item order inside a key), seg = exclusive prefix of the key counts.
__global__ void iota_kernel(uint32_t* p, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        p[i] = (uint32_t)i;
}

__global__ void seg_from_sorted_kernel(const uint32_t* __restrict__ sorted_keys, long long n,
                                       int nkeys, uint32_t* __restrict__ seg) {
    // seg[c] = first position with key >= c
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c <= nkeys;
         c += (long long)gridDim.x * blockDim.x) {
        long long lo = 0, hi = n;
        while (lo < hi) {
            const long long mid = (lo + hi) >> 1;
            if (sorted_keys[mid] < (uint32_t)c) lo = mid + 1; else hi = mid;
        }
        seg[c] = (uint32_t)lo;
    }
}

GroupWork::~GroupWork() {
    if (tmp) cudaFree(tmp);
    if (keys_out) cudaFree(keys_out);
    if (vals_in) cudaFree(vals_in);
}

void group_by_key(const uint32_t* keys, long long n, int nkeys, uint32_t* order, uint32_t* seg,
                  GroupWork& w, cudaStream_t st) {
    if (n > 0) {
        if ((size_t)n > w.cap) {
            if (w.keys_out) cudaFree(w.keys_out);
            if (w.vals_in) cudaFree(w.vals_in);
            VGPU_CHECK(cudaMalloc(&w.keys_out, sizeof(uint32_t) * n));
            VGPU_CHECK(cudaMalloc(&w.vals_in, sizeof(uint32_t) * n));
            w.cap = (size_t)n;
        }
        const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
        iota_kernel<<<blocks, 256, 0, st>>>(w.vals_in, n);
        VGPU_LAUNCH("iota_kernel");
        int bits = 1;
        while ((1ll << bits) < (long long)nkeys) ++bits;
        size_t need = 0;
        VGPU_CHECK(cub::DeviceRadixSort::SortPairs(nullptr, need, keys, w.keys_out, w.vals_in, order,
                                                   (int)n, 0, bits, st));
        if (need > w.tmp_bytes) {
            if (w.tmp) cudaFree(w.tmp);
            VGPU_CHECK(cudaMalloc(&w.tmp, need));
            w.tmp_bytes = need;
        }
        VGPU_CHECK(cub::DeviceRadixSort::SortPairs(w.tmp, need, keys, w.keys_out, w.vals_in, order,
                                                   (int)n, 0, bits, st));
        seg_from_sorted_kernel<<<ceil_div(nkeys + 1, 256), 256, 0, st>>>(w.keys_out, n, nkeys, seg);
        VGPU_LAUNCH("seg_from_sorted_kernel");
    } else {
        VGPU_CHECK(cudaMemsetAsync(seg, 0, sizeof(uint32_t) * (nkeys + 1), st));
    }
}

// decoded[i] = concat_s cb[s][codes[i][s]]
__global__ void pq_decode_kernel(const uint8_t* __restrict__ codes, long long n, int m, int ksub,
                                 int dsub, const float* __restrict__ cb, float* __restrict__ out) {
    const long long dim = (long long)m * dsub;
    const long long total = n * dim;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long i = e / dim;
        const int k = (int)(e % dim);
        const int s = k / dsub, t = k % dsub;
        out[e] = cb[((long long)s * ksub + codes[i * m + s]) * dsub + t];
    }
}

void launch_pq_decode(const uint8_t* codes, long long n, int m, int ksub, int dsub, const float* cb,
                      float* out, cudaStream_t st) {
    const long long total = n * (long long)m * dsub;
    if (total <= 0) return;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 32);
    pq_decode_kernel<<<blocks, 256, 0, st>>>(codes, n, m, ksub, dsub, cb, out);
    VGPU_LAUNCH("pq_decode_kernel");
}

// out[i] = l2_ref(a_i, b_i) (one warp per row; lanes 0..7 run the 8 lane chains)
__global__ void row_l2_kernel(const float* __restrict__ a, const float* __restrict__ b, long long n,
                              int dim, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    const int simd_end = dim & ~7;
    for (long long i = warp; i < n; i += nwarps) {
        const float* p = a + i * dim;
        const float* q = b + i * dim;
        float acc = 0.0f;
        if (lane < 8)
            for (int t = lane; t < simd_end; t += 8) {
                const float d = __fsub_rn(p[t], q[t]);
                acc = __fmaf_rn(d, d, acc);
            }
        const float a4 = __shfl_down_sync(0xffffffffu, acc, 4);
        const float s = __fadd_rn(a4, acc);
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1);
        const float s2 = __shfl_down_sync(0xffffffffu, s, 2);
        const float s3 = __shfl_down_sync(0xffffffffu, s, 3);
        if (lane == 0) {
            float r = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
            for (int t = simd_end; t < dim; ++t) {
                const float d = __fsub_rn(p[t], q[t]);
                r = __fadd_rn(r, __fmul_rn(d, d));
            }
            out[i] = r;
        }
    }
}

void launch_row_l2(const float* a, const float* b, long long n, int dim, float* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n * 32 + 255) / 256, 148LL * 64);
    row_l2_kernel<<<blocks, 256, 0, st>>>(a, b, n, dim, out);
    VGPU_LAUNCH("row_l2_kernel");
}

__global__ void transpose_kernel(const float* __restrict__ in, int d, float* __restrict__ out) {
    __shared__ float t[32][33];
    const int x0 = blockIdx.x * 32, y0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = y0 + j, c = x0 + threadIdx.x;
        if (r < d && c < d) t[j][threadIdx.x] = in[(long long)r * d + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = x0 + j, c = y0 + threadIdx.x;
        if (r < d && c < d) out[(long long)r * d + c] = t[threadIdx.x][j];
    }
}

void launch_transpose(const float* in, int d, float* out, cudaStream_t st) {
    dim3 grid(ceil_div(d, 32), ceil_div(d, 32));
    transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(in, d, out);
    VGPU_LAUNCH("transpose_kernel");
}

__global__ void gather_rows_kernel(const float* __restrict__ x, int dim, const uint32_t* __restrict__ idx,
                                   long long n, float* __restrict__ out) {
    const long long total = n * dim;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long i = e / dim;
        out[e] = x[(long long)idx[i] * dim + (e % dim)];
    }
}

void launch_gather_rows(const float* x, int dim, const uint32_t* idx, long long n, float* out,
                        cudaStream_t st) {
    const long long total = n * dim;
    if (total <= 0) return;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 32);
    gather_rows_kernel<<<blocks, 256, 0, st>>>(x, dim, idx, n, out);
    VGPU_LAUNCH("gather_rows_kernel");
}

__global__ void gather_u32_kernel(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx, long long n,
                                  uint32_t* __restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = src[idx[i]];
}

void launch_gather_u32(const uint32_t* src, const uint32_t* idx, long long n, uint32_t* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 32);
    gather_u32_kernel<<<blocks, 256, 0, st>>>(src, idx, n, out);
    VGPU_LAUNCH("gather_u32_kernel");
}

__global__ void d2f_kernel(const double* __restrict__ in, long long n, float* __restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = (float)in[i];
}

void launch_d2f(const double* in, long long n, float* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 8);
    d2f_kernel<<<blocks, 256, 0, st>>>(in, n, out);
    VGPU_LAUNCH("d2f_kernel");
}

}  // namespace vgpu
