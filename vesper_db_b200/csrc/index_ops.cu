// Kernels behind IvfPqIndex's maintenance and inspection API (reconstruct,
// reconstruct_cluster, reassign_vector, debug_explain_*; src/index/ivf_pq.cpp:4997-5541).
// Reconstruction follows the reference operation for operation: the decoded code
// (codebook rows), apply_rotation_T in sequential order (residual_rotate_kernel with
// R transposed), then centroid + residual with one rounded add per element.
#include <cfloat>

#include "kernels.cuh"

namespace vgpu {

// out[i] = decode(codes[entry(i)]), entry(i) = entries ? entries[i] : e0 + i.
__global__ void decode_rows_kernel(const uint32_t* __restrict__ entries, unsigned long long e0, long long n,
                                   const uint8_t* __restrict__ codes, int m, int ksub, int dsub,
                                   const float* __restrict__ cb, float* __restrict__ out) {
    const int dim = m * dsub;
    for (long long i = blockIdx.x; i < n; i += gridDim.x) {
        const unsigned long long e = entries ? entries[i] : e0 + (unsigned long long)i;
        const uint8_t* cd = codes + e * (unsigned long long)m;
        for (int d = threadIdx.x; d < dim; d += blockDim.x) {
            const int s = d / dsub;
            out[i * dim + d] = cb[((long long)s * ksub + cd[s]) * dsub + (d - s * dsub)];
        }
    }
}

// out[i][d] = cent[list(i)][d] + res[i][d] (rounded), list(i) = lists ? lists[i] : list0.
__global__ void add_centroid_kernel(const float* __restrict__ res, const uint32_t* __restrict__ lists, uint32_t list0,
                                    const float* __restrict__ cent, long long n, int dim, float* __restrict__ out) {
    const long long total = n * dim;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long i = t / dim;
        const int d = (int)(t % dim);
        const uint32_t l = lists ? lists[i] : list0;
        out[t] = __fadd_rn(cent[(long long)l * dim + d], res[t]);
    }
}

void launch_reconstruct_rows(const uint32_t* entries, unsigned long long e0, const uint32_t* lists, uint32_t list0,
                             long long n, const uint8_t* codes, int m, int ksub, int dsub, const float* cb,
                             const float* cent, const float* rotT, float* tmp_dec, float* tmp_rot, float* out,
                             cudaStream_t st) {
    if (n <= 0) return;
    const int dim = m * dsub;
    decode_rows_kernel<<<(unsigned)std::min<long long>(n, 148LL * 16), 128, 0, st>>>(entries, e0, n, codes, m, ksub,
                                                                                   dsub, cb, tmp_dec);
    VGPU_LAUNCH("decode_rows_kernel");
    const float* res = tmp_dec;
    if (rotT) {
        launch_residual_rotate(tmp_dec, nullptr, nullptr, nullptr, n, dim, rotT, tmp_rot, st);
        res = tmp_rot;
    }
    const int blocks = (int)std::min<long long>((n * dim + 255) / 256, 148LL * 32);
    add_centroid_kernel<<<blocks, 256, 0, st>>>(res, lists, list0, cent, n, dim, out);
    VGPU_LAUNCH("add_centroid_kernel");
}

// One CTA per list: the list's exact lookup table (reference order, from the residual
// row rres[l]) and the exact ADC distance of each of its entries into adc[e].
constexpr int AA_NT = 256;
__global__ void __launch_bounds__(AA_NT) adc_all_kernel(const float* __restrict__ rres, int dim,
                                                        const float* __restrict__ cb, int m, int ksub, int dsub,
                                                        const uint64_t* __restrict__ offs,
                                                        const uint8_t* __restrict__ codes, float* __restrict__ adc) {
    extern __shared__ __align__(16) float sm[];
    float* r = sm;                          // [dim]
    float* lut = sm + ((dim + 3) & ~3);     // [m * ksub]
    const long long l = blockIdx.x;
    const uint64_t e0 = offs[l], e1 = offs[l + 1];
    if (e0 == e1) return;
    for (int d = threadIdx.x; d < dim; d += AA_NT) r[d] = rres[l * dim + d];
    __syncthreads();
    for (int e = threadIdx.x; e < m * ksub; e += AA_NT) {
        const int s = e / ksub, j = e % ksub;
        lut[e] = l2_ref(r + s * dsub, cb + ((long long)s * ksub + j) * dsub, dsub);
    }
    __syncthreads();
    for (uint64_t e = e0 + threadIdx.x; e < e1; e += AA_NT) {
        const uint8_t* code = codes + e * (uint64_t)m;
        float dd = 0.0f;
        for (int s = 0; s < m; ++s) dd = __fadd_rn(dd, lut[s * ksub + code[s]]);
        adc[e] = dd;
    }
}

void launch_adc_all(const float* rres, int dim, int nlist, const float* cb, int m, int ksub, int dsub,
                    const uint64_t* offs, const uint8_t* codes, float* adc, cudaStream_t st) {
    if (nlist <= 0) return;
    const size_t smem = ((size_t)((dim + 3) & ~3) + (size_t)m * ksub) * sizeof(float);
    if (smem > 227 * 1024) throw CudaError("adc_all: lookup table does not fit in shared memory");
    VGPU_CHECK(cudaFuncSetAttribute(adc_all_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    adc_all_kernel<<<nlist, AA_NT, smem, st>>>(rres, dim, cb, m, ksub, dsub, offs, codes, adc);
    VGPU_LAUNCH("adc_all_kernel");
}

// *count += number of v[i] < v[target] (i over n).
__global__ void count_less_kernel(const float* __restrict__ v, long long n, long long target,
                                  unsigned long long* __restrict__ count) {
    const float t = v[target];
    unsigned long long c = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        c += v[i] < t ? 1ull : 0ull;
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, c);
}

void launch_count_less(const float* v, long long n, long long target, unsigned long long* count, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    count_less_kernel<<<blocks, 256, 0, st>>>(v, n, target, count);
    VGPU_LAUNCH("count_less_kernel");
}

// out[0] = the first entry (list order) holding id, or 0xffffffff; out[1] = its list.
__global__ void id_lookup_kernel(const uint64_t* __restrict__ sid, const uint32_t* __restrict__ sent, long long n,
                                 uint64_t id, const uint64_t* __restrict__ offs, int nlist, uint32_t* __restrict__ out) {
    long long lo = 0, hi = n;
    while (lo < hi) {
        const long long mid = (lo + hi) >> 1;
        if (sid[mid] < id) lo = mid + 1; else hi = mid;
    }
    uint32_t e = 0xffffffffu, l = 0;
    if (lo < n && sid[lo] == id) {
        e = sent[lo];
        int a = 0, b = nlist;
        while (b - a > 1) {
            const int mid = (a + b) >> 1;
            if (offs[mid] <= (uint64_t)e) a = mid; else b = mid;
        }
        l = (uint32_t)a;
    }
    out[0] = e;
    out[1] = l;
}

void launch_id_lookup(const uint64_t* sid, const uint32_t* sent, long long n, uint64_t id, const uint64_t* offs,
                      int nlist, uint32_t* out, cudaStream_t st) {
    id_lookup_kernel<<<1, 1, 0, st>>>(sid, sent, n, id, offs, nlist, out);
    VGPU_LAUNCH("id_lookup_kernel");
}

// codes2[i] / ids2[i] = entry order[i] of codes / ids, or the new entry (new_code, new_id)
// where order[i] == 0xffffffff.  One warp per entry.
__global__ void gather_entries_kernel(const uint32_t* __restrict__ order, long long n,
                                      const uint8_t* __restrict__ codes, const uint64_t* __restrict__ ids, int m,
                                      const uint8_t* __restrict__ new_code, uint64_t new_id,
                                      uint8_t* __restrict__ codes2, uint64_t* __restrict__ ids2) {
    const int lane = threadIdx.x & 31;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long i = w; i < n; i += nw) {
        const uint32_t o = order[i];
        const uint8_t* src = o == 0xffffffffu ? new_code : codes + (unsigned long long)o * m;
        for (int b = lane; b < m; b += 32) codes2[i * m + b] = src[b];
        if (lane == 0) ids2[i] = o == 0xffffffffu ? new_id : ids[o];
    }
}

void launch_gather_entries(const uint32_t* order, long long n, const uint8_t* codes, const uint64_t* ids, int m,
                           const uint8_t* new_code, uint64_t new_id, uint8_t* codes2, uint64_t* ids2,
                           cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n * 32 + 255) / 256, 148LL * 32);
    gather_entries_kernel<<<blocks, 256, 0, st>>>(order, n, codes, ids, m, new_code, new_id, codes2, ids2);
    VGPU_LAUNCH("gather_entries_kernel");
}

}  // namespace vgpu
