// B200 kernels for the IVF-PQ search and add paths.
//
// Exact kernels reproduce the reference arithmetic bit for bit:
//   * distances in the AVX2 lane order (common.cuh: l2_ref / hsum8),
//   * rotations as sequential-k dots with a rounded multiply and a rounded add
//     (apply_rotation, src/index/ivf_pq.cpp:2947-2968),
//   * ADC sums in sub-quantizer order from 0.0f (pq_fastscan.hpp:284-317).
// The fast scan (lut_fast_kernel + scan_fast2_kernel) regroups the ADC algebra so the table is
// built once per query instead of once per (query, list); its distances agree with
// the exact ones to fp32 rounding.
#include <cub/cub.cuh>

#include <cfloat>
#include <cstdint>

#include <cstdlib>

#include "kernels.cuh"
#include "select.cuh"
#include "tc_common.cuh"

namespace vgpu {

// =====================================================================================
// Exact L2 distance tiles:  D[i][j] = l2_ref(x_i, c_j)
//
// CTA tile 64 rows x 32 centroids, 256 threads, each thread 4 rows x 2 centroids x 8
// lane accumulators.  The dimension loop runs over [0, floor(dim/8)*8) in chunks of
// 32 staged in shared memory; element k always feeds lane k%8, so the chunking does
// not change the order of any lane's FMA chain.  Padding past floor(dim/8)*8 is zero,
// which adds exact zeros.  The scalar tail (dim%8 elements) is applied after hsum8.
// =====================================================================================
namespace {
constexpr int DT_Q = 64, DT_C = 32, DT_K = 32, DT_P = DT_K + 4;
}

__global__ void __launch_bounds__(256) l2_dist_kernel(const float* __restrict__ x, long long nx,
                                                      const float* __restrict__ c, int nc, int dim,
                                                      float* __restrict__ D, long long ldd) {
    __shared__ __align__(16) float Xs[DT_Q][DT_P];
    __shared__ __align__(16) float Cs[DT_C][DT_P];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qrow = (warp >> 1) * 16 + (lane >> 3) * 4;
    const int ccol = (warp & 1) * 16 + (lane & 7) * 2;
    const long long q0 = (long long)blockIdx.x * DT_Q;
    const long long c0 = (long long)blockIdx.y * DT_C;
    const int simd_end = dim & ~7;

    float acc[4][2][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int l = 0; l < 8; ++l) acc[i][j][l] = 0.0f;

    for (int k0 = 0; k0 < simd_end; k0 += DT_K) {
        {
            const int r = tid >> 2, s = (tid & 3) * 8;
            const long long g = q0 + r;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int kk = k0 + s + j;
                Xs[r][s + j] = (g < nx && kk < simd_end) ? x[g * dim + kk] : 0.0f;
            }
        }
        {
            const int r = tid >> 3, s = (tid & 7) * 4;
            const long long g = c0 + r;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kk = k0 + s + j;
                Cs[r][s + j] = (g < nc && kk < simd_end) ? c[g * dim + kk] : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < DT_K; kk += 4) {
            float4 xv[4], cv[2];
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(&Xs[qrow + i][kk]);
#pragma unroll
            for (int j = 0; j < 2; ++j) cv[j] = *reinterpret_cast<const float4*>(&Cs[ccol + j][kk]);
            const int lb = kk & 7;  // compile-time after unrolling: 0 or 4
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    float d;
                    d = __fsub_rn(xv[i].x, cv[j].x); acc[i][j][lb + 0] = __fmaf_rn(d, d, acc[i][j][lb + 0]);
                    d = __fsub_rn(xv[i].y, cv[j].y); acc[i][j][lb + 1] = __fmaf_rn(d, d, acc[i][j][lb + 1]);
                    d = __fsub_rn(xv[i].z, cv[j].z); acc[i][j][lb + 2] = __fmaf_rn(d, d, acc[i][j][lb + 2]);
                    d = __fsub_rn(xv[i].w, cv[j].w); acc[i][j][lb + 3] = __fmaf_rn(d, d, acc[i][j][lb + 3]);
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long g = q0 + qrow + i;
        if (g >= nx) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const long long h = c0 + ccol + j;
            if (h >= nc) continue;
            float r = hsum8(acc[i][j]);
            for (int t = simd_end; t < dim; ++t) {
                const float d = __fsub_rn(x[g * dim + t], c[h * dim + t]);
                r = __fadd_rn(r, __fmul_rn(d, d));
            }
            D[g * ldd + h] = r;
        }
    }
}

void launch_l2_dist(const float* x, long long nx, const float* c, int nc, int dim, float* D,
                    long long ldd, cudaStream_t st) {
    if (nx <= 0 || nc <= 0) return;
    dim3 grid(ceil_div(nx, DT_Q), ceil_div(nc, DT_C));
    l2_dist_kernel<<<grid, 256, 0, st>>>(x, nx, c, nc, dim, D, ldd);
    VGPU_LAUNCH("l2_dist_kernel");
}

// =====================================================================================
// Streaming top-k over long rows: the row is consumed in chunks; each round selects
// the k best of [carried k | chunk].  Carried entries always precede the chunk, so
// position order equals column order among equal values.
// =====================================================================================
namespace {
constexpr int SEL_NT = 256;
constexpr int SEL_CH = 2048;
}

template <int NT>
__device__ int carry_round(float* buf, int carry_n, int chunk_n, int k, float* carry_d,
                           uint32_t* carry_tag, uint32_t* tag_tmp, unsigned long long* sortb,
                           SelectSmem& sm, uint32_t chunk_tag0) {
    // buf[0..carry_n) already holds carry_d; buf[carry_n..) the chunk values.
    const int n = carry_n + chunk_n;
    const int got = block_select_k<NT>(buf, n, k, sortb, sm);
    for (int i = threadIdx.x; i < got; i += NT) {
        const uint32_t pos = (uint32_t)(sortb[i] & 0xffffffffull);
        tag_tmp[i] = pos < (uint32_t)carry_n ? carry_tag[pos] : chunk_tag0 + (pos - carry_n);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < got; i += NT) {
        carry_d[i] = key_float((uint32_t)(sortb[i] >> 32));
        carry_tag[i] = tag_tmp[i];
    }
    __syncthreads();
    return got;
}

struct TopkSmem {
    float buf[kMaxK + SEL_CH];
    float carry_d[kMaxK];
    uint32_t carry_tag[kMaxK];
    uint32_t tag_tmp[kMaxK];
    unsigned long long sortb[kMaxK];
    SelectSmem sel;
};

__global__ void __launch_bounds__(SEL_NT) row_topk_kernel(const float* __restrict__ D, int ncols,
                                                          long long ldd, int k,
                                                          uint32_t* __restrict__ out_idx,
                                                          float* __restrict__ out_val) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TopkSmem& S = *reinterpret_cast<TopkSmem*>(smem_raw);
    const long long row = blockIdx.x;
    const float* d = D + row * ldd;
    int carry_n = 0;
    for (int c0 = 0; c0 < ncols; c0 += SEL_CH) {
        const int cn = min(SEL_CH, ncols - c0);
        for (int i = threadIdx.x; i < carry_n; i += SEL_NT) S.buf[i] = S.carry_d[i];
        for (int i = threadIdx.x; i < cn; i += SEL_NT) S.buf[carry_n + i] = d[c0 + i];
        __syncthreads();
        carry_n = carry_round<SEL_NT>(S.buf, carry_n, cn, k, S.carry_d, S.carry_tag, S.tag_tmp,
                                      S.sortb, S.sel, (uint32_t)c0);
    }
    for (int i = threadIdx.x; i < k; i += SEL_NT) {
        out_idx[row * k + i] = i < carry_n ? S.carry_tag[i] : 0u;
        out_val[row * k + i] = i < carry_n ? S.carry_d[i] : FLT_MAX;
    }
}

void launch_row_topk(const float* D, long long n_rows, int ncols, long long ldd, int k,
                     uint32_t* out_idx, float* out_val, cudaStream_t st) {
    if (n_rows <= 0) return;
    if (k > kMaxK) throw CudaError("row_topk: k exceeds the supported maximum");
    const size_t smem = sizeof(TopkSmem);
    VGPU_CHECK(cudaFuncSetAttribute(row_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    row_topk_kernel<<<(unsigned)n_rows, SEL_NT, smem, st>>>(D, ncols, ldd, k, out_idx, out_val);
    VGPU_LAUNCH("row_topk_kernel");
}

// =====================================================================================
// Row arg-min with the reference's strict-< scan semantics.
// =====================================================================================
__global__ void __launch_bounds__(256) row_argmin_kernel(const float* __restrict__ D, int ncols,
                                                         long long ldd,
                                                         const uint32_t* __restrict__ keep,
                                                         uint32_t* __restrict__ out_idx,
                                                         float* __restrict__ out_val) {
    __shared__ unsigned long long red[8];
    const long long row = blockIdx.x;
    const float* d = D + row * ldd;
    unsigned long long best = ~0ull;
    for (int j = threadIdx.x; j < ncols; j += 256) {
        const unsigned long long v = ((unsigned long long)float_key(d[j]) << 32) | (uint32_t)j;
        best = v < best ? v : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v < best ? v : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) best = red[w] < best ? red[w] : best;
        red[0] = best;
        float mv = key_float((uint32_t)(best >> 32));
        uint32_t mi = (uint32_t)(best & 0xffffffffu);
        // A strict `<` scan starting from FLT_MAX never moves off index 0 unless some
        // value is below FLT_MAX.
        if (!(mv < FLT_MAX)) { mi = 0; mv = FLT_MAX; }
        if (keep) {
            const uint32_t kc = keep[row];
            if (d[kc] == mv) mi = kc;
        }
        out_idx[row] = mi;
        if (out_val) out_val[row] = mv;
    }
}

void launch_row_argmin(const float* D, long long n_rows, int ncols, long long ldd,
                       const uint32_t* keep, uint32_t* out_idx, float* out_val, cudaStream_t st) {
    if (n_rows <= 0) return;
    row_argmin_kernel<<<(unsigned)n_rows, 256, 0, st>>>(D, ncols, ldd, keep, out_idx, out_val);
    VGPU_LAUNCH("row_argmin_kernel");
}

// =====================================================================================
// Residual + rotation, exact order: out[r][j] = sum_k a[r][k] * R[k][j], a = x - c.
// CTA tile 64 rows x 64 columns, 256 threads, 4x4 outputs per thread, k staged in
// chunks of 32 and consumed in increasing order (one rounded multiply and one rounded
// add per term, exactly as the reference's scalar loop).
// =====================================================================================
namespace {
constexpr int RT_R = 64, RT_C = 64, RT_K = 32;
}

__global__ void __launch_bounds__(256) residual_rotate_kernel(
    const float* __restrict__ x, const uint32_t* __restrict__ xidx, const float* __restrict__ c,
    const uint32_t* __restrict__ cidx, long long rows, int dim, const float* __restrict__ R,
    float* __restrict__ out) {
    __shared__ __align__(16) float As[RT_R][RT_K + 1];
    __shared__ __align__(16) float Bs[RT_K][RT_C + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long long r0 = (long long)blockIdx.x * RT_R;
    const int j0 = blockIdx.y * RT_C;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < dim; k0 += RT_K) {
        for (int e = tid; e < RT_R * RT_K; e += 256) {
            const int r = e / RT_K, kk = e % RT_K;
            const long long g = r0 + r;
            float v = 0.0f;
            if (g < rows && k0 + kk < dim) {
                const long long xr = xidx ? (long long)xidx[g] : g;
                v = x[xr * dim + k0 + kk];
                if (c) v = __fsub_rn(v, c[(long long)cidx[g] * dim + k0 + kk]);
            }
            As[r][kk] = v;
        }
        for (int e = tid; e < RT_K * RT_C; e += 256) {
            const int kk = e / RT_C, j = e % RT_C;
            Bs[kk][j] = (k0 + kk < dim && j0 + j < dim) ? R[(long long)(k0 + kk) * dim + j0 + j] : 0.0f;
        }
        __syncthreads();
        const int kmax = min(RT_K, dim - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            float a[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[ty * 4 + i][kk];
            const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[i][0] = __fadd_rn(acc[i][0], __fmul_rn(a[i], b.x));
                acc[i][1] = __fadd_rn(acc[i][1], __fmul_rn(a[i], b.y));
                acc[i][2] = __fadd_rn(acc[i][2], __fmul_rn(a[i], b.z));
                acc[i][3] = __fadd_rn(acc[i][3], __fmul_rn(a[i], b.w));
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long g = r0 + ty * 4 + i;
        if (g >= rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = j0 + tx * 4 + j;
            if (col < dim) out[g * dim + col] = acc[i][j];
        }
    }
}

__global__ void residual_copy_kernel(const float* __restrict__ x, const uint32_t* __restrict__ xidx,
                                     const float* __restrict__ c, const uint32_t* __restrict__ cidx,
                                     long long rows, int dim, float* __restrict__ out) {
    const long long total = rows * dim;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / dim;
        const int k = (int)(e % dim);
        const long long xr = xidx ? (long long)xidx[r] : r;
        float v = x[xr * dim + k];
        if (c) v = __fsub_rn(v, c[(long long)cidx[r] * dim + k]);
        out[e] = v;
    }
}

void launch_residual_rotate(const float* x, const uint32_t* xidx, const float* c,
                            const uint32_t* cidx, long long rows, int dim, const float* R,
                            float* out, cudaStream_t st) {
    if (rows <= 0) return;
    if (!R) {
        const long long total = rows * dim;
        const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 32);
        residual_copy_kernel<<<blocks, 256, 0, st>>>(x, xidx, c, cidx, rows, dim, out);
        VGPU_LAUNCH("residual_copy_kernel");
        return;
    }
    dim3 grid(ceil_div(rows, RT_R), ceil_div(dim, RT_C));
    residual_rotate_kernel<<<grid, 256, 0, st>>>(x, xidx, c, cidx, rows, dim, R, out);
    VGPU_LAUNCH("residual_rotate_kernel");
}

void launch_rotate_fast(const float* x, long long rows, int dim, const float* R, float* out,
                        cudaStream_t st) {
    launch_residual_rotate(x, nullptr, nullptr, nullptr, rows, dim, R, out, st);
}

// =====================================================================================
// PQ encode: one thread per (vector, sub-space); the sub-space codebook is staged in
// shared memory when it fits.  Strict `<` from FLT_MAX -> lowest code wins ties
// (find_nearest_code, src/index/pq_fastscan.cpp:78-99).
// =====================================================================================
template <int DS>
__global__ void __launch_bounds__(128) pq_encode_kernel(const float* __restrict__ x, long long n,
                                                        int m, int ksub, int dsub_rt,
                                                        const float* __restrict__ cb,
                                                        uint8_t* __restrict__ codes, int cb_in_smem) {
    extern __shared__ __align__(16) float ycb[];
    const int dsub = DS > 0 ? DS : dsub_rt;
    const int s = blockIdx.y;
    const float* y = cb + (long long)s * ksub * dsub;
    if (cb_in_smem) {
        for (int e = threadIdx.x; e < ksub * dsub; e += blockDim.x) ycb[e] = y[e];
        __syncthreads();
        y = ycb;
    }
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* v = x + i * (long long)m * dsub + (long long)s * dsub;
    float best = FLT_MAX;
    int code = 0;
    if (DS > 0) {
        float vr[DS > 0 ? DS : 1];
#pragma unroll
        for (int e = 0; e < DS; ++e) vr[e] = v[e];
        for (int j = 0; j < ksub; ++j) {
            const float d = l2_ref(vr, y + j * DS, DS);
            if (d < best) { best = d; code = j; }
        }
    } else {
        for (int j = 0; j < ksub; ++j) {
            const float d = l2_ref(v, y + (long long)j * dsub, dsub);
            if (d < best) { best = d; code = j; }
        }
    }
    codes[i * m + s] = (uint8_t)code;
}

void launch_pq_encode(const float* x, long long n, int m, int ksub, int dsub, const float* cb,
                      uint8_t* codes, cudaStream_t st) {
    if (n <= 0) return;
    const size_t cb_bytes = (size_t)ksub * dsub * sizeof(float);
    const int in_smem = cb_bytes <= 96 * 1024 ? 1 : 0;
    const size_t smem = in_smem ? cb_bytes : 0;
    dim3 grid(ceil_div(n, 128), m);
#define VGPU_ENC(DSV)                                                                              \
    do {                                                                                           \
        VGPU_CHECK(cudaFuncSetAttribute(pq_encode_kernel<DSV>,                                     \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));  \
        pq_encode_kernel<DSV><<<grid, 128, smem, st>>>(x, n, m, ksub, dsub, cb, codes, in_smem);   \
    } while (0)
    if (dsub == 4) VGPU_ENC(4);
    else if (dsub == 8) VGPU_ENC(8);
    else if (dsub == 16) VGPU_ENC(16);
    else VGPU_ENC(0);
#undef VGPU_ENC
    VGPU_LAUNCH("pq_encode_kernel");
}

// =====================================================================================
// Exact scan: one CTA per (query, probe rank).  Builds the (query, list) LUT in shared
// memory with l2_ref over each codeword (compute_lookup_tables order), sums each
// entry's LUT values in sub-quantizer order from 0.0f, and keeps the k best of the
// list by (distance, list position).
// =====================================================================================
struct ScanSmemTail {
    float carry_d[kMaxK];
    uint32_t carry_tag[kMaxK];
    uint32_t tag_tmp[kMaxK];
    unsigned long long sortb[kMaxK];
    SelectSmem sel;
};

__global__ void __launch_bounds__(SEL_NT) scan_exact_kernel(
    const float* __restrict__ queries, int dim, const float* __restrict__ centroids,
    const float* __restrict__ rres, const uint32_t* __restrict__ probe, int nprobe,
    const float* __restrict__ cb, int m, int ksub, int dsub, const uint64_t* __restrict__ offs,
    const uint8_t* __restrict__ codes, int k, float* __restrict__ cand_d,
    uint32_t* __restrict__ cand_pos, uint32_t* __restrict__ cand_n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const long long q = blockIdx.x;
    const int t = blockIdx.y;
    const long long pair = q * nprobe + t;
    float* r = reinterpret_cast<float*>(smem_raw);                       // [dim]
    float* lut = r + ((dim + 3) & ~3);                                   // [m * ksub]
    float* buf = lut + (((size_t)m * ksub + 3) & ~(size_t)3);                                 // [kMaxK + SEL_CH]
    ScanSmemTail& S = *reinterpret_cast<ScanSmemTail*>(buf + kMaxK + SEL_CH);

    const uint32_t l = probe[pair];
    if (rres) {
        for (int d = threadIdx.x; d < dim; d += SEL_NT) r[d] = rres[pair * dim + d];
    } else {
        const float* qv = queries + q * dim;
        const float* cv = centroids + (long long)l * dim;
        for (int d = threadIdx.x; d < dim; d += SEL_NT) r[d] = __fsub_rn(qv[d], cv[d]);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < m * ksub; e += SEL_NT) {
        const int s = e / ksub, j = e % ksub;
        lut[e] = l2_ref(r + s * dsub, cb + ((long long)s * ksub + j) * dsub, dsub);
    }
    __syncthreads();
    const uint64_t base = offs[l];
    const long long L = (long long)(offs[l + 1] - base);
    int carry_n = 0;
    for (long long c0 = 0; c0 < L; c0 += SEL_CH) {
        const int cn = (int)min((long long)SEL_CH, L - c0);
        for (int i = threadIdx.x; i < carry_n; i += SEL_NT) buf[i] = S.carry_d[i];
        for (int i = threadIdx.x; i < cn; i += SEL_NT) {
            const uint8_t* code = codes + (base + c0 + i) * (uint64_t)m;
            float dd = 0.0f;
            for (int s = 0; s < m; ++s) dd = __fadd_rn(dd, lut[s * ksub + code[s]]);
            buf[carry_n + i] = dd;
        }
        __syncthreads();
        carry_n = carry_round<SEL_NT>(buf, carry_n, cn, k, S.carry_d, S.carry_tag, S.tag_tmp,
                                      S.sortb, S.sel, (uint32_t)c0);
    }
    for (int i = threadIdx.x; i < carry_n; i += SEL_NT) {
        cand_d[pair * k + i] = S.carry_d[i];
        cand_pos[pair * k + i] = S.carry_tag[i];
    }
    if (threadIdx.x == 0) cand_n[pair] = (uint32_t)carry_n;
}

void launch_scan_exact(const float* queries, long long nq, int dim, const float* centroids,
                       const float* rres, const uint32_t* probe, int nprobe, const float* cb, int m,
                       int ksub, int dsub, const uint64_t* list_offsets, const uint8_t* codes,
                       int k, float* cand_d, uint32_t* cand_pos, uint32_t* cand_n,
                       cudaStream_t st) {
    if (nq <= 0 || nprobe <= 0) return;
    if (k > kMaxK) throw CudaError("scan_exact: k exceeds the supported maximum");
    const size_t smem = ((size_t)((dim + 3) & ~3) + (((size_t)m * ksub + 3) & ~(size_t)3) + kMaxK + SEL_CH) * sizeof(float) +
                        sizeof(ScanSmemTail);
    if (smem > 227 * 1024) throw CudaError("scan_exact: LUT does not fit in shared memory");
    VGPU_CHECK(cudaFuncSetAttribute(scan_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)nq, nprobe);
    scan_exact_kernel<<<grid, SEL_NT, smem, st>>>(queries, dim, centroids, rres, probe, nprobe, cb, m,
                                                  ksub, dsub, list_offsets, codes, k, cand_d, cand_pos,
                                                  cand_n);
    VGPU_LAUNCH("scan_exact_kernel");
}

// =====================================================================================
// Merge per query: candidates of probe rank t sit at [t*k, t*k + cand_n) sorted by
// (distance, list position); concatenated in probe order they are in scan order, so
// the streaming select's position tie-break is the scan-order tie-break.
// =====================================================================================
__global__ void __launch_bounds__(SEL_NT) merge_kernel(
    const float* __restrict__ cand_d, const uint32_t* __restrict__ cand_pos,
    const uint32_t* __restrict__ cand_n, int nprobe, int k, const uint32_t* __restrict__ probe,
    const uint64_t* __restrict__ offs, const uint64_t* __restrict__ ids,
    uint64_t* __restrict__ out_ids, float* __restrict__ out_d, uint32_t* __restrict__ out_n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    TopkSmem& S = *reinterpret_cast<TopkSmem*>(smem_raw);
    __shared__ uint32_t chunk_tags[SEL_CH];
    const long long q = blockIdx.x;
    int carry_n = 0;
    int t = 0;
    while (t < nprobe) {
        // Gather whole probe runs into a chunk of at most SEL_CH entries.
        __shared__ int s_cn, s_tend;
        if (threadIdx.x == 0) {
            int cn = 0, te = t;
            while (te < nprobe) {
                const int c = (int)cand_n[q * nprobe + te];
                if (cn + c > SEL_CH && te > t) break;
                cn += c; ++te;
                if (cn >= SEL_CH) break;
            }
            s_cn = cn; s_tend = te;
        }
        __syncthreads();
        const int cn = s_cn, te = s_tend;
        for (int i = threadIdx.x; i < carry_n; i += SEL_NT) S.buf[i] = S.carry_d[i];
        if (threadIdx.x == 0) {
            int o = 0;
            for (int tt = t; tt < te; ++tt) {
                const int c = (int)cand_n[q * nprobe + tt];
                for (int i = 0; i < c; ++i) chunk_tags[o + i] = ((uint32_t)tt << 16) | (uint32_t)i;
                o += c;
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < cn; i += SEL_NT) {
            const uint32_t tg = chunk_tags[i];
            const long long pair = q * nprobe + (tg >> 16);
            S.buf[carry_n + i] = cand_d[pair * k + (tg & 0xffffu)];
        }
        __syncthreads();
        // Select; map positions to tags (probe << 16 | rank within probe run).
        const int n = carry_n + cn;
        const int got = block_select_k<SEL_NT>(S.buf, n, k, S.sortb, S.sel);
        for (int i = threadIdx.x; i < got; i += SEL_NT) {
            const uint32_t pos = (uint32_t)(S.sortb[i] & 0xffffffffull);
            S.tag_tmp[i] = pos < (uint32_t)carry_n ? S.carry_tag[pos] : chunk_tags[pos - carry_n];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < got; i += SEL_NT) {
            S.carry_d[i] = key_float((uint32_t)(S.sortb[i] >> 32));
            S.carry_tag[i] = S.tag_tmp[i];
        }
        __syncthreads();
        carry_n = got;
        t = te;
    }
    for (int i = threadIdx.x; i < k; i += SEL_NT) {
        if (i < carry_n) {
            const uint32_t tg = S.carry_tag[i];
            const uint32_t tt = tg >> 16, rk = tg & 0xffffu;
            const long long pair = q * nprobe + tt;
            const uint32_t l = probe[pair];
            const uint64_t e = offs[l] + cand_pos[pair * k + rk];
            out_ids[q * k + i] = ids[e];
            out_d[q * k + i] = S.carry_d[i];
        } else {
            out_ids[q * k + i] = 0;
            out_d[q * k + i] = carry_n > 0 ? S.carry_d[carry_n - 1] : 0.0f;
        }
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)carry_n;
}

void launch_merge(const float* cand_d, const uint32_t* cand_pos, const uint32_t* cand_n,
                  long long nq, int nprobe, int k, const uint32_t* probe,
                  const uint64_t* list_offsets, const uint64_t* ids, uint64_t* out_ids,
                  float* out_d, uint32_t* out_n, cudaStream_t st) {
    if (nq <= 0) return;
    if (k > kMaxK || nprobe > 65535) throw CudaError("merge: k or nprobe exceeds the supported maximum");
    const size_t smem = sizeof(TopkSmem);
    VGPU_CHECK(cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    merge_kernel<<<(unsigned)nq, SEL_NT, smem, st>>>(cand_d, cand_pos, cand_n, nprobe, k, probe,
                                                     list_offsets, ids, out_ids, out_d, out_n);
    VGPU_LAUNCH("merge_kernel");
}

// =====================================================================================
// Per-vector term of the fast scan, fp64: u(x) = sum_s ||y||^2 + 2 <(Rc_l)_s, y>.
// One CTA per list.
// =====================================================================================
__global__ void __launch_bounds__(256) vector_terms_kernel(const float* __restrict__ rc, int dim,
                                                           const float* __restrict__ cb, int m,
                                                           int ksub, int dsub,
                                                           const uint64_t* __restrict__ offs,
                                                           const uint8_t* __restrict__ codes,
                                                           float* __restrict__ vterm) {
    const int l = blockIdx.x;
    const float* c = rc + (long long)l * dim;
    for (uint64_t e = offs[l] + threadIdx.x; e < offs[l + 1]; e += blockDim.x) {
        const uint8_t* code = codes + e * (uint64_t)m;
        double u = 0.0;
        for (int s = 0; s < m; ++s) {
            const float* y = cb + ((long long)s * ksub + code[s]) * dsub;
            const float* cs = c + s * dsub;
            for (int t = 0; t < dsub; ++t) {
                const double yv = y[t];
                u += yv * yv + 2.0 * (double)cs[t] * yv;
            }
        }
        vterm[e] = (float)u;
    }
}

void launch_vector_terms(const float* rc, int nlist, int dim, const float* cb, int m, int ksub,
                         int dsub, const uint64_t* list_offsets, const uint8_t* codes,
                         long long n_entries, float* vterm, cudaStream_t st) {
    if (nlist <= 0 || n_entries <= 0) return;
    vector_terms_kernel<<<nlist, 256, 0, st>>>(rc, dim, cb, m, ksub, dsub, list_offsets, codes, vterm);
    VGPU_LAUNCH("vector_terms_kernel");
}

// Sum of the probed lists' sizes (bytes scanned = this * m): one atomic per warp.
__global__ void probe_sizes_kernel(const uint32_t* __restrict__ probe, long long n,
                                   const uint64_t* __restrict__ offs, unsigned long long* out) {
    unsigned long long s = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const uint32_t l = probe[i];
        s += offs[l + 1] - offs[l];
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0 && s) atomicAdd(out, s);
}

void launch_probe_sizes(const uint32_t* probe, long long n, const uint64_t* list_offsets,
                        unsigned long long* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 4);
    probe_sizes_kernel<<<blocks, 256, 0, st>>>(probe, n, list_offsets, out);
    VGPU_LAUNCH("probe_sizes_kernel");
}

// =====================================================================================
// CSR maintenance for add().
// =====================================================================================
__global__ void csr_move_kernel(const uint8_t* __restrict__ old_codes, const uint64_t* __restrict__ old_ids,
                                const uint64_t* __restrict__ old_off, const uint64_t* __restrict__ new_off,
                                int m, uint8_t* __restrict__ codes, uint64_t* __restrict__ ids) {
    const int l = blockIdx.x;
    const uint64_t ob = old_off[l], nb = new_off[l];
    const uint64_t len = old_off[l + 1] - ob;
    for (uint64_t i = threadIdx.x; i < len; i += blockDim.x) ids[nb + i] = old_ids[ob + i];
    for (uint64_t b = threadIdx.x; b < len * m; b += blockDim.x) codes[nb * m + b] = old_codes[ob * m + b];
}

__global__ void csr_scatter_kernel(const uint8_t* __restrict__ new_codes, const uint64_t* __restrict__ new_ids,
                                   const uint64_t* __restrict__ dest, long long n, int m,
                                   uint8_t* __restrict__ codes, uint64_t* __restrict__ ids) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const uint64_t d = dest[i];
        ids[d] = new_ids[i];
        for (int s = 0; s < m; ++s) codes[d * m + s] = new_codes[i * m + s];
    }
}

void launch_csr_move(const uint8_t* old_codes, const uint64_t* old_ids, const uint64_t* old_off,
                     const uint64_t* new_off, int nlist, int m, uint8_t* codes, uint64_t* ids,
                     cudaStream_t st) {
    if (nlist <= 0) return;
    csr_move_kernel<<<nlist, 256, 0, st>>>(old_codes, old_ids, old_off, new_off, m, codes, ids);
    VGPU_LAUNCH("csr_move_kernel");
}

void launch_csr_scatter(const uint8_t* new_codes, const uint64_t* new_ids, const uint64_t* dest,
                        long long n, int m, uint8_t* codes, uint64_t* ids, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    csr_scatter_kernel<<<blocks, 256, 0, st>>>(new_codes, new_ids, dest, n, m, codes, ids);
    VGPU_LAUNCH("csr_scatter_kernel");
}

}  // namespace vgpu

namespace vgpu {

// =====================================================================================
// Fast path, stage 1: per-query lookup tables for a batch of queries,
//   T[q][s][j] = -2 <(Rq)_s, y_sj>.
// CTA = (32 queries, one sub-space): the sub-space codebook is staged once in shared
// memory (transposed, so consecutive codewords are consecutive banks) and reused by
// all 32 queries; outputs are written coalesced along j.
// =====================================================================================
__global__ void __launch_bounds__(256) lut_fast_kernel(const float* __restrict__ rq, long long nq,
                                                       int dim, const float* __restrict__ cb, int m,
                                                       int ksub, int dsub, float* __restrict__ T) {
    extern __shared__ __align__(16) float sm[];
    float* Yt = sm;                       // [dsub][ksub]
    float* Q = sm + (size_t)dsub * ksub;  // [32][dsub]
    const int s = blockIdx.y;
    const long long q0 = (long long)blockIdx.x * 32;
    const float* y = cb + (long long)s * ksub * dsub;
    for (int e = threadIdx.x; e < ksub * dsub; e += blockDim.x) {
        const int j = e / dsub, t = e % dsub;
        Yt[t * ksub + j] = y[e];
    }
    for (int e = threadIdx.x; e < 32 * dsub; e += blockDim.x) {
        const int qi = e / dsub, t = e % dsub;
        Q[e] = (q0 + qi < nq) ? rq[(q0 + qi) * dim + (long long)s * dsub + t] : 0.0f;
    }
    __syncthreads();
    const long long row = (long long)m * ksub;
    for (int e = threadIdx.x; e < 32 * ksub; e += blockDim.x) {
        const int qi = e / ksub, j = e % ksub;
        if (q0 + qi >= nq) continue;
        float acc = 0.0f;
        for (int t = 0; t < dsub; ++t) acc = fmaf(Q[qi * dsub + t], Yt[t * ksub + j], acc);
        T[(q0 + qi) * row + (long long)s * ksub + j] = -2.0f * acc;
    }
}

static size_t lut_fast_smem(int ksub, int dsub) {
    return ((size_t)dsub * ksub + 32 * (size_t)dsub) * sizeof(float);
}

bool lut_fast_fits(int ksub, int dsub) { return lut_fast_smem(ksub, dsub) <= 200 * 1024; }

void launch_lut_fast(const float* rq, long long nq, int dim, const float* cb, int m, int ksub, int dsub,
                     float* T, cudaStream_t st) {
    if (nq <= 0) return;
    const size_t smem = lut_fast_smem(ksub, dsub);
    if (!lut_fast_fits(ksub, dsub)) throw CudaError("lut_fast: sub-space codebook too large for shared memory");
    VGPU_CHECK(cudaFuncSetAttribute(lut_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(ceil_div(nq, 32), m);
    lut_fast_kernel<<<grid, 256, smem, st>>>(rq, nq, dim, cb, m, ksub, dsub, T);
    VGPU_LAUNCH("lut_fast_kernel");
}

// =====================================================================================
// Fast path, stage 2: inverted-list scan with a running top-k.
//
// One CTA per query; the query's table (m x ksub fp32) is copied into shared memory.
// Lists are scanned in probe order, 256 entries per round (one per thread).  Each
// entry gets the 64-bit key (order-preserving distance bits << 32 | scan position);
// only keys below the current k-th key tau are appended to a shared candidate buffer,
// which is merged with the running top-k (bitonic sort) when it could overflow and at
// the end.  The key order is (distance, scan position), so ties resolve to the earlier
// scanned entry, as in the exact path.
// =====================================================================================
namespace {
constexpr int FS_NT = 256;
constexpr int FS_CB = 512;   // candidate buffer entries (>= 2 rounds of FS_NT)
}

template <int MC>
__device__ __forceinline__ float adc_sum(const uint8_t* __restrict__ code, const float* __restrict__ lut,
                                         int m_rt, int ksub) {
    float acc = 0.0f;
    if (MC > 0) {
        const uint4* c4 = reinterpret_cast<const uint4*>(code);
#pragma unroll
        for (int v = 0; v < MC / 16; ++v) {
            const uint4 w = __ldg(c4 + v);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const uint32_t byte = (words[b >> 2] >> ((b & 3) * 8)) & 0xffu;
                acc = __fadd_rn(acc, lut[(v * 16 + b) * ksub + byte]);
            }
        }
    } else {
        for (int s = 0; s < m_rt; ++s) acc = __fadd_rn(acc, lut[s * ksub + code[s]]);
    }
    return acc;
}

template <int MC>
__global__ void __launch_bounds__(FS_NT, 2) scan_fast2_kernel(
    const float* __restrict__ T, const float* __restrict__ rq, int dim,
    const uint32_t* __restrict__ probe, const float* __restrict__ probe_d, const float* __restrict__ rc,
    int nprobe, int m_rt, int ksub, const uint64_t* __restrict__ offs, const uint8_t* __restrict__ codes,
    const float* __restrict__ vterm, const uint64_t* __restrict__ ids, int k, int kp2, int bp2,
    uint64_t* __restrict__ out_ids, float* __restrict__ out_d, uint32_t* __restrict__ out_n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int m = MC > 0 ? MC : m_rt;
    float* lut = reinterpret_cast<float*>(smem_raw);                              // [m*ksub]
    unsigned long long* buf = reinterpret_cast<unsigned long long*>(lut + (((size_t)m * ksub + 3) & ~(size_t)3));
    unsigned long long* top = buf + bp2;                                          // [kp2]
    uint32_t* prefix = reinterpret_cast<uint32_t*>(top + kp2);                     // [nprobe + 1]
    __shared__ uint32_t cnt;
    __shared__ int have;
    __shared__ unsigned long long tau;
    __shared__ float s_base;

    const long long q = blockIdx.x;
    {
        const float4* src = reinterpret_cast<const float4*>(T + q * (long long)m * ksub);
        float4* dst = reinterpret_cast<float4*>(lut);
        const int n4 = (m * ksub) >> 2;
        for (int i = threadIdx.x; i < n4; i += FS_NT) dst[i] = __ldg(src + i);
        for (int i = (n4 << 2) + threadIdx.x; i < m * ksub; i += FS_NT) lut[i] = T[q * (long long)m * ksub + i];
    }
    if (threadIdx.x == 0) { cnt = 0; have = 0; tau = ~0ull; }
    __syncthreads();

    auto merge = [&]() {
        // buf[0..cnt) candidates; append the current top, sort, keep k.
        const int c = (int)cnt, h = have;
        const int n = c + h;
        const int p2 = next_pow2(n < 2 ? 2 : n);
        for (int i = threadIdx.x; i < h; i += FS_NT) buf[c + i] = top[i];
        for (int i = n + threadIdx.x; i < p2; i += FS_NT) buf[i] = ~0ull;
        bitonic_sort_u64<FS_NT>(buf, p2);
        const int nh = n < k ? n : k;
        for (int i = threadIdx.x; i < nh; i += FS_NT) top[i] = buf[i];
        __syncthreads();
        if (threadIdx.x == 0) {
            have = nh;
            cnt = 0;
            tau = (nh == k) ? top[k - 1] : ~0ull;
        }
        __syncthreads();
    };

    uint32_t seq_base = 0;
    for (int t = 0; t < nprobe; ++t) {
        const long long pr = q * nprobe + t;
        const uint32_t l = probe[pr];
        if (threadIdx.x == 0) prefix[t] = seq_base;
        if (rc) {
            if (threadIdx.x < 32) {
                const float* cl = rc + (long long)l * dim;
                const float* qv = rq + q * dim;
                float acc = 0.0f;
                for (int d = threadIdx.x; d < dim; d += 32) {
                    const float df = qv[d] - cl[d];
                    acc = fmaf(df, df, acc);
                }
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (threadIdx.x == 0) s_base = acc;
            }
        } else if (threadIdx.x == 0) {
            s_base = probe_d[pr];
        }
        __syncthreads();
        const float base_d = s_base;
        const uint64_t b = offs[l];
        const uint32_t L = (uint32_t)(offs[l + 1] - b);
        for (uint32_t r0 = 0; r0 < L; r0 += FS_NT) {
            const uint32_t i = r0 + threadIdx.x;
            if (i < L) {
                const uint64_t e = b + i;
                const float acc = adc_sum<MC>(codes + e * (uint64_t)m, lut, m, ksub);
                const float dist = __fadd_rn(__fadd_rn(base_d, __ldg(vterm + e)), acc);
                const unsigned long long key = ((unsigned long long)float_key(dist) << 32) | (seq_base + i);
                if (key < tau) {
                    const uint32_t slot = atomicAdd(&cnt, 1u);
                    buf[slot] = key;
                }
            }
            __syncthreads();
            if (cnt > (uint32_t)(FS_CB - FS_NT)) merge();
        }
        seq_base += L;
    }
    if (threadIdx.x == 0) prefix[nprobe] = seq_base;
    __syncthreads();
    if (cnt > 0) merge();
    const int h = have;
    for (int i = threadIdx.x; i < k; i += FS_NT) {
        if (i < h) {
            const unsigned long long key = top[i];
            const uint32_t sq = (uint32_t)(key & 0xffffffffull);
            int lo = 0, hi = nprobe;  // find t with prefix[t] <= sq < prefix[t+1]
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (prefix[mid] <= sq) lo = mid; else hi = mid;
            }
            // skip empty lists that share the same prefix value
            while (lo + 1 < nprobe && prefix[lo + 1] <= sq) ++lo;
            const uint32_t l = probe[q * nprobe + lo];
            out_ids[q * k + i] = ids[offs[l] + (sq - prefix[lo])];
            out_d[q * k + i] = key_float((uint32_t)(key >> 32));
        } else {
            out_ids[q * k + i] = 0;
            out_d[q * k + i] = h > 0 ? key_float((uint32_t)(top[h - 1] >> 32)) : 0.0f;
        }
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)h;
}

static size_t scan_fast2_smem(int m, int ksub, int k, int nprobe) {
    const int kp2 = next_pow2(k < 2 ? 2 : k);
    const int bp2 = next_pow2(FS_CB + kp2);
    return (((size_t)m * ksub + 3) & ~(size_t)3) * sizeof(float) +
           (size_t)(bp2 + kp2) * sizeof(unsigned long long) + (size_t)(nprobe + 1) * 4;
}

bool scan_fast2_fits(int m, int ksub, int k, int nprobe) {
    return k >= 1 && k <= kMaxK && scan_fast2_smem(m, ksub, k, nprobe) <= 227 * 1024;
}

void launch_scan_fast2(const float* T, const float* rq, long long nq, int dim, const uint32_t* probe,
                       const float* probe_d, const float* rc, int nprobe, int m, int ksub,
                       const uint64_t* list_offsets, const uint8_t* codes, const float* vterm,
                       const uint64_t* ids, int k, uint64_t* out_ids, float* out_d, uint32_t* out_n,
                       cudaStream_t st) {
    if (nq <= 0) return;
    if (k > kMaxK) throw CudaError("scan_fast: k exceeds the supported maximum");
    const int kp2 = next_pow2(k < 2 ? 2 : k);
    const int bp2 = next_pow2(FS_CB + kp2);   // merge buffer: candidates + current top, padded
    const size_t smem = scan_fast2_smem(m, ksub, k, nprobe);
    if (!scan_fast2_fits(m, ksub, k, nprobe))
        throw CudaError("scan_fast: lookup table does not fit in shared memory");
#define VGPU_SF2(MCV)                                                                             \
    do {                                                                                          \
        VGPU_CHECK(cudaFuncSetAttribute(scan_fast2_kernel<MCV>,                                   \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        scan_fast2_kernel<MCV><<<(unsigned)nq, FS_NT, smem, st>>>(                                \
            T, rq, dim, probe, probe_d, rc, nprobe, m, ksub, list_offsets, codes, vterm, ids, k,  \
            kp2, bp2, out_ids, out_d, out_n);                                                     \
    } while (0)
    if (m == 16) VGPU_SF2(16);
    else if (m == 32) VGPU_SF2(32);
    else if (m == 64) VGPU_SF2(64);
    else if (m == 96) VGPU_SF2(96);
    else VGPU_SF2(0);
#undef VGPU_SF2
    VGPU_LAUNCH("scan_fast2_kernel");
}

}  // namespace vgpu

namespace vgpu {

// =====================================================================================
// Fast path, blocked layout ("scan layout").
//
// Each list is cut into blocks of 128 entries (the last one padded).  Inside a block,
// lane l of a warp owns entries 4l..4l+3 and at step r looks up sub-space
//   s(l, r) = G*floor(r/G) + ((l + r) mod G),     G = 32 (or 16/8/4 when m is smaller),
// so the 32 lanes of a warp touch 32 different sub-spaces at every step.  The block
// stores, for each step r, each lane's 4 code bytes as one word, 4 steps per 16-byte
// segment, lane-contiguous:  byte((r/4*32 + l)*16 + (r%4)*4 + j) = code(4l + j, s(l, r)),
// so a warp reads a block with fully coalesced 16-byte loads and no staging.  The
// per-query table is laid out as Tb[(g*256 + c)*G + (s mod G)] (g = s / G): the bank of
// a lookup is its sub-space, and the lookups of one step never conflict.
// =====================================================================================

__host__ __device__ inline int scan_group(int m) {
    return (m % 32 == 0) ? 32 : (m % 16 == 0) ? 16 : (m % 8 == 0) ? 8 : (m % 4 == 0) ? 4 : 0;
}

// One thread per (entry, sub-space) of the CSR codes -> blocked layout; vterm likewise.
__global__ void build_blocks_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ vterm,
                                    const uint64_t* __restrict__ offs, const uint64_t* __restrict__ blk_off,
                                    int m, int G, int nlist, uint8_t* __restrict__ bcodes,
                                    float* __restrict__ bvterm) {
    const int l = blockIdx.x;
    const uint64_t b0 = offs[l];
    const uint64_t L = offs[l + 1] - b0;
    const uint64_t nb = blk_off[l + 1] - blk_off[l];
    const uint64_t total = nb * 128 * (uint64_t)m;
    for (uint64_t e = threadIdx.x; e < total; e += blockDim.x) {
        const uint64_t p = e / m;            // position in list (padded)
        const int s = (int)(e % m);
        const uint64_t blk = blk_off[l] + p / 128;
        const int c = (int)(p % 128), lane = c >> 2, j = c & 3;
        const int g = s / G, s_lo = s % G;
        const int r = g * G + ((s_lo - lane) % G + G) % G;
        const uint64_t off = blk * 128ull * m + (uint64_t)((r >> 2) * 32 + lane) * 16 + (r & 3) * 4 + j;
        bcodes[off] = p < L ? codes[(b0 + p) * (uint64_t)m + s] : (uint8_t)0;
        if (s == 0) bvterm[blk * 128 + c] = p < L ? vterm[b0 + p] : 0.0f;
    }
}

void launch_build_blocks(const uint8_t* codes, const float* vterm, const uint64_t* offs, const uint64_t* blk_off,
                         int m, int nlist, uint8_t* bcodes, float* bvterm, cudaStream_t st) {
    const int G = scan_group(m);
    if (G == 0) throw CudaError("build_blocks: m must be a multiple of 4");
    if (nlist <= 0) return;
    build_blocks_kernel<<<nlist, 256, 0, st>>>(codes, vterm, offs, blk_off, m, G, nlist, bcodes, bvterm);
    VGPU_LAUNCH("build_blocks_kernel");
}

// Tables in the blocked order, T[q][(g*256 + c)*G + s_lo] = -2 <(Rq)_s, y_sc>.
// A CTA owns one sub-space group g, 64 codes and 32 queries: it stages those codes'
// sub-vectors and the queries' slices of the group's G sub-spaces in shared memory once,
// then writes each query's 64 x G contiguous table entries (thread e -> query, code,
// sub-space), with no barrier between queries.
namespace {
constexpr int LB_C = 64;    // codes per CTA
constexpr int LB_Q = 32;    // queries per CTA
}

__global__ void __launch_bounds__(256) lut_blocked_kernel(const float* __restrict__ rq, long long nq, int dim,
                                                          const float* __restrict__ cb, int m, int dsub, int G,
                                                          float* __restrict__ T) {
    extern __shared__ __align__(16) float sm[];
    float* ys = sm;                                 // [LB_C][dsub][G]
    float* qs = ys + (size_t)LB_C * dsub * G;       // [LB_Q][dsub][G]
    const int g = blockIdx.y, c0 = blockIdx.z * LB_C;
    for (int e = threadIdx.x; e < LB_C * dsub * G; e += blockDim.x) {
        const int s_lo = e % G, t = (e / G) % dsub, c = e / (G * dsub);
        ys[e] = cb[((long long)(g * G + s_lo) * 256 + c0 + c) * dsub + t];
    }
    // every query's slice of the group's sub-spaces at once (coalesced: t fastest)
    const long long qb = (long long)blockIdx.x * LB_Q;
    const int nqq = (int)min((long long)LB_Q, nq - qb);
    for (int e = threadIdx.x; e < nqq * dsub * G; e += blockDim.x) {
        const int qi = e / (dsub * G), r = e % (dsub * G), t = r % dsub, s_lo = r / dsub;
        qs[(qi * dsub + t) * G + s_lo] = rq[(qb + qi) * dim + (long long)g * G * dsub + r];
    }
    __syncthreads();
    const long long row = (long long)m * 256;
    const int per_q = LB_C * G;
    for (int e = threadIdx.x; e < nqq * per_q; e += blockDim.x) {
        const int qi = e / per_q, r = e % per_q, c = r / G, s_lo = r % G;
        float acc = 0.0f;
        for (int t = 0; t < dsub; ++t)
            acc = fmaf(qs[(qi * dsub + t) * G + s_lo], ys[(c * dsub + t) * G + s_lo], acc);
        T[(qb + qi) * row + ((long long)g * 256 + c0) * G + r] = -2.0f * acc;
    }
}

// The same tables with each thread's entries fixed: thread x owns entries r = x + 256 j
// (j < R = G / 4) of every query, which share the sub-space s_lo = x % G, so it keeps
// their codebook sub-vectors in registers, reads one query slice per query from shared
// memory, and writes R coalesced entries per query.  No integer division per entry;
// the store of T is the bound.  Same arithmetic, same order as lut_blocked_kernel.
template <int DSUB, int R>
__global__ void __launch_bounds__(256) lut_blocked_reg_kernel(const float* __restrict__ rq, long long nq, int dim,
                                                              const float* __restrict__ cb, int m, int G,
                                                              float* __restrict__ T) {
    extern __shared__ __align__(16) float qs[];     // [LB_Q][DSUB][G]
    const int g = blockIdx.y, c0 = blockIdx.z * LB_C;
    const long long qb = (long long)blockIdx.x * LB_Q;
    const int nqq = (int)min((long long)LB_Q, nq - qb);
    for (int e = threadIdx.x; e < nqq * DSUB * G; e += blockDim.x) {
        const int qi = e / (DSUB * G), r = e % (DSUB * G), t = r % DSUB, s_lo = r / DSUB;
        qs[(qi * DSUB + t) * G + s_lo] = rq[(qb + qi) * dim + (long long)g * G * DSUB + r];
    }
    const int s_lo = threadIdx.x % G;
    float y[R][DSUB];
#pragma unroll
    for (int j = 0; j < R; ++j) {
        const int c = (threadIdx.x + 256 * j) / G;
        const float* src = cb + ((long long)(g * G + s_lo) * 256 + c0 + c) * DSUB;
#pragma unroll
        for (int t = 0; t < DSUB; ++t) y[j][t] = src[t];
    }
    __syncthreads();
    const long long row = (long long)m * 256;
    float* Tb = T + qb * row + ((long long)g * 256 + c0) * G + threadIdx.x;
    for (int qi = 0; qi < nqq; ++qi) {
        float qv[DSUB];
#pragma unroll
        for (int t = 0; t < DSUB; ++t) qv[t] = qs[(qi * DSUB + t) * G + s_lo];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            float acc = 0.0f;
#pragma unroll
            for (int t = 0; t < DSUB; ++t) acc = fmaf(qv[t], y[j][t], acc);
            Tb[qi * row + 256 * j] = -2.0f * acc;
        }
    }
}

// The same with 16-byte accesses, for groups of 16 or 32 sub-spaces (R = G / 4 >= 4
// entries per thread): thread x owns the quads of entries r = 4 (x + 256 h) + e, which
// share a code and four consecutive sub-spaces, so a query's slice is read as DSUB
// float4 loads and each quad is written with one float4 store.  Same arithmetic, same
// order per entry.
template <int DSUB, int R>
__global__ void __launch_bounds__(256) lut_blocked_vec_kernel(const float* __restrict__ rq, long long nq, int dim,
                                                              const float* __restrict__ cb, int m, int G,
                                                              float* __restrict__ T) {
    extern __shared__ __align__(16) float qs[];     // [LB_Q][DSUB][G]
    constexpr int H = R / 4;                        // quads per thread
    const int g = blockIdx.y, c0 = blockIdx.z * LB_C;
    const long long qb = (long long)blockIdx.x * LB_Q;
    const int nqq = (int)min((long long)LB_Q, nq - qb);
    for (int e = threadIdx.x; e < nqq * DSUB * G; e += blockDim.x) {
        const int qi = e / (DSUB * G), r = e % (DSUB * G), t = r % DSUB, s_lo = r / DSUB;
        qs[(qi * DSUB + t) * G + s_lo] = rq[(qb + qi) * dim + (long long)g * G * DSUB + r];
    }
    const int s0 = (4 * threadIdx.x) % G;           // the same for every quad of the thread
    float y[H][4][DSUB];
#pragma unroll
    for (int h = 0; h < H; ++h) {
        const int c = 4 * (threadIdx.x + 256 * h) / G;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float* src = cb + ((long long)(g * G + s0 + e) * 256 + c0 + c) * DSUB;
#pragma unroll
            for (int t = 0; t < DSUB; ++t) y[h][e][t] = src[t];
        }
    }
    __syncthreads();
    const long long row = (long long)m * 256;
    float* Tb = T + qb * row + ((long long)g * 256 + c0) * G + 4 * threadIdx.x;
    for (int qi = 0; qi < nqq; ++qi) {
        float4 qv[DSUB];
#pragma unroll
        for (int t = 0; t < DSUB; ++t) qv[t] = *reinterpret_cast<const float4*>(&qs[(qi * DSUB + t) * G + s0]);
#pragma unroll
        for (int h = 0; h < H; ++h) {
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
            for (int t = 0; t < DSUB; ++t) {
                a0 = fmaf(qv[t].x, y[h][0][t], a0);
                a1 = fmaf(qv[t].y, y[h][1][t], a1);
                a2 = fmaf(qv[t].z, y[h][2][t], a2);
                a3 = fmaf(qv[t].w, y[h][3][t], a3);
            }
            *reinterpret_cast<float4*>(Tb + qi * row + 1024 * h) =
                make_float4(-2.0f * a0, -2.0f * a1, -2.0f * a2, -2.0f * a3);
        }
    }
}

namespace {
template <int DSUB, int R>
bool lut_reg_launch(const float* rq, long long nq, int dim, const float* cb, int m, int G, float* T, cudaStream_t st) {
    const size_t smem = (size_t)LB_Q * DSUB * G * sizeof(float);
    VGPU_CHECK(cudaFuncSetAttribute(lut_blocked_reg_kernel<DSUB, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    dim3 grid(ceil_div(nq, LB_Q), m / G, 256 / LB_C);
    if constexpr (R >= 4) {
        // float4 stores: every store offset is a multiple of 4 floats (row = m * 256,
        // G a multiple of 4), so only the table's own address needs 16-byte alignment.
        if (!std::getenv("VGPU_LUT_SCALAR") && reinterpret_cast<uintptr_t>(T) % 16 == 0) {
            VGPU_CHECK(cudaFuncSetAttribute(lut_blocked_vec_kernel<DSUB, R>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            lut_blocked_vec_kernel<DSUB, R><<<grid, 256, smem, st>>>(rq, nq, dim, cb, m, G, T);
            VGPU_LAUNCH("lut_blocked_vec_kernel");
            return true;
        }
    }
    lut_blocked_reg_kernel<DSUB, R><<<grid, 256, smem, st>>>(rq, nq, dim, cb, m, G, T);
    VGPU_LAUNCH("lut_blocked_reg_kernel");
    return true;
}

template <int DSUB>
bool lut_reg_dispatch(const float* rq, long long nq, int dim, const float* cb, int m, int G, float* T,
                      cudaStream_t st) {
    const int R = LB_C * G / 256;
    if (R * DSUB > 64) return false;
    switch (R) {
        case 1: return lut_reg_launch<DSUB, 1>(rq, nq, dim, cb, m, G, T, st);
        case 2: return lut_reg_launch<DSUB, 2>(rq, nq, dim, cb, m, G, T, st);
        case 4: return lut_reg_launch<DSUB, 4>(rq, nq, dim, cb, m, G, T, st);
        case 8:
            if constexpr (DSUB <= 8) return lut_reg_launch<DSUB, 8>(rq, nq, dim, cb, m, G, T, st);
            return false;
        default: return false;
    }
}
}  // namespace

void launch_lut_blocked(const float* rq, long long nq, int dim, const float* cb, int m, int dsub, float* T,
                        cudaStream_t st) {
    if (nq <= 0) return;
    const int G = scan_group(m);
    if (G > 0 && 256 % G == 0 && !std::getenv("VGPU_LUT_GENERIC")) {
        bool done = false;
        switch (dsub) {
            case 2: done = lut_reg_dispatch<2>(rq, nq, dim, cb, m, G, T, st); break;
            case 4: done = lut_reg_dispatch<4>(rq, nq, dim, cb, m, G, T, st); break;
            case 8: done = lut_reg_dispatch<8>(rq, nq, dim, cb, m, G, T, st); break;
            case 16: done = lut_reg_dispatch<16>(rq, nq, dim, cb, m, G, T, st); break;
            default: break;
        }
        if (done) return;
    }
    const size_t smem = ((size_t)LB_C * dsub * G + (size_t)LB_Q * dsub * G) * sizeof(float);
    if (smem > 200 * 1024) throw CudaError("lut_blocked: sub-space codebook slice too large for shared memory");
    VGPU_CHECK(cudaFuncSetAttribute(lut_blocked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid(ceil_div(nq, LB_Q), m / G, 256 / LB_C);
    lut_blocked_kernel<<<grid, 256, smem, st>>>(rq, nq, dim, cb, m, dsub, G, T);
    VGPU_LAUNCH("lut_blocked_kernel");
}

namespace {
constexpr int FB_NT = 512;                    // 16 warps; one 128-entry block per warp per round
constexpr int FB_WARPS = FB_NT / 32;
constexpr int FB_ROUND = FB_WARPS * 128;      // entries per round
constexpr int FB_CB = FB_ROUND;               // candidate buffer: one round (merged every round)
constexpr int FB_PF = 8;                      // 16-byte code segments a lane keeps in flight
}

template <int MC, int G>
__global__ void __launch_bounds__(FB_NT, 1) scan_blocked_kernel(
    const float* __restrict__ T, const float* __restrict__ pbase, const uint32_t* __restrict__ probe,
    int nprobe, int nscan, const uint64_t* __restrict__ offs, const uint64_t* __restrict__ blk_off,
    const uint8_t* __restrict__ bcodes, const float* __restrict__ bvterm, const uint64_t* __restrict__ ids,
    int k, int kp2, int bp2, uint64_t* __restrict__ out_ids, float* __restrict__ out_d,
    uint32_t* __restrict__ out_n, const uint32_t* __restrict__ only_over, uint32_t over_cap,
    const uint4* __restrict__ items, unsigned long long* __restrict__ part_keys) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int m = MC;
    float* lut = reinterpret_cast<float*>(smem_raw);                                   // [m*256]
    unsigned long long* buf = reinterpret_cast<unsigned long long*>(lut + m * 256);     // [bp2]
    unsigned long long* top = buf + bp2;                                               // [kp2]
    uint32_t* eprefix = reinterpret_cast<uint32_t*>(top + kp2);                         // [nscan+1]
    uint32_t* bprefix = eprefix + (nscan + 1);                                         // [nscan+1]
    float* base = reinterpret_cast<float*>(bprefix + (nscan + 1));                      // [nscan]
    __shared__ uint32_t cnt;
    __shared__ int have;
    __shared__ unsigned long long tau;

    // Split mode (items != nullptr): this CTA scans blocks [b_begin, b_end) of query
    // items[blockIdx.x].x and writes its k smallest keys to part_keys.
    const long long q = items ? (long long)items[blockIdx.x].x : (long long)blockIdx.x;
    if (!items && only_over && only_over[q] <= over_cap) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // The query's table arrives by one bulk copy while the prefixes are computed.
    __shared__ uint64_t lut_bar;
    const float* tq = T + q * (long long)m * 256;
    tc::lut_stage_begin(lut, tq, (uint32_t)(m * 256 * 4), &lut_bar);
    // Per-probe prefixes (entries, blocks) and base terms.
    if (threadIdx.x < 32) probe_prefixes_warp(probe + q * nprobe, nscan, offs, blk_off, eprefix, bprefix);
    if (threadIdx.x == 0) { cnt = 0; have = 0; tau = ~0ull; }
    for (int t = threadIdx.x; t < nscan; t += FB_NT) base[t] = pbase[q * nprobe + t];
    tc::lut_stage_wait(lut, tq, (uint32_t)(m * 256 * 4), &lut_bar);
    (void)lane;

    auto merge = [&]() {
        const int c = (int)cnt, h = have;
        const int n = c + h;
        const int p2 = next_pow2(n < 2 ? 2 : n);
        for (int i = threadIdx.x; i < h; i += FB_NT) buf[c + i] = top[i];
        for (int i = n + threadIdx.x; i < p2; i += FB_NT) buf[i] = ~0ull;
        bitonic_sort_u64<FB_NT>(buf, p2);
        const int nh = n < k ? n : k;
        for (int i = threadIdx.x; i < nh; i += FB_NT) top[i] = buf[i];
        __syncthreads();
        if (threadIdx.x == 0) { have = nh; cnt = 0; tau = (nh == k) ? top[k - 1] : ~0ull; }
        __syncthreads();
    };

    const uint32_t NB = items ? min(items[blockIdx.x].z, bprefix[nscan]) : bprefix[nscan];
    const uint32_t B0 = items ? items[blockIdx.x].y : 0u;
    for (uint32_t r0 = B0; r0 < NB; r0 += FB_WARPS) {
        const uint32_t bi = r0 + warp;
        if (bi < NB) {
            int lo = 0, hi = nscan;  // largest t with bprefix[t] <= bi
            while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (bprefix[mid] <= bi) lo = mid; else hi = mid; }
            const uint32_t l = probe[q * nprobe + lo];
            const uint32_t b = bi - bprefix[lo];
            const uint64_t gblk = blk_off[l] + b;
            const uint32_t L = eprefix[lo + 1] - eprefix[lo];
            const uint4* src = reinterpret_cast<const uint4*>(bcodes + gblk * 128ull * m) + lane;
            float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
            // m/4 segments of 16 bytes per lane, fetched FB_PF at a time ahead of use.
#pragma unroll
            for (int r0 = 0; r0 < m / 4; r0 += FB_PF) {
                uint4 w[FB_PF];
#pragma unroll
                for (int u = 0; u < FB_PF; ++u)
                    if (r0 + u < m / 4) w[u] = __ldg(src + (r0 + u) * 32);
#pragma unroll
                for (int u = 0; u < FB_PF; ++u) {
                    if (r0 + u >= m / 4) break;
                    const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const int r = (r0 + u) * 4 + jj;
                        const int g = r / G;
                        const int s_lo = (lane + r) & (G - 1);
                        const float* tb = lut + (g * 256) * G + s_lo;
                        const uint32_t v = ws[jj];
                        acc0 += tb[(v & 0xffu) * G];
                        acc1 += tb[((v >> 8) & 0xffu) * G];
                        acc2 += tb[((v >> 16) & 0xffu) * G];
                        acc3 += tb[(v >> 24) * G];
                    }
                }
            }
            const float4 vt = __ldg(reinterpret_cast<const float4*>(bvterm + gblk * 128) + lane);
            const float bd = base[lo];
            const float accs[4] = {acc0, acc1, acc2, acc3};
            const float vts[4] = {vt.x, vt.y, vt.z, vt.w};
            const uint32_t p0 = b * 128 + lane * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t p = p0 + j;
                if (p < L) {
                    const float dist = (bd + vts[j]) + accs[j];
                    const unsigned long long key =
                        ((unsigned long long)float_key(dist) << 32) | (eprefix[lo] + p);
                    if (key < tau) {
                        const uint32_t slot = atomicAdd(&cnt, 1u);
                        buf[slot] = key;
                    }
                }
            }
        }
        __syncthreads();
        if (cnt > 0) merge();
    }
    const int h = have;
    if (part_keys) {
        for (int i = threadIdx.x; i < k; i += FB_NT) part_keys[(long long)blockIdx.x * k + i] = i < h ? top[i] : ~0ull;
        return;
    }
    for (int i = threadIdx.x; i < k; i += FB_NT) {
        if (i < h) {
            const unsigned long long key = top[i];
            const uint32_t sq = (uint32_t)(key & 0xffffffffull);
            int lo = 0, hi = nscan;
            while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (eprefix[mid] <= sq) lo = mid; else hi = mid; }
            const uint32_t l = probe[q * nprobe + lo];
            out_ids[q * k + i] = ids[offs[l] + (sq - eprefix[lo])];
            out_d[q * k + i] = key_float((uint32_t)(key >> 32));
        } else {
            out_ids[q * k + i] = 0;
            out_d[q * k + i] = h > 0 ? key_float((uint32_t)(top[h - 1] >> 32)) : 0.0f;
        }
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)h;
}

// Base term of every (query, probe) pair: ||Rq - R c_l||^2 (lane-strided fp32 FMAs
// and a butterfly sum, one warp per pair) when rotated centroids are given, else the
// coarse distance.  Shared by the blocked scan and the tensor-core list scan so both
// see the same value.
__global__ void probe_base_kernel(const float* __restrict__ rq, int dim, const uint32_t* __restrict__ probe,
                                  const float* __restrict__ probe_d, const float* __restrict__ rc, int nprobe,
                                  long long npairs, float* __restrict__ pbase) {
    const int lane = threadIdx.x & 31;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long pr = w; pr < npairs; pr += nw) {
        float b;
        if (rc) {
            const float* cl = rc + (long long)probe[pr] * dim;
            const float* qv = rq + (pr / nprobe) * dim;
            float acc = 0.0f;
            for (int d = lane; d < dim; d += 32) {
                const float df = qv[d] - cl[d];
                acc = fmaf(df, df, acc);
            }
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            b = acc;
        } else {
            b = probe_d[pr];
        }
        if (lane == 0) pbase[pr] = b;
    }
}

void launch_probe_base(const float* rq, long long nq, int dim, const uint32_t* probe, const float* probe_d,
                       const float* rc, int nprobe, float* pbase, cudaStream_t st) {
    const long long npairs = nq * nprobe;
    if (npairs <= 0) return;
    const int blocks = (int)std::min<long long>((npairs * 32 + 255) / 256, 148LL * 32);
    probe_base_kernel<<<blocks, 256, 0, st>>>(rq, dim, probe, probe_d, rc, nprobe, npairs, pbase);
    VGPU_LAUNCH("probe_base_kernel");
}

bool scan_blocked_supported(int m, int ksub) {
    return ksub == 256 && (m == 16 || m == 32 || m == 64 || m == 96 || m == 128);
}

namespace {
void scan_blocked_impl(const float* T, long long grid, const float* pbase, const uint32_t* probe, int nprobe,
                       int nscan, int m, const uint64_t* offs, const uint64_t* blk_off, const uint8_t* bcodes,
                       const float* bvterm, const uint64_t* ids, int k, uint64_t* out_ids, float* out_d,
                       uint32_t* out_n, const uint32_t* only_over, uint32_t over_cap, const uint4* items,
                       unsigned long long* part_keys, cudaStream_t st) {
    const long long nq = grid;
    if (nq <= 0) return;
    if (nscan < 1 || nscan > nprobe) throw CudaError("scan_blocked: nscan must be in [1, nprobe]");
    if (k > kMaxK) throw CudaError("scan_blocked: k exceeds the supported maximum");
    const int kp2 = next_pow2(k < 2 ? 2 : k);
    const int bp2 = next_pow2(FB_CB + kp2);
    const size_t smem = (size_t)m * 256 * sizeof(float) + (size_t)(bp2 + kp2) * sizeof(unsigned long long) +
                        (size_t)(nscan + 1) * 8 + (size_t)nscan * 4;
    if (smem > 227 * 1024) throw CudaError("scan_blocked: lookup table does not fit in shared memory");
#define VGPU_SB(MCV, GV)                                                                          \
    do {                                                                                          \
        VGPU_CHECK(cudaFuncSetAttribute(scan_blocked_kernel<MCV, GV>,                             \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        scan_blocked_kernel<MCV, GV><<<(unsigned)nq, FB_NT, smem, st>>>(                          \
            T, pbase, probe, nprobe, nscan, offs, blk_off, bcodes, bvterm, ids, k, kp2, bp2,      \
            out_ids, out_d, out_n, only_over, over_cap, items, part_keys);                        \
    } while (0)
    if (m == 16) VGPU_SB(16, 16);
    else if (m == 32) VGPU_SB(32, 32);
    else if (m == 64) VGPU_SB(64, 32);
    else if (m == 96) VGPU_SB(96, 32);
    else if (m == 128) VGPU_SB(128, 32);
    else throw CudaError("scan_blocked: unsupported m");
#undef VGPU_SB
    VGPU_LAUNCH("scan_blocked_kernel");
}
}  // namespace

void launch_scan_blocked(const float* T, long long nq, const float* pbase, const uint32_t* probe, int nprobe,
                         int nscan, int m, const uint64_t* offs, const uint64_t* blk_off, const uint8_t* bcodes,
                         const float* bvterm, const uint64_t* ids, int k, uint64_t* out_ids, float* out_d,
                         uint32_t* out_n, const uint32_t* only_over, uint32_t over_cap, cudaStream_t st) {
    scan_blocked_impl(T, nq, pbase, probe, nprobe, nscan, m, offs, blk_off, bcodes, bvterm, ids, k, out_ids, out_d,
                      out_n, only_over, over_cap, nullptr, nullptr, st);
}

// ---------------------------------------------------------------------------------
// Split blocked scan: a query's blocks are cut into parts of at most SPLIT_BLOCKS
// blocks, each scanned by its own CTA (keys = (distance, scan position), so the
// merge reproduces the single-CTA result exactly).
// ---------------------------------------------------------------------------------
namespace {
constexpr uint32_t SPLIT_BLOCKS = 64;   // 128-entry blocks per part
constexpr uint32_t SPLIT_BLOCKS_OVER = 64;  // ... when only overflowed queries run (smaller parts measured slower)
constexpr int SPLIT_MAX_KEYS = 8192;    // keys merged per query (parts x next_pow2(k))
}

__global__ void split_count_kernel(const uint32_t* __restrict__ probe, int nprobe, int nscan,
                                   const uint64_t* __restrict__ blk_off, long long nq,
                                   const uint32_t* __restrict__ only_over, uint32_t over_cap, uint32_t max_parts,
                                   uint32_t blocks_per_part, uint32_t max_blocks, uint32_t* __restrict__ parts,
                                   uint32_t* __restrict__ nblocks) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        uint32_t nb = 0;
        for (int t = 0; t < nscan; ++t) {
            const uint32_t l = probe[q * nprobe + t];
            nb += (uint32_t)(blk_off[l + 1] - blk_off[l]);
        }
        nb = min(nb, max_blocks);
        const bool run = !only_over || only_over[q] > over_cap;
        const uint32_t p = (nb + blocks_per_part - 1) / blocks_per_part;
        parts[q] = run ? max(1u, min(p, max_parts)) : 0u;
        nblocks[q] = nb;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) parts[nq] = 0;
}

__global__ void split_fill_kernel(const uint32_t* __restrict__ parts, const uint32_t* __restrict__ part_off,
                                  const uint32_t* __restrict__ nblocks, long long nq, uint4* __restrict__ items) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        const uint32_t np = parts[q];
        if (np == 0) continue;
        const uint32_t nb = nblocks[q];
        const uint32_t per = (nb + np - 1) / np;
        for (uint32_t i = 0; i < np; ++i)
            items[part_off[q] + i] = make_uint4((uint32_t)q, i * per, min(nb, (i + 1) * per), 0u);
    }
}

// Per query: the k smallest of its parts' keys, written like the unsplit scan.
__global__ void __launch_bounds__(256) split_merge_kernel(
    const unsigned long long* __restrict__ part_keys, const uint32_t* __restrict__ parts,
    const uint32_t* __restrict__ part_off, const uint32_t* __restrict__ probe, int nprobe, int nscan,
    const uint64_t* __restrict__ offs, const uint64_t* __restrict__ ids, int k, uint64_t* __restrict__ out_ids,
    float* __restrict__ out_d, uint32_t* __restrict__ out_n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);    // [SPLIT_MAX_KEYS]
    uint32_t* eprefix = reinterpret_cast<uint32_t*>(keys + SPLIT_MAX_KEYS);          // [nscan + 1]
    const long long q = blockIdx.x;
    const uint32_t np = parts[q];
    if (np == 0) return;
    const int n = (int)np * k;
    const int p2 = next_pow2(n < 2 ? 2 : n);
    const unsigned long long* src = part_keys + (long long)part_off[q] * k;
    for (int i = threadIdx.x; i < p2; i += 256) keys[i] = i < n ? src[i] : ~0ull;
    if (threadIdx.x < 32) probe_prefixes_warp(probe + q * nprobe, nscan, offs, nullptr, eprefix, nullptr);
    bitonic_sort_u64<256>(keys, p2);
    __shared__ int h_s;
    if (threadIdx.x == 0) {
        int h = 0;
        while (h < k && h < n && keys[h] != ~0ull) ++h;
        h_s = h;
    }
    __syncthreads();
    const int h = h_s;
    for (int i = threadIdx.x; i < k; i += 256) {
        if (i < h) {
            const unsigned long long key = keys[i];
            const uint32_t sq = (uint32_t)(key & 0xffffffffull);
            int lo = 0, hi = nscan;
            while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (eprefix[mid] <= sq) lo = mid; else hi = mid; }
            const uint32_t l = probe[q * nprobe + lo];
            out_ids[q * k + i] = ids[offs[l] + (sq - eprefix[lo])];
            out_d[q * k + i] = key_float((uint32_t)(key >> 32));
        } else {
            out_ids[q * k + i] = 0;
            out_d[q * k + i] = h > 0 ? key_float((uint32_t)(keys[h - 1] >> 32)) : 0.0f;
        }
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)h;
}

void SplitWork::reserve(long long nq) {
    parts.reserve(nq + 1);
    part_off.reserve(nq + 1);
    nblocks.reserve(nq);
    size_t need = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, need, parts.data(), part_off.data(), (int)(nq + 1));
    scan_tmp.reserve(need + 256);
    if (!host_total) check(cudaMallocHost(&host_total, sizeof(uint32_t)), "cudaMallocHost");
}

SplitWork::~SplitWork() {
    if (host_total) cudaFreeHost(host_total);
}

void launch_scan_blocked_split(const float* T, long long nq, const float* pbase, const uint32_t* probe, int nprobe,
                               int nscan, int m, const uint64_t* offs, const uint64_t* blk_off,
                               const uint8_t* bcodes, const float* bvterm, const uint64_t* ids, int k,
                               uint64_t* out_ids, float* out_d, uint32_t* out_n, const uint32_t* only_over,
                               uint32_t over_cap, SplitWork& w, cudaStream_t st, uint32_t max_blocks) {
    if (nq <= 0) return;
    if (k > kMaxK) throw CudaError("scan_blocked_split: k exceeds the supported maximum");
    w.reserve(nq);
    const uint32_t max_parts = (uint32_t)std::max(1, SPLIT_MAX_KEYS / k);
    const int gb = (int)std::min<long long>((nq + 255) / 256, 148LL * 4);
    split_count_kernel<<<gb, 256, 0, st>>>(probe, nprobe, nscan, blk_off, nq, only_over, over_cap, max_parts,
                                           only_over ? SPLIT_BLOCKS_OVER : SPLIT_BLOCKS, max_blocks,
                                           w.parts.data(), w.nblocks.data());
    VGPU_LAUNCH("split_count_kernel");
    size_t tmp = w.scan_tmp.size();
    check(cub::DeviceScan::ExclusiveSum(w.scan_tmp.data(), tmp, w.parts.data(), w.part_off.data(), (int)(nq + 1), st),
          "cub::DeviceScan::ExclusiveSum(split parts)");
    check(cudaMemcpyAsync(w.host_total, w.part_off.data() + nq, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    const uint32_t total = *w.host_total;
    if (total == 0) return;
    w.items.reserve(total);
    w.part_keys.reserve((size_t)total * k);
    split_fill_kernel<<<gb, 256, 0, st>>>(w.parts.data(), w.part_off.data(), w.nblocks.data(), nq, w.items.data());
    VGPU_LAUNCH("split_fill_kernel");
    scan_blocked_impl(T, total, pbase, probe, nprobe, nscan, m, offs, blk_off, bcodes, bvterm, ids, k, nullptr, nullptr,
                      nullptr, nullptr, 0, w.items.data(), w.part_keys.data(), st);
    const size_t smem = (size_t)SPLIT_MAX_KEYS * 8 + (size_t)(nscan + 1) * 4;
    check(cudaFuncSetAttribute(split_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute(split_merge)");
    split_merge_kernel<<<(unsigned)nq, 256, smem, st>>>(w.part_keys.data(), w.parts.data(), w.part_off.data(), probe,
                                                        nprobe, nscan, offs, ids, k, out_ids, out_d, out_n);
    VGPU_LAUNCH("split_merge_kernel");
}

}  // namespace vgpu
