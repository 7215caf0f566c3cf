// Exact flat top-k (find_nearest_centroids_batch_fused,
// include/vesper/kernels/batch_distances.hpp:338-456): for each query the k best base
// vectors under L2 (smallest first) or inner product (largest first), scores in the
// reference's AVX2 lane order (kernels/backends/avx2.hpp:76-154), ties to the smaller
// index (:362-369), k_eff = min(k, N).
//
// Small bases (N <= 65536): one tf32 tensor-core screen of every (query, base) pair and
// the exact band refine of screen_select (the coarse quantizer's path).
// Larger bases, two passes over tensor-core screens:
//   1. the screen + exact refine over a strided sample of the base gives each query the
//      exact k_eff-th best score of the sample, tau -- no worse than the k_eff-th best of
//      the whole base, so every member of the true top-k scores at least as well as tau;
//   2. the screen over the whole base keeps the columns whose proven bound can reach tau
//      (tc_screen_kernel filter modes, column tiles streamed from HBM once), then
//      flat_refine_kernel takes U* = the k_eff-th smallest upper bound among them,
//      re-scores exactly every kept column whose lower bound is <= U*, and selects by
//      (score, index).
// A query whose kept-column list overflows its capacity is redone by the single-pass
// path, which handles any number of columns.
#include <algorithm>
#include <cfloat>
#include <vector>

#include "kernels.cuh"
#include "kernels_tc.cuh"
#include "select.cuh"
#include "tc_screen.cuh"

namespace vgpu {
namespace {
constexpr int FR_NT = 256;
constexpr long long FLAT_SINGLE = 65536;        // bases up to this size take the single-pass path
constexpr size_t SCREEN_BUDGET = size_t(512) << 20;  // bytes of screen values per query chunk
constexpr long long FILTER_ROWS = 16384;        // queries per filter chunk (kept-column lists)
constexpr long long FILTER_COLS = 65535LL * 256;  // columns per filter launch (grid.y limit)

// Ordering key: ascending (score, index) for L2, (-score, index) for inner products
// (zero canonicalised so that -0 and +0 tie).
template <bool IP>
__device__ __forceinline__ unsigned long long order_key(float v, uint32_t idx) {
    const float o = IP ? (v == 0.0f ? 0.0f : -v) : v;
    return ((unsigned long long)float_key(o) << 32) | idx;
}
template <bool IP>
__device__ __forceinline__ float key_score(unsigned long long key) {
    const float o = key_float((uint32_t)(key >> 32));
    return IP ? (o == 0.0f ? 0.0f : -o) : o;
}

template <bool IP>
__device__ __forceinline__ float eps_of(float rn, float cn, float dt, int dim) {
    return IP ? screen_eps_ip(rn, cn, dim) : screen_eps(rn, cn, dt, dim);
}
}  // namespace

// One CTA per query: kept columns -> U* -> exact band -> the k_eff best.  Queries whose
// list overflowed are recorded in `over` (global row ids) and left to the caller.
template <bool IP>
__global__ void __launch_bounds__(FR_NT) flat_refine_kernel(const float* __restrict__ q, const float* __restrict__ base,
                                                            int dim, const float* __restrict__ xn,
                                                            const float* __restrict__ cn, const uint2* __restrict__ cand,
                                                            const uint32_t* __restrict__ cand_cnt, int cap, int k,
                                                            int ke, long long row0, uint32_t* __restrict__ out_idx,
                                                            float* __restrict__ out_score, uint32_t* __restrict__ over,
                                                            uint32_t* __restrict__ n_over) {
    extern __shared__ __align__(16) unsigned long long keys[];  // [next_pow2(cap)]
    uint32_t* band = reinterpret_cast<uint32_t*>(keys + next_pow2(cap));  // [cap]
    __shared__ uint32_t s_band;
    const long long row = blockIdx.x;
    const uint32_t n_all = cand_cnt[row];
    if (n_all > (uint32_t)cap) {
        if (threadIdx.x == 0) over[atomicAdd(n_over, 1u)] = (uint32_t)(row0 + row);
        return;
    }
    const int n = (int)n_all;
    const uint2* cr = cand + row * cap;
    const float* xr = q + row * dim;
    const float rn = xn[row];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // 1) U* = the ke-th smallest upper bound among the kept columns.
    const int p2 = next_pow2(n < 2 ? 2 : n);
    for (int i = threadIdx.x; i < p2; i += FR_NT) {
        unsigned long long key = ~0ull;
        if (i < n) {
            const uint2 e = cr[i];
            const float dt = __uint_as_float(e.y);
            key = ((unsigned long long)float_key(dt + eps_of<IP>(rn, cn[e.x], dt, dim)) << 32) | (uint32_t)i;
        }
        keys[i] = key;
    }
    if (threadIdx.x == 0) s_band = 0;
    bitonic_sort_u64<FR_NT>(keys, p2);
    const bool take_all = n < ke;
    const float ustar = take_all ? FLT_MAX : key_float((uint32_t)(keys[ke - 1] >> 32));

    // 2) The band: every kept column whose lower bound is <= U*.
    for (int i0 = 0; i0 < n; i0 += FR_NT) {
        const int i = i0 + threadIdx.x;
        bool in = false;
        if (i < n) {
            const uint2 e = cr[i];
            const float dt = __uint_as_float(e.y);
            in = take_all || dt - eps_of<IP>(rn, cn[e.x], dt, dim) <= ustar;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, in);
        if (bal) {
            uint32_t b = 0;
            if (lane == 0) b = atomicAdd(&s_band, (uint32_t)__popc(bal));
            b = __shfl_sync(0xffffffffu, b, 0);
            if (in) band[b + __popc(bal & ((1u << lane) - 1u))] = (uint32_t)i;
        }
    }
    __syncthreads();
    const int nb = (int)s_band;

    // 3) Exact scores in the reference's lane order, 4 columns per warp per step.
    for (int b0 = warp * 4; b0 < nb; b0 += (FR_NT / 32) * 4) {
        const int bi = b0 + (lane >> 3);
        const bool act = bi < nb;
        const uint32_t c = act ? cr[band[bi]].x : 0u;
        const float* crow = base + (long long)c * dim;
        const float v = IP ? warp_ip_group(xr, crow, dim, act) : warp_l2_group(xr, crow, dim, act);
        if (act && (lane & 7) == 0) keys[bi] = order_key<IP>(v, c);
    }
    const int p2b = next_pow2(nb < 2 ? 2 : nb);
    __syncthreads();
    for (int i = nb + threadIdx.x; i < p2b; i += FR_NT) keys[i] = ~0ull;
    bitonic_sort_u64<FR_NT>(keys, p2b);
    const int take = nb < ke ? nb : ke;
    for (int i = threadIdx.x; i < k; i += FR_NT) {
        const bool real = i < take;
        out_idx[row * k + i] = real ? (uint32_t)(keys[i] & 0xffffffffull) : 0xffffffffu;
        out_score[row * k + i] = real ? key_score<IP>(keys[i]) : (IP ? -FLT_MAX : FLT_MAX);
    }
}

// dst[i] = src[i * stride] (norms of a strided sample).
__global__ void gather_stride_kernel(const float* __restrict__ src, long long n, long long stride,
                                     float* __restrict__ dst) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[i * stride];
}

// tau[q] = the ke-th best sample score in screen units (L2: distance; IP: -2 * score).
__global__ void flat_tau_kernel(const float* __restrict__ s_val, long long nq, int k, int ke, int ip,
                                float* __restrict__ tau) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nq; i += (long long)gridDim.x * blockDim.x) {
        const float v = s_val[i * k + ke - 1];
        tau[i] = ip ? -2.0f * v : v;
    }
}

// Copies rows[i] of src (n x dim) and its norm into dst row i.
__global__ void gather_rows_kernel(const float* __restrict__ src, const float* __restrict__ src_n,
                                   const uint32_t* __restrict__ rows, int n, int dim, float* __restrict__ dst,
                                   float* __restrict__ dst_n) {
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const long long r = rows[i];
        for (int d = threadIdx.x; d < dim; d += blockDim.x) dst[(long long)i * dim + d] = src[r * dim + d];
        if (threadIdx.x == 0) dst_n[i] = src_n[r];
    }
}

// Writes result row i to row rows[i] of the outputs.
__global__ void scatter_rows_kernel(const uint32_t* __restrict__ idx, const float* __restrict__ val,
                                    const uint32_t* __restrict__ rows, int n, int k, uint32_t* __restrict__ out_idx,
                                    float* __restrict__ out_val) {
    for (int i = blockIdx.x; i < n; i += gridDim.x) {
        const long long r = rows[i];
        for (int j = threadIdx.x; j < k; j += blockDim.x) {
            out_idx[r * k + j] = idx[(long long)i * k + j];
            out_val[r * k + j] = val[(long long)i * k + j];
        }
    }
}

// Columns ke..k-1 of every row (k > N): index 0xffffffff, the worst score.
__global__ void pad_topk_kernel(long long nq, int k, int ke, bool ip, uint32_t* __restrict__ out_idx,
                                float* __restrict__ out_val) {
    const long long total = nq * (k - ke);
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long r = t / (k - ke), j = ke + t % (k - ke);
        out_idx[r * k + j] = 0xffffffffu;
        out_val[r * k + j] = ip ? -FLT_MAX : FLT_MAX;
    }
}

namespace {
int grid_for(long long n, int nt) { return (int)std::max<long long>(1, std::min<long long>((n + nt - 1) / nt, 148LL * 16)); }

// Exact top-k of x rows against nc columns (row j of c at j * c_ld) through a full
// screen + screen_select, in query chunks of SCREEN_BUDGET screen bytes.
void exact_rows(bool ip, const float* x, long long nx, const float* xn, const float* c, long long nc, long long c_ld,
                const float* cn, int dim, int k, uint32_t* out_idx, float* out_val, FlatWork& w, cudaStream_t st) {
    const long long qc = std::max<long long>(1, (long long)(SCREEN_BUDGET / (sizeof(float) * (size_t)nc)));
    w.dt.reserve((size_t)std::min(qc, nx) * nc);
    for (long long q0 = 0; q0 < nx; q0 += qc) {
        const long long n = std::min(qc, nx - q0);
        launch_tc_screen_op(ip, x + q0 * dim, n, c, nc, c_ld, dim, xn + q0, cn, w.dt.data(), nc, w.err.data(), st);
        launch_screen_select_op(ip, w.dt.data(), n, nc, (int)nc, x + q0 * dim, dim, c, c_ld, xn + q0, cn, k,
                                out_idx + q0 * k, out_val + q0 * k, w.err.data(), st);
    }
}

template <bool IP>
void refine_launch(const float* q, const float* base, int dim, const float* xn, const float* cn, const uint2* cand,
                   const uint32_t* cnt, int cap, long long nrows, int k, int ke, long long row0, uint32_t* out_idx,
                   float* out_score, uint32_t* over, uint32_t* n_over, cudaStream_t st) {
    const size_t smem = (size_t)next_pow2(cap) * 8 + (size_t)cap * 4;
    check(cudaFuncSetAttribute(flat_refine_kernel<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute(flat_refine)");
    flat_refine_kernel<IP><<<(unsigned)nrows, FR_NT, smem, st>>>(q, base, dim, xn, cn, cand, cnt, cap, k, ke, row0,
                                                                out_idx, out_score, over, n_over);
    check(cudaGetLastError(), "flat_refine_kernel");
}
}  // namespace

FlatWork::~FlatWork() {
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
}

void launch_flat_topk(bool ip, const float* q, long long nq, const float* base, long long nb, int dim, int k,
                      uint32_t* out_idx, float* out_score, FlatWork& w, cudaStream_t st) {
    w.last = FlatStats{};
    if (nq <= 0 || nb <= 0 || k <= 0) return;
    if (k > kMaxK) throw CudaError("flat_topk: k exceeds the supported maximum (1024)");
    if (!tc_screen_supported(dim)) throw CudaError("flat_topk: dim must be a multiple of 4 and >= 32");
    if (nb > 0x7fffffffLL) throw CudaError("flat_topk: at most 2^31 - 1 base vectors");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(base)) & 15)
        throw CudaError("flat_topk: queries and base must be 16-byte aligned");
    if (!w.ev[0])
        for (auto& e : w.ev) check(cudaEventCreate(&e), "cudaEventCreate");
    const int ke = (int)std::min<long long>(k, nb);
    w.err.reserve(1);
    w.xn.reserve(nq);
    w.cn.reserve(nb);
    check(cudaMemsetAsync(w.err.data(), 0, sizeof(int), st), "memset");
    check(cudaEventRecord(w.ev[0], st), "event");
    launch_row_norms(q, nq, dim, w.xn.data(), st);
    launch_row_norms(base, nb, dim, w.cn.data(), st);
    uint32_t n_over = 0;
    if (nb <= FLAT_SINGLE) {
        check(cudaEventRecord(w.ev[1], st), "event");
        exact_rows(ip, q, nq, w.xn.data(), base, nb, dim, w.cn.data(), dim, k, out_idx, out_score, w, st);
        if (k > ke) {
            pad_topk_kernel<<<grid_for(nq * (k - ke), 256), 256, 0, st>>>(nq, k, ke, ip, out_idx, out_score);
            check(cudaGetLastError(), "pad_topk_kernel");
        }
        check(cudaEventRecord(w.ev[2], st), "event");
        w.last.single_pass = 1;
    } else {
        // Capacity of the kept-column lists and sample stride: the sample's k-th best is
        // about the (k * stride)-th best of the base, so about k * stride columns survive.
        const int cap = k <= 256 ? 4096 : 16384;
        long long stride = 16;
        while (stride > 1 && (long long)k * stride * 4 > cap) stride >>= 1;
        while (stride > 1 && (nb + stride - 1) / stride < ke) stride >>= 1;
        const long long ns = (nb + stride - 1) / stride;
        w.cs.reserve(ns);
        w.s_idx.reserve((size_t)nq * k);
        w.s_val.reserve((size_t)nq * k);
        w.tau.reserve(nq);
        gather_stride_kernel<<<grid_for(ns, 256), 256, 0, st>>>(w.cn.data(), ns, stride, w.cs.data());
        check(cudaGetLastError(), "gather_stride_kernel");
        check(cudaEventRecord(w.ev[1], st), "event");
        // pass 1: exact top-ke of the sample
        exact_rows(ip, q, nq, w.xn.data(), base, ns, stride * dim, w.cs.data(), dim, k, w.s_idx.data(),
                   w.s_val.data(), w, st);
        flat_tau_kernel<<<grid_for(nq, 256), 256, 0, st>>>(w.s_val.data(), nq, k, ke, ip ? 1 : 0, w.tau.data());
        check(cudaGetLastError(), "flat_tau_kernel");
        check(cudaEventRecord(w.ev[2], st), "event");
        // pass 2: filter the whole base, refine the kept columns
        const long long qc = std::min(nq, FILTER_ROWS);
        w.cand.reserve((size_t)qc * cap);
        w.cand_cnt.reserve(nq);
        w.over.reserve(nq + 1);
        check(cudaMemsetAsync(w.cand_cnt.data(), 0, (size_t)nq * sizeof(uint32_t), st), "memset");
        check(cudaMemsetAsync(w.over.data() + nq, 0, sizeof(uint32_t), st), "memset");
        float filter_ms = 0.0f, refine_ms = 0.0f;
        for (long long q0 = 0; q0 < nq; q0 += qc) {
            const long long n = std::min(qc, nq - q0);
            check(cudaEventRecord(w.ev[3], st), "event");
            for (long long c0 = 0; c0 < nb; c0 += FILTER_COLS)
                launch_tc_filter(ip, q + q0 * dim, n, base + c0 * dim, std::min(FILTER_COLS, nb - c0), dim,
                                 w.xn.data() + q0, w.cn.data() + c0, w.tau.data() + q0, (uint32_t)c0, w.cand.data(),
                                 w.cand_cnt.data() + q0, cap, w.err.data(), st);
            check(cudaEventRecord(w.ev[4], st), "event");
            if (ip)
                refine_launch<true>(q + q0 * dim, base, dim, w.xn.data() + q0, w.cn.data(), w.cand.data(),
                                    w.cand_cnt.data() + q0, cap, n, k, ke, q0, out_idx + q0 * k, out_score + q0 * k,
                                    w.over.data(), w.over.data() + nq, st);
            else
                refine_launch<false>(q + q0 * dim, base, dim, w.xn.data() + q0, w.cn.data(), w.cand.data(),
                                     w.cand_cnt.data() + q0, cap, n, k, ke, q0, out_idx + q0 * k, out_score + q0 * k,
                                     w.over.data(), w.over.data() + nq, st);
            check(cudaEventRecord(w.ev[5], st), "event");
            check(cudaEventSynchronize(w.ev[5]), "cudaEventSynchronize");
            float a = 0.0f, b = 0.0f;
            check(cudaEventElapsedTime(&a, w.ev[3], w.ev[4]), "elapsed");
            check(cudaEventElapsedTime(&b, w.ev[4], w.ev[5]), "elapsed");
            filter_ms += a;
            refine_ms += b;
        }
        check(cudaMemcpyAsync(&n_over, w.over.data() + nq, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
        std::vector<uint32_t> cnt((size_t)nq);
        check(cudaMemcpyAsync(cnt.data(), w.cand_cnt.data(), (size_t)nq * sizeof(uint32_t), cudaMemcpyDeviceToHost, st),
              "d2h");
        check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        for (uint32_t c : cnt) w.last.candidates += std::min<uint32_t>(c, (uint32_t)cap);
        w.last.filter_ms = filter_ms;
        w.last.refine_ms = refine_ms;
        w.last.sample_stride = (int)stride;
        w.last.cap = cap;
        if (n_over) {
            // the single-pass path for the queries whose lists overflowed
            w.oq.reserve((size_t)n_over * dim);
            w.oxn.reserve(n_over);
            w.o_idx.reserve((size_t)n_over * k);
            w.o_val.reserve((size_t)n_over * k);
            gather_rows_kernel<<<std::min<uint32_t>(n_over, 4096), 256, 0, st>>>(q, w.xn.data(), w.over.data(),
                                                                                 (int)n_over, dim, w.oq.data(),
                                                                                 w.oxn.data());
            check(cudaGetLastError(), "gather_rows_kernel");
            exact_rows(ip, w.oq.data(), n_over, w.oxn.data(), base, nb, dim, w.cn.data(), dim, k, w.o_idx.data(),
                       w.o_val.data(), w, st);
            scatter_rows_kernel<<<std::min<uint32_t>(n_over, 4096), 128, 0, st>>>(
                w.o_idx.data(), w.o_val.data(), w.over.data(), (int)n_over, k, out_idx, out_score);
            check(cudaGetLastError(), "scatter_rows_kernel");
        }
    }
    check(cudaEventRecord(w.ev[6], st), "event");
    int e = 0;
    check(cudaMemcpyAsync(&e, w.err.data(), sizeof(int), cudaMemcpyDeviceToHost, st), "d2h");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (e) throw CudaError("flat_topk: tensor-core screen wait expired (code " + std::to_string(e) + ")");
    w.last.overflow_queries = n_over;
    float t = 0.0f;
    check(cudaEventElapsedTime(&t, w.ev[0], w.ev[6]), "elapsed");
    w.last.total_ms = t;
    check(cudaEventElapsedTime(&t, w.ev[0], w.ev[1]), "elapsed");
    w.last.norms_ms = t;
    check(cudaEventElapsedTime(&t, w.ev[1], w.ev[2]), "elapsed");
    w.last.sample_ms = t;  // single pass: the whole screen + select
    w.last.fallback_ms =
        std::max(0.0f, w.last.total_ms - w.last.norms_ms - w.last.sample_ms - w.last.filter_ms - w.last.refine_ms);
}

}  // namespace vgpu
