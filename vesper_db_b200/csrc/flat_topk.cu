// Exact flat top-k (find_nearest_centroids_batch_fused,
// include/vesper/kernels/batch_distances.hpp:338-456): for each query the k best base
// vectors under L2 (smallest first) or inner product (largest first), scores in the
// reference's AVX2 lane order (kernels/backends/avx2.hpp:76-154), ties to the smaller
// index (:362-369), k_eff = min(k, N).
//
// Small bases (N <= 16384): one tf32 tensor-core screen of every (query, base) pair and
// the exact band refine of screen_select (the coarse quantizer's path).
// Larger bases, two passes over tensor-core screens:
//   1. the exact top-k of a strided sample of the base (every 16th row, computed the
//      same way, recursively) gives each query the exact k_eff-th best score of the
//      sample, tau -- no worse than the k_eff-th best of the whole base, so every member
//      of the true top-k scores at least as well as tau;
//   2. the screen over the whole base keeps the columns whose proven bound can reach tau
//      (tc_screen_kernel filter modes, column tiles streamed from HBM once), then
//      flat_refine_kernel takes U* = the k_eff-th smallest upper bound among them,
//      re-scores exactly every kept column whose lower bound is <= U*, and selects by
//      (score, index).
// A query whose kept-column list overflows its capacity is redone by one full screen,
// which handles any number of columns.
#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "kernels_tc.cuh"
#include "select.cuh"
#include "tc_screen.cuh"

namespace vgpu {
namespace {
constexpr int FR_NT = 256;
constexpr long long FLAT_SINGLE = 16384;        // views up to this size take one screen (shared-memory select)
constexpr long long FLAT_STRIDE = 16;           // sample stride of the threshold pass
constexpr size_t SCREEN_BUDGET = size_t(512) << 20;  // bytes of screen values per query chunk
constexpr size_t CAND_BUDGET = size_t(1) << 30;  // bytes of kept-column lists per filter chunk
constexpr long long FILTER_COLS = 65535LL * 256;  // columns per filter launch (grid.y limit)
constexpr size_t AUG_BUDGET = size_t(1) << 30;     // bytes of an augmented L2 view (launch_aug_cols)

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
// Shared memory: u64[cap] (the upper-bound keys as u32 first, later the exact keys)
// and u32[cap] (the band's positions).
template <bool IP>
__global__ void __launch_bounds__(FR_NT) flat_refine_kernel(const float* __restrict__ q, const float* __restrict__ base,
                                                            long long ld, int dim, const float* __restrict__ xn,
                                                            const float* __restrict__ cn, const uint2* __restrict__ cand,
                                                            const uint32_t* __restrict__ cand_cnt, int cap, int k,
                                                            int ke, long long row0, uint32_t* __restrict__ out_idx,
                                                            float* __restrict__ out_score, uint32_t* __restrict__ over,
                                                            uint32_t* __restrict__ n_over) {
    extern __shared__ __align__(16) unsigned long long keys[];         // [cap]
    uint32_t* ukey = reinterpret_cast<uint32_t*>(keys);               // [cap], aliases keys
    uint32_t* band = reinterpret_cast<uint32_t*>(keys + cap);         // [cap]
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_band, s_rem, s_bin;
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

    // 1) U* = the ke-th smallest upper bound among the kept columns (4-pass radix
    //    select on order-preserving keys; histogram updates aggregated per warp).
    for (int i = threadIdx.x; i < n; i += FR_NT) {
        const uint2 e = cr[i];
        const float dt = __uint_as_float(e.y);
        ukey[i] = float_key(dt + eps_of<IP>(rn, cn[e.x], dt, dim));
    }
    const bool take_all = n < ke;
    uint32_t prefix = 0, mask = 0;
    if (threadIdx.x == 0) { s_rem = (uint32_t)ke; s_band = 0; }
    if (!take_all) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = threadIdx.x; i < 256; i += FR_NT) hist[i] = 0;
            __syncthreads();
            for (int i0 = 0; i0 < n; i0 += FR_NT) {
                const int i = i0 + threadIdx.x;
                const uint32_t key = i < n ? ukey[i] : 0u;
                const bool part = i < n && (key & mask) == prefix;
                const unsigned act = __ballot_sync(0xffffffffu, part);
                if (act) {
                    const int lead = __ffs(act) - 1;
                    const uint32_t bin = (key >> shift) & 255u;
                    const uint32_t bin0 = __shfl_sync(0xffffffffu, bin, lead);
                    const unsigned same = __ballot_sync(0xffffffffu, part && bin == bin0);
                    if (lane == lead) atomicAdd(&hist[bin0], (uint32_t)__popc(same));
                    if (part && bin != bin0) atomicAdd(&hist[bin], 1u);
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                uint32_t rem = s_rem, acc = 0, b = 0;
                for (; b < 256; ++b) { const uint32_t h = hist[b]; if (acc + h >= rem) break; acc += h; }
                s_rem = rem - acc;
                s_bin = b;
            }
            __syncthreads();
            prefix |= s_bin << shift;
            mask |= 255u << shift;
        }
    } else {
        __syncthreads();
    }
    const float ustar = take_all ? FLT_MAX : key_float(prefix);

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
        const float* crow = base + (long long)c * ld;
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
// The filter screen on the persistent pipeline (tc_filter_kernel) unless
// VGPU_FILTER=tile asks for one CTA per 128 x 256 tile (tc_screen_kernel's filter modes).
bool persistent_filter() {
    static const bool on = [] {
        const char* v = std::getenv("VGPU_FILTER");
        return !(v && std::string(v) == "tile");
    }();
    return on;
}

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
        w.launches += 2;
    }
}

template <bool IP>
void refine_launch(const float* q, const float* base, long long ld, int dim, const float* xn, const float* cn,
                   const uint2* cand, const uint32_t* cnt, int cap, long long nrows, int k, int ke, long long row0,
                   uint32_t* out_idx, float* out_score, uint32_t* over, uint32_t* n_over, cudaStream_t st) {
    const size_t smem = (size_t)cap * 12;  // cap is a power of two
    check(cudaFuncSetAttribute(flat_refine_kernel<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute(flat_refine)");
    flat_refine_kernel<IP><<<(unsigned)nrows, FR_NT, smem, st>>>(q, base, ld, dim, xn, cn, cand, cnt, cap, k, ke,
                                                                row0, out_idx, out_score, over, n_over);
    VGPU_LAUNCH("flat_refine_kernel");
}


// Sample stride of a view of n rows at top-k k: the sample's k-th best is about the
// (k * stride)-th best of the view, so about k * stride columns survive the filter:
// stride <= cap / (2k).  Below 2 the view is screened in one pass.
long long flat_sample_stride(long long n, int k, long long max_stride = FLAT_STRIDE) {
    const int cap = k <= 128 ? 4096 : 16384;
    const long long ke = std::min<long long>(k, n);
    long long stride = std::min<long long>(max_stride, std::max(1, cap / (2 * k)));
    while (stride > 1 && (n + stride - 1) / stride < ke) stride >>= 1;
    return stride;
}

// A base arriving from host memory in chunks (launch_flat_topk_host): rows [0, normed)
// have landed as far as the compute stream knows and have their norms.
struct Feed {
    const float* base;
    long long nb, chunk;
    int dim;
    float* cn;
    float* cs;
    const float* sample_rows;   // every stride-th base row, contiguous, copied first
    cudaEvent_t sample;
    const std::vector<cudaEvent_t>* ev;
    long long normed = 0;
    void ready(long long upto, cudaStream_t st, int& launches) {
        while (normed < upto) {
            const long long i = normed / chunk, r1 = std::min(nb, (i + 1) * chunk);
            check(cudaStreamWaitEvent(st, (*ev)[(size_t)i], 0), "cudaStreamWaitEvent");
            launch_row_norms(base + normed * dim, r1 - normed, dim, cn + normed, st);
            launch_sqrt(cn + normed, r1 - normed, cs + normed, st);
            launches += 2;
            normed = r1;
        }
    }
};

// A view of the base: row j at base + j * ld, with its squared norms and their roots.
struct View {
    const float* base;
    long long n, ld;
    const float* cn;
    const float* cs;
};

// Exact top-k of every query against the view (indices local to the view).  Views
// that fit screen_select's shared-memory path take one screen; larger ones get their
// threshold from the exact top-k of a strided sample of themselves (recursively), then
// one filtering screen and the refine.  `stats` (top level only) receives stage times.
void view_topk(bool ip, const float* q, long long nq, const float* xn, int dim, const View& v, int k,
               uint32_t* out_idx, float* out_val, FlatWork& w, int depth, FlatStats* stats, cudaStream_t st,
               Feed* feed = nullptr, long long single_max = FLAT_SINGLE, long long max_stride = FLAT_STRIDE) {
    const int ke = (int)std::min<long long>(k, v.n);
    const int cap = k <= 128 ? 4096 : 16384;
    const long long stride = flat_sample_stride(v.n, k, max_stride);
    if (v.n <= single_max || depth + 1 >= FlatWork::kLevels || stride < 2) {
        if (feed) feed->ready(v.n, st, w.launches);
        exact_rows(ip, q, nq, xn, v.base, v.n, v.ld, v.cn, dim, k, out_idx, out_val, w, st);
        if (stats) stats->single_pass = 1;
        return;
    }
    FlatWork::Level& L = w.level[depth];
    const long long ns = (v.n + stride - 1) / stride;
    L.cn.reserve(ns);
    L.cs.reserve(ns);
    L.s_idx.reserve((size_t)nq * k);
    L.s_val.reserve((size_t)nq * k);
    if (feed) {
        // the sample rows were copied first, into their own buffer (so the chunk copies
        // never write rows the sample pass reads); their norms come straight from them
        // (the same arithmetic as the full-base norms they would be gathered from)
        check(cudaStreamWaitEvent(st, feed->sample, 0), "cudaStreamWaitEvent");
        launch_row_norms(feed->sample_rows, ns, dim, L.cn.data(), st);
        launch_sqrt(L.cn.data(), ns, L.cs.data(), st);
    } else {
        gather_stride_kernel<<<grid_for(ns, 256), 256, 0, st>>>(v.cn, ns, stride, L.cn.data());
        VGPU_LAUNCH("gather_stride_kernel");
        gather_stride_kernel<<<grid_for(ns, 256), 256, 0, st>>>(v.cs, ns, stride, L.cs.data());
        VGPU_LAUNCH("gather_stride_kernel");
    }
    w.launches += 2;
    if (stats) check(cudaEventRecord(w.ev[1], st), "event");
    const View sample = feed ? View{feed->sample_rows, ns, (long long)dim, L.cn.data(), L.cs.data()}
                             : View{v.base, ns, v.ld * stride, L.cn.data(), L.cs.data()};
    view_topk(ip, q, nq, xn, dim, sample, k, L.s_idx.data(), L.s_val.data(), w, depth + 1, nullptr, st, nullptr,
              single_max, max_stride);
    w.tau.reserve(nq);
    flat_tau_kernel<<<grid_for(nq, 256), 256, 0, st>>>(L.s_val.data(), nq, k, ke, ip ? 1 : 0, w.tau.data());
    VGPU_LAUNCH("flat_tau_kernel");
    ++w.launches;
    if (stats) check(cudaEventRecord(w.ev[2], st), "event");

    // filter the whole view, refine the kept columns
    const long long qc = std::min<long long>(nq, (long long)(CAND_BUDGET / ((size_t)cap * sizeof(uint2))));
    w.cand.reserve((size_t)qc * cap);
    w.cand_cnt.reserve(nq);
    w.over.reserve(nq + 1);
    check(cudaMemsetAsync(w.cand_cnt.data(), 0, (size_t)nq * sizeof(uint32_t), st), "memset");
    check(cudaMemsetAsync(w.over.data() + nq, 0, sizeof(uint32_t), st), "memset");
    // L2 on a resident view of bounded size (coarse centroids, k-means centres): the
    // augmented operand moves ||c||^2 into the tensor-core product (launch_aug_cols).
    const long long ldo = aug_ld(dim);
    const float* caug = nullptr;
    if (!ip && !feed && persistent_filter() && (size_t)v.n * (size_t)ldo * sizeof(float) <= AUG_BUDGET) {
        w.caug.reserve((size_t)v.n * (size_t)ldo);
        launch_aug_cols(v.base, v.n, dim, v.ld, v.cn, w.caug.data(), st);
        ++w.launches;
        caug = w.caug.data();
    }
    float filter_ms = 0.0f, refine_ms = 0.0f;
    for (long long q0 = 0; q0 < nq; q0 += qc) {
        const long long n = std::min(qc, nq - q0);
        if (stats) check(cudaEventRecord(w.ev[3], st), "event");
        // with a feed, one launch per copied chunk, each after its chunk lands
        const long long step = feed ? std::min(FILTER_COLS, feed->chunk) : FILTER_COLS;
        for (long long c0 = 0; c0 < v.n; c0 += step, ++w.launches) {
            if (feed) feed->ready(std::min(v.n, c0 + step), st, w.launches);
            const long long nc = std::min(step, v.n - c0);
            if (persistent_filter()) {
                w.cmax.reserve(2);
                launch_col_max(v.cn + c0, v.cs + c0, (int)nc, w.cmax.data(), st);
                ++w.launches;
                launch_tc_filter_persistent(ip, q + q0 * dim, n, v.base + c0 * v.ld, nc, v.ld, dim, xn + q0,
                                            v.cn + c0, v.cs + c0, w.cmax.data(), w.tau.data() + q0, (uint32_t)c0,
                                            w.cand.data(), w.cand_cnt.data() + q0, cap, w.err.data(), st,
                                            caug ? caug + c0 * ldo : nullptr);
            } else {
                launch_tc_filter(ip, q + q0 * dim, n, v.base + c0 * v.ld, nc, v.ld, dim, xn + q0, v.cn + c0,
                                 v.cs + c0, w.tau.data() + q0, (uint32_t)c0, w.cand.data(), w.cand_cnt.data() + q0,
                                 cap, w.err.data(), st);
            }
        }
        if (stats) check(cudaEventRecord(w.ev[4], st), "event");
        ++w.launches;
        if (ip)
            refine_launch<true>(q + q0 * dim, v.base, v.ld, dim, xn + q0, v.cn, w.cand.data(), w.cand_cnt.data() + q0,
                                cap, n, k, ke, q0, out_idx + q0 * k, out_val + q0 * k, w.over.data(),
                                w.over.data() + nq, st);
        else
            refine_launch<false>(q + q0 * dim, v.base, v.ld, dim, xn + q0, v.cn, w.cand.data(),
                                 w.cand_cnt.data() + q0, cap, n, k, ke, q0, out_idx + q0 * k, out_val + q0 * k,
                                 w.over.data(), w.over.data() + nq, st);
        if (stats) {
            check(cudaEventRecord(w.ev[5], st), "event");
            check(cudaEventSynchronize(w.ev[5]), "cudaEventSynchronize");
            float a = 0.0f, b = 0.0f;
            check(cudaEventElapsedTime(&a, w.ev[3], w.ev[4]), "elapsed");
            check(cudaEventElapsedTime(&b, w.ev[4], w.ev[5]), "elapsed");
            filter_ms += a;
            refine_ms += b;
        }
    }
    uint32_t n_over = 0;
    check(cudaMemcpyAsync(&n_over, w.over.data() + nq, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
    std::vector<uint32_t> cnt;
    if (stats) {
        cnt.resize((size_t)nq);
        check(cudaMemcpyAsync(cnt.data(), w.cand_cnt.data(), (size_t)nq * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                              st),
              "d2h");
    }
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (stats) {
        for (uint32_t c : cnt) stats->candidates += std::min<uint32_t>(c, (uint32_t)cap);
        stats->filter_ms = filter_ms;
        stats->refine_ms = refine_ms;
        stats->sample_stride = (int)stride;
        stats->cap = cap;
        stats->overflow_queries = n_over;
    }
    if (n_over) {
        // one screen over the view for the queries whose lists overflowed
        w.oq.reserve((size_t)n_over * dim);
        w.oxn.reserve(n_over);
        w.o_idx.reserve((size_t)n_over * k);
        w.o_val.reserve((size_t)n_over * k);
        w.o_rows.reserve(n_over);
        check(cudaMemcpyAsync(w.o_rows.data(), w.over.data(), n_over * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st),
              "d2d");
        gather_rows_kernel<<<std::min<uint32_t>(n_over, 4096), 256, 0, st>>>(q, xn, w.o_rows.data(), (int)n_over, dim,
                                                                             w.oq.data(), w.oxn.data());
        VGPU_LAUNCH("gather_rows_kernel");
        exact_rows(ip, w.oq.data(), n_over, w.oxn.data(), v.base, v.n, v.ld, v.cn, dim, k, w.o_idx.data(),
                   w.o_val.data(), w, st);
        scatter_rows_kernel<<<std::min<uint32_t>(n_over, 4096), 128, 0, st>>>(w.o_idx.data(), w.o_val.data(),
                                                                              w.o_rows.data(), (int)n_over, k, out_idx,
                                                                              out_val);
        VGPU_LAUNCH("scatter_rows_kernel");
        w.launches += 2;
    }
}
}  // namespace

FlatWork::~FlatWork() {
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    for (auto& e : chunk_ev) cudaEventDestroy(e);
    if (sample_ev) cudaEventDestroy(sample_ev);
    if (copy_st) {
        cudaStreamSynchronize(copy_st);
        cudaStreamDestroy(copy_st);
    }
}

namespace {
void flat_topk_body(bool ip, const float* q, long long nq, const float* base, long long nb, int dim, int k,
                    uint32_t* out_idx, float* out_score, FlatWork& w, cudaStream_t st, Feed* feed,
                    long long single_max = FLAT_SINGLE, long long max_stride = FLAT_STRIDE) {
    if (!w.ev[0])
        for (auto& e : w.ev) check(cudaEventCreate(&e), "cudaEventCreate");
    const int ke = (int)std::min<long long>(k, nb);
    w.err.reserve(1);
    w.xn.reserve(nq);
    w.cn.reserve(nb);
    w.csq.reserve(nb);
    check(cudaMemsetAsync(w.err.data(), 0, sizeof(int), st), "memset");
    check(cudaEventRecord(w.ev[0], st), "event");
    launch_row_norms(q, nq, dim, w.xn.data(), st);
    w.launches = 1;
    if (feed) {
        feed->cn = w.cn.data();
        feed->cs = w.csq.data();
    } else {
        launch_row_norms(base, nb, dim, w.cn.data(), st);
        launch_sqrt(w.cn.data(), nb, w.csq.data(), st);
        w.launches += 2;
    }
    check(cudaEventRecord(w.ev[1], st), "event");
    check(cudaEventRecord(w.ev[2], st), "event");
    FlatStats stats;
    const View v{base, nb, dim, w.cn.data(), w.csq.data()};
    view_topk(ip, q, nq, w.xn.data(), dim, v, k, out_idx, out_score, w, 0, &stats, st, feed, single_max, max_stride);
    if (k > ke) {
        pad_topk_kernel<<<grid_for(nq * (k - ke), 256), 256, 0, st>>>(nq, k, ke, ip, out_idx, out_score);
        VGPU_LAUNCH("pad_topk_kernel");
        ++w.launches;
    }
    check(cudaEventRecord(w.ev[6], st), "event");
    int e = 0;
    check(cudaMemcpyAsync(&e, w.err.data(), sizeof(int), cudaMemcpyDeviceToHost, st), "d2h");
    check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (e) throw CudaError("flat_topk: tensor-core screen wait expired (code " + std::to_string(e) + ")");
    float t = 0.0f;
    check(cudaEventElapsedTime(&t, w.ev[0], w.ev[6]), "elapsed");
    stats.total_ms = t;
    check(cudaEventElapsedTime(&t, w.ev[0], w.ev[1]), "elapsed");
    stats.norms_ms = t;
    if (stats.single_pass) {
        stats.sample_ms = stats.total_ms - stats.norms_ms;  // the whole screen + select
    } else {
        check(cudaEventElapsedTime(&t, w.ev[1], w.ev[2]), "elapsed");
        stats.sample_ms = t;
        stats.fallback_ms = std::max(0.0f, stats.total_ms - stats.norms_ms - stats.sample_ms - stats.filter_ms -
                                               stats.refine_ms);
    }
    stats.launches = (uint32_t)w.launches;
    w.last = stats;
}

void check_flat_args(const float* q, const float* base, long long nb, int dim, int k) {
    if (k > kMaxK) throw CudaError("flat_topk: k exceeds the supported maximum (1024)");
    if (!tc_screen_supported(dim)) throw CudaError("flat_topk: dim must be a multiple of 4 and >= 32");
    if (nb > 0x7fffffffLL) throw CudaError("flat_topk: at most 2^31 - 1 base vectors");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(base)) & 15)
        throw CudaError("flat_topk: queries and base must be 16-byte aligned");
}
}  // namespace

namespace {
// Elkan's keep-on-tie rule on a top-1: where the current assignment's exact distance
// (reference lane order) equals the nearest one, the current assignment stays.
// Four rows per warp, eight lanes per row.
__global__ void keep_on_tie_kernel(const float* __restrict__ x, long long n, int dim, const float* __restrict__ c,
                                   const uint32_t* __restrict__ keep, uint32_t* __restrict__ idx,
                                   const float* __restrict__ val) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp * 4; b < n; b += nw * 4) {   // warp-uniform trip count
        const long long i = b + (lane >> 3);
        const bool act = i < n;
        const uint32_t kc = act ? keep[i] : 0u;
        const float v = warp_l2_group(x + (act ? i : 0) * dim, c + (long long)kc * dim, dim, act);
        if (act && (lane & 7) == 0 && kc != idx[i] && v == val[i]) idx[i] = kc;
    }
}
}  // namespace

// Views above this many columns take the sampled threshold and the filtering screen in
// launch_exact_nearest (a one-pass screen writes and re-reads nx * nc screen values).
constexpr long long kNearestSingle = 1024;

// Sample stride cap of launch_exact_nearest's threshold recursion.  Each level's filter
// keeps about k x stride columns per row, all of which the refine re-scores; a smaller
// stride adds sample levels.  Measured on the coarse probes (65,536 x 128 centroids,
// 100k rows, k = 64: 32.1 / 28.7 / 32.3 ms at stride 16 / 8 / 4; 16,384 x 768, 10k
// rows, k = 32: 2.34 / 2.95 ms at 16 / 8) the best keeps about 512 columns per row.
// VGPU_NEAREST_STRIDE overrides it.
long long nearest_stride(int k) {
    if (const char* v = std::getenv("VGPU_NEAREST_STRIDE")) return std::max(2L, std::strtol(v, nullptr, 10));
    return std::max<long long>(2, std::min<long long>(FLAT_STRIDE, 512 / std::max(1, k)));
}

void launch_exact_nearest(const float* x, long long nx, const float* c, long long nc, int dim, int k,
                          const uint32_t* keep, uint32_t* out_idx, float* out_val, FlatWork& w, cudaStream_t st) {
    w.last = FlatStats{};
    if (nx <= 0 || nc <= 0 || k <= 0) return;
    check_flat_args(x, c, nc, dim, k);
    if (keep && k != 1) throw CudaError("exact_nearest: the keep-on-tie rule applies to k = 1");
    flat_topk_body(false, x, nx, c, nc, dim, k, out_idx, out_val, w, st, nullptr, kNearestSingle, nearest_stride(k));
    if (keep) {
        keep_on_tie_kernel<<<grid_for(nx * 8, 256), 256, 0, st>>>(x, nx, dim, c, keep, out_idx, out_val);
        VGPU_LAUNCH("keep_on_tie_kernel");
        ++w.launches;
    }
}

void launch_flat_topk(bool ip, const float* q, long long nq, const float* base, long long nb, int dim, int k,
                      uint32_t* out_idx, float* out_score, FlatWork& w, cudaStream_t st) {
    w.last = FlatStats{};
    if (nq <= 0 || nb <= 0 || k <= 0) return;
    check_flat_args(q, base, nb, dim, k);
    flat_topk_body(ip, q, nq, base, nb, dim, k, out_idx, out_score, w, st, nullptr);
}

void launch_flat_topk_host(bool ip, const float* q, long long nq, const float* host_base, float* dev_base,
                           long long nb, int dim, int k, uint32_t* out_idx, float* out_score, FlatWork& w,
                           cudaStream_t st) {
    w.last = FlatStats{};
    if (nq <= 0 || nb <= 0 || k <= 0) return;
    check_flat_args(q, dev_base, nb, dim, k);
    const size_t row = (size_t)dim * sizeof(float);
    const long long stride = flat_sample_stride(nb, k);
    if (nb <= FLAT_SINGLE || stride < 2) {
        // one screen over the whole base: nothing to overlap
        check(cudaMemcpyAsync(dev_base, host_base, (size_t)nb * row, cudaMemcpyHostToDevice, st), "h2d");
        flat_topk_body(ip, q, nq, dev_base, nb, dim, k, out_idx, out_score, w, st, nullptr);
        return;
    }
    constexpr int kChunks = 8;
    const long long chunk = ((nb + kChunks - 1) / kChunks + 255) / 256 * 256;
    const long long n_chunks = (nb + chunk - 1) / chunk;
    if (!w.copy_st) {
        check(cudaStreamCreateWithFlags(&w.copy_st, cudaStreamNonBlocking), "cudaStreamCreate");
        check(cudaEventCreateWithFlags(&w.sample_ev, cudaEventDisableTiming), "cudaEventCreate");
    }
    while ((long long)w.chunk_ev.size() < n_chunks) {
        cudaEvent_t e = nullptr;
        check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        w.chunk_ev.push_back(e);
    }
    // The copies must not outlive this call's use of dev_base, whatever happens.
    struct CopyDone {
        cudaStream_t s;
        ~CopyDone() { cudaStreamSynchronize(s); }
    } done{w.copy_st};
    // order the copies after the caller's earlier work on st
    check(cudaEventRecord(w.sample_ev, st), "cudaEventRecord");
    check(cudaStreamWaitEvent(w.copy_st, w.sample_ev, 0), "cudaStreamWaitEvent");
    const long long ns = (nb + stride - 1) / stride;
    w.sample_rows.reserve((size_t)ns * dim);
    check(cudaMemcpy2DAsync(w.sample_rows.data(), row, host_base, (size_t)stride * row, row, (size_t)ns,
                            cudaMemcpyHostToDevice, w.copy_st),
          "h2d (sample rows)");
    check(cudaEventRecord(w.sample_ev, w.copy_st), "cudaEventRecord");
    for (long long i = 0; i < n_chunks; ++i) {
        const long long r0 = i * chunk, r1 = std::min(nb, r0 + chunk);
        check(cudaMemcpyAsync(dev_base + r0 * dim, host_base + r0 * dim, (size_t)(r1 - r0) * row,
                              cudaMemcpyHostToDevice, w.copy_st),
              "h2d (chunk)");
        check(cudaEventRecord(w.chunk_ev[(size_t)i], w.copy_st), "cudaEventRecord");
    }
    Feed feed{dev_base, nb, chunk, dim, nullptr, nullptr, w.sample_rows.data(), w.sample_ev, &w.chunk_ev};
    flat_topk_body(ip, q, nq, dev_base, nb, dim, k, out_idx, out_score, w, st, &feed);
}

}  // namespace vgpu
