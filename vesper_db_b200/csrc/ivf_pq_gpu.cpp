// Host orchestration of the B200 IVF-PQ index (mirror of the reference's
// IvfPqIndex::Impl, src/index/ivf_pq.cpp).  All arithmetic on vectors runs in the
// CUDA kernels declared in kernels*.cuh; this file owns state, chunking, the
// k-means++ random stream and the file format.
#include "ivf_pq_gpu.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <chrono>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <mutex>
#include <random>
#include <thread>

#include "kernels.cuh"
#include "kernels_opq.cuh"
#include "kernels_tc.cuh"
#include "kernels_train.cuh"
#include "kmeans_gpu.hpp"
#include "noalloc_search.hpp"

namespace vesper::index {

using core::error;
using core::error_code;
using vgpu::DeviceBuffer;

namespace {

constexpr size_t kDistBudget = size_t(512) << 20;  // bytes per distance-matrix chunk
// Search batches are chunked by their coarse distance matrix; one chunk per batch keeps
// every probed list's codes streamed once and its queries in full tiles (a 10k-query
// batch at nlist 16384 is 655 MB).
constexpr size_t kSearchDistBudget = size_t(1) << 30;
// With the filtering probe (no distance matrix) a chunk is bounded by its per-query
// tables instead: m * 2^nbits floats per query.
constexpr size_t kSearchTableBudget = size_t(4) << 30;
constexpr size_t kJacobiMaxDim = 256;               // OPQ Procrustes: the reference's Jacobi sweeps up to this dim
constexpr int kListScanCap = 4096;                   // screened candidates kept per query (2048: more overflow fallbacks, 8192: no faster)

auto fail(error_code c, std::string msg, std::string comp = "ivf_pq") {
    return std::unexpected(error{c, std::move(msg), std::move(comp)});
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) vgpu::check(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Pinned host staging buffer (grow-only).
struct Pinned {
    void* p = nullptr;
    size_t bytes = 0;
    ~Pinned() { if (p) cudaFreeHost(p); }
    template <class T>
    T* get(size_t n) {
        const size_t need = n * sizeof(T);
        if (need > bytes) {
            if (p) cudaFreeHost(p);
            vgpu::check(cudaMallocHost(&p, need), "cudaMallocHost");
            bytes = need;
        }
        return static_cast<T*>(p);
    }
};

template <class T>
void h2d(T* d, const T* h, size_t n, cudaStream_t st) {
    if (n) vgpu::check(cudaMemcpyAsync(d, h, n * sizeof(T), cudaMemcpyHostToDevice, st), "h2d");
}
template <class T>
void d2h(T* h, const T* d, size_t n, cudaStream_t st) {
    if (n) vgpu::check(cudaMemcpyAsync(h, d, n * sizeof(T), cudaMemcpyDeviceToHost, st), "d2h");
}
template <class T>
void d2d(T* dst, const T* src, size_t n, cudaStream_t st) {
    if (n) vgpu::check(cudaMemcpyAsync(dst, src, n * sizeof(T), cudaMemcpyDeviceToDevice, st), "d2d");
}
void sync(cudaStream_t st) { vgpu::check(cudaStreamSynchronize(st), "cudaStreamSynchronize"); }

bool env_flag(const char* name) {
    const char* v = std::getenv(name);
    return v && v[0] == '1';
}

}  // namespace

class IvfPqIndex::Impl {
public:
    Impl() {
        vgpu::check(cudaGetDevice(&dev), "cudaGetDevice");
        vgpu::check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
        for (auto& e : ev) vgpu::check(cudaEventCreate(&e), "cudaEventCreate");
    }
    ~Impl() {
        if (st) { cudaStreamSynchronize(st); cudaStreamDestroy(st); }
        for (auto& e : ev) if (e) cudaEventDestroy(e);
    }

    // ------------------------------------------------------------------ state
    int dev = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[6] = {};
    mutable std::mutex mu;

    bool trained = false;
    size_t dim = 0, dsub = 0;
    IvfPqTrainParams params;
    uint32_t ksub = 256;
    bool has_rot = false;
    std::string metadata_json;

    std::vector<float> h_cent, h_cb, h_rot;
    std::vector<uint64_t> h_offs;   // [nlist + 1]

    DeviceBuffer<float> d_cent, d_cb, d_rot, d_rotT, d_rc, d_cn;
    DeviceBuffer<float> d_rot3;   // [dim x 3 dim]: R split for the tensor-core query rotation
    mutable DeviceBuffer<int> d_err;
    mutable DeviceBuffer<float> w_xn, w_cn;
    DeviceBuffer<uint64_t> d_offs, d_ids;
    DeviceBuffer<uint8_t> d_codes;
    DeviceBuffer<float> d_vterm;
    size_t n_vectors = 0;
    // Blocked copy of the lists for the FAST scan (built after every add / load).
    bool has_blocks = false;
    // Mean size of the list holding a random entry (sum |l|^2 / sum |l|): the expected
    // size of a list a query from the data's distribution probes.
    double weighted_list_len = 0.0;
    DeviceBuffer<uint64_t> d_blk_off;
    DeviceBuffer<uint8_t> d_bcodes;
    DeviceBuffer<float> d_bvterm;
    // Tensor-core list scan: bf16 codebooks, per-entry decoded norms, batch scratch.
    DeviceBuffer<uint16_t> d_cbb;
    DeviceBuffer<float> d_xnorm;
    mutable vgpu::TlWork tlw;
    mutable DeviceBuffer<float> w_pbase;
    // threshold exchange between shards (set_threshold_exchange)
    IvfPqIndex::ThresholdExchangeFn tau_fn = nullptr;
    void* tau_user = nullptr;
    uint32_t tau_shard = 0, tau_shards = 1;
    mutable DeviceBuffer<float> w_tau_inf;

    double t_assign_ms = 0, t_encode_ms = 0, t_lists_ms = 0;
    mutable SearchTimings timings;

    // search workspace (grow-only), guarded by mu
    mutable DeviceBuffer<float> w_q, w_D, w_probe_d, w_rq, w_rq3, w_rres, w_cand_d, w_out_d, w_T;
    mutable DeviceBuffer<uint32_t> w_probe, w_cand_pos, w_cand_n, w_out_n, w_pair_q;
    mutable DeviceBuffer<uint64_t> w_out_ids;
    mutable DeviceBuffer<unsigned long long> w_scanned;
    mutable Pinned pin_a, pin_b, pin_c;
    mutable std::unique_ptr<vgpu::KmeansEngine> kme;
    mutable vgpu::FlatWork w_flat;   // the coarse probe's sampled-threshold filter
    // Exact rerank: id -> first entry map (rebuilt after the lists change) and scratch.
    mutable bool id_map_ok = false;
    mutable DeviceBuffer<uint64_t> d_sid, w_pool_ids;
    mutable DeviceBuffer<uint32_t> d_sent, w_iota, w_pool_n, w_rr_ent, w_rr_lst;
    mutable DeviceBuffer<unsigned char> w_cub;
    mutable DeviceBuffer<float> w_pool_d, w_rr_q, w_rr_dec, w_rr_rot, w_rr_exact;
    mutable DeviceBuffer<float> w_rc_dec, w_rc_rot;
    mutable DeviceBuffer<uint32_t> w_lookup;
    mutable DeviceBuffer<unsigned long long> w_count;

    uint32_t nlist() const { return params.nlist; }
    uint32_t m() const { return params.m; }

    // ------------------------------------------------------------------ helpers
    void upload_model() {
        d_cent.resize(h_cent.size());
        h2d(d_cent.data(), h_cent.data(), h_cent.size(), st);
        d_cn.resize(nlist());
        vgpu::launch_row_norms(d_cent.data(), nlist(), (int)dim, d_cn.data(), st);
        d_cb.resize(h_cb.size());
        h2d(d_cb.data(), h_cb.data(), h_cb.size(), st);
        if (has_rot) {
            d_rot.resize(dim * dim);
            h2d(d_rot.data(), h_rot.data(), dim * dim, st);
            d_rotT.resize(dim * dim);
            vgpu::launch_transpose(d_rot.data(), (int)dim, d_rotT.data(), st);
            d_rc.resize(h_cent.size());
            vgpu::launch_rotate_fast(d_cent.data(), nlist(), (int)dim, d_rot.data(), d_rc.data(), st);
            if (vgpu::rotate_3xtf32_supported((int)dim)) {
                d_rot3.resize(dim * dim * 3);
                // the rotation computes x R (apply_rotation), i.e. row j of the product's
                // second operand is column j of R: the GEMM takes R^T
                vgpu::prepare_rotation_3xtf32(d_rotT.data(), (int)dim, d_rot3.data(), st);
            } else {
                d_rot3.release();
            }
        } else {
            d_rot.release();
            d_rotT.release();
            d_rot3.release();
            d_rc.resize(h_cent.size());
            d2d(d_rc.data(), d_cent.data(), h_cent.size(), st);
        }
    }

    void reset_lists() {
        h_offs.assign(nlist() + 1, 0);
        d_offs.resize(nlist() + 1);
        h2d(d_offs.data(), h_offs.data(), h_offs.size(), st);
        d_ids.release();
        d_codes.release();
        d_vterm.release();
        n_vectors = 0;
        id_map_ok = false;
        has_blocks = false;
        d_bcodes.release();
        d_bvterm.release();
        d_xnorm.release();
    }

    void rebuild_blocks() {
        id_map_ok = false;
        has_blocks = false;
        d_bcodes.release();
        d_bvterm.release();
        d_xnorm.release();
        if (!vgpu::scan_blocked_supported((int)m(), (int)ksub)) return;
        std::vector<uint64_t> boff(nlist() + 1, 0);
        double s1 = 0.0, s2 = 0.0;
        for (uint32_t l = 0; l < nlist(); ++l) {
            const double len = (double)(h_offs[l + 1] - h_offs[l]);
            s1 += len;
            s2 += len * len;
            boff[l + 1] = boff[l] + (h_offs[l + 1] - h_offs[l] + 127) / 128;
        }
        weighted_list_len = s1 > 0 ? s2 / s1 : 0.0;
        const uint64_t nb = boff[nlist()];
        d_blk_off.resize(nlist() + 1);
        h2d(d_blk_off.data(), boff.data(), boff.size(), st);
        d_bcodes.resize(std::max<uint64_t>(nb, 1) * 128 * m());
        d_bvterm.resize(std::max<uint64_t>(nb, 1) * 128);
        if (nb) vgpu::launch_build_blocks(d_codes.data(), d_vterm.data(), d_offs.data(), d_blk_off.data(), (int)m(),
                                          (int)nlist(), d_bcodes.data(), d_bvterm.data(), st);
        if (vgpu::tc_list_scan_supported((int)dim, (int)m(), (int)ksub)) {
            // Tensor-core list scan: bf16 codebooks and per-entry decoded norms.
            d_cbb.resize((size_t)m() * ksub * dsub);
            vgpu::launch_codebook_bf16(d_cb.data(), (long long)d_cbb.size(), d_cbb.data(), st);
            d_xnorm.resize(std::max<size_t>(n_vectors, 1));
            vgpu::launch_entry_norms(d_codes.data(), (long long)n_vectors, d_cb.data(), (int)m(), (int)dsub,
                                     d_xnorm.data(), st);
        }
        sync(st);
        has_blocks = true;
    }

    // VGPU_SCAN=split: the blocked scan with each query's blocks spread over several CTAs.
    static bool use_split_scan() {
        const char* v = std::getenv("VGPU_SCAN");
        return v && std::string(v) == "split";
    }

    // FAST-scan kernel for this call: the tensor-core list scan where the shapes allow
    // it and the batch scans enough entries per query to amortise its set-up, else the
    // blocked scan.  VGPU_SCAN=tc / blocked overrides the choice.
    // VGPU_ROTATE=seq keeps FAST search on the sequential fp32 rotation kernel.
    bool use_rotation_gemm() const {
        static const bool off = [] {
            const char* v = std::getenv("VGPU_ROTATE");
            return v && std::string(v) == "seq";
        }();
        return !off && d_rot3.size() > 0;
    }

    bool use_list_scan(size_t nq, uint32_t np) const {
        if (!has_blocks || np < 2 || !vgpu::tc_list_scan_supported((int)dim, (int)m(), (int)ksub)) return false;
        const char* v = std::getenv("VGPU_SCAN");
        if (v && std::string(v) == "tc") return true;
        if (v && (std::string(v) == "blocked" || std::string(v) == "split")) return false;
        // Expected entries a query scans: its probes weighted by list size (uneven lists
        // put queries in the long ones), not the mean list size.
        const double per_query = weighted_list_len * np;
        return per_query >= 1024.0 && nq >= 256;
    }

    // The coarse probe's route for queries at dq: the tensor-core filter with the
    // sampled threshold (launch_exact_nearest) unless the shapes rule the tensor cores
    // out or VGPU_NEAREST=screen asks for the one-pass screen + screen_select.
    bool filter_probe(const float* dq) const {
        return vgpu::use_tensor_cores(dq, d_cent.data(), (int)dim, nlist()) && !vgpu::screen_all_columns();
    }

    void recompute_vterms() {
        d_vterm.resize(std::max<size_t>(n_vectors, 1));
        vgpu::launch_vector_terms(d_rc.data(), (int)nlist(), (int)dim, d_cb.data(), (int)m(), (int)ksub,
                                  (int)dsub, d_offs.data(), d_codes.data(), (long long)n_vectors,
                                  d_vterm.data(), st);
    }

    // Brute-force assignment (the reference's brute branch, src/index/ivf_pq.cpp:3252-3265).
    void assign_rows(const float* d_x, size_t n, int d, const float* d_c, uint32_t k, uint32_t* d_assign) const {
        kmeans_engine().assign(d_x, n, d, d_c, k, d_assign, nullptr, false);
    }
    vgpu::KmeansEngine& kmeans_engine() const {
        if (!kme) kme = std::make_unique<vgpu::KmeansEngine>(st);
        return *kme;
    }

    void reset_err() const {
        d_err.reserve(1);
        vgpu::check(cudaMemsetAsync(d_err.data(), 0, sizeof(int), st), "memset err");
    }
    // Reads the device error word of the tensor-core kernels (synchronizes the stream).
    void check_err() const {
        int e = 0;
        d2h(&e, d_err.data(), 1, st);
        sync(st);
        if (e) throw vgpu::CudaError("tensor-core screen: bounded wait expired (code " + std::to_string(e) + ")");
    }

    // Sum of a device float array in index order, in fp64 (host).
    double ordered_sum(const float* d, size_t n) const {
        float* h = pin_a.get<float>(n);
        d2h(h, d, n, st);
        sync(st);
        double t = 0.0;
        for (size_t i = 0; i < n; ++i) t += h[i];
        return t;
    }

    // FastScanPq::train (src/index/pq_fastscan.cpp:15-76): one k-means per sub-space,
    // all sub-spaces advanced together on the GPU.  x: [n x dim] device rows.
    void pq_train(const float* d_x, size_t n, float* d_out_cb) {
        const int M = (int)m(), DS = (int)dsub, K = (int)ksub, D = (int)dim;
        vgpu::check(cudaMemsetAsync(d_out_cb, 0, sizeof(float) * (size_t)M * K * DS, st), "memset cb");
        if (n < (size_t)K) return;  // the reference's sub-k-means fails; codebooks stay 0
        std::vector<std::mt19937> gens;
        for (int s = 0; s < M; ++s) gens.emplace_back(42u + (uint32_t)s);
        std::vector<uint32_t> pick(M);
        DeviceBuffer<uint32_t> d_pick(M);
        DeviceBuffer<float> picks((size_t)M * DS), mind((size_t)M * n);
        for (int s = 0; s < M; ++s) {
            std::uniform_int_distribution<size_t> first(0, n - 1);
            pick[s] = (uint32_t)first(gens[s]);
        }
        h2d(d_pick.data(), pick.data(), M, st);
        vgpu::launch_pq_gather_picks(d_x, D, M, DS, d_pick.data(), 0, K, picks.data(), d_out_cb, st);
        vgpu::launch_fill(mind.data(), (long long)M * n, std::numeric_limits<float>::max(), st);
        float* h = pin_b.get<float>((size_t)M * n);
        const unsigned nthreads = std::max(1u, std::min<unsigned>(std::thread::hardware_concurrency(), (unsigned)M));
        for (int c = 1; c < K; ++c) {
            vgpu::launch_pq_kpp_update(d_x, (long long)n, D, M, DS, picks.data(), mind.data(), st);
            d2h(h, mind.data(), (size_t)M * n, st);
            sync(st);
            auto work = [&](unsigned t) {
                std::vector<double> cum(n);
                for (int s = (int)t; s < M; s += (int)nthreads) {
                    const float* hs = h + (size_t)s * n;
                    cum[0] = hs[0];
                    for (size_t i = 1; i < n; ++i) cum[i] = cum[i - 1] + hs[i];
                    std::uniform_real_distribution<double> sd(0.0, cum.back());
                    const double target = sd(gens[s]);
                    pick[s] = (uint32_t)(std::lower_bound(cum.begin(), cum.end(), target) - cum.begin());
                }
            };
            std::vector<std::thread> pool;
            for (unsigned t = 1; t < nthreads; ++t) pool.emplace_back(work, t);
            work(0);
            for (auto& th : pool) th.join();
            h2d(d_pick.data(), pick.data(), M, st);
            vgpu::launch_pq_gather_picks(d_x, D, M, DS, d_pick.data(), c, K, picks.data(), d_out_cb, st);
        }
        // Elkan iterations per sub-space.
        DeviceBuffer<uint32_t> codes((size_t)M * n), keys((size_t)M * n), order((size_t)M * n),
            seg((size_t)M * K + 1);
        DeviceBuffer<int> d_active(M);
        std::vector<int> active(M, 1);
        std::vector<float> prev(M, std::numeric_limits<float>::max());
        vgpu::GroupWork gw;
        h2d(d_active.data(), active.data(), M, st);
        vgpu::launch_pq_assign(d_x, (long long)n, D, M, K, DS, d_out_cb, codes.data(), mind.data(), 0,
                               nullptr, st);
        for (uint32_t it = 0; it < 25; ++it) {
            if (it > 0)
                vgpu::launch_pq_assign(d_x, (long long)n, D, M, K, DS, d_out_cb, codes.data(), mind.data(),
                                       1, d_active.data(), st);
            d2h(h, mind.data(), (size_t)M * n, st);
            sync(st);
            bool any = false;
            for (int s = 0; s < M; ++s) {
                if (!active[s]) continue;
                double t = 0.0;
                const float* hs = h + (size_t)s * n;
                for (size_t i = 0; i < n; ++i) t += hs[i];
                const float inertia = (float)t;
                const float change = std::fabs(prev[s] - inertia) / (prev[s] + 1e-10f);
                if (change < 1e-4f) { active[s] = 0; continue; }
                prev[s] = inertia;
                any = true;
            }
            if (!any) break;
            h2d(d_active.data(), active.data(), M, st);
            vgpu::launch_pq_keys(codes.data(), (long long)n, M, K, keys.data(), st);
            vgpu::group_by_key(keys.data(), (long long)M * n, M * K, order.data(), seg.data(), gw, st);
            vgpu::launch_pq_segment_mean(d_x, (long long)n, D, M, DS, K, order.data(), seg.data(),
                                         d_active.data(), d_out_cb, st);
        }
        sync(st);
    }

    // Mean squared reconstruction error (compute_error lambda, ivf_pq.cpp:2468-2490):
    // encode -> decode (-> R^T) -> l2 to the original residual, fp64 mean.
    double recon_error(const float* d_enc_in, const float* d_res, size_t n, const float* d_cbk,
                       const float* d_RT) {
        DeviceBuffer<uint8_t> codes(n * m());
        DeviceBuffer<float> dec(n * dim), back, l2(n);
        vgpu::launch_pq_encode(d_enc_in, (long long)n, (int)m(), (int)ksub, (int)dsub, d_cbk, codes.data(), st);
        vgpu::launch_pq_decode(codes.data(), (long long)n, (int)m(), (int)ksub, (int)dsub, d_cbk, dec.data(), st);
        const float* cmp = dec.data();
        if (d_RT) {
            back.resize(n * dim);
            vgpu::launch_residual_rotate(dec.data(), nullptr, nullptr, nullptr, (long long)n, (int)dim, d_RT,
                                         back.data(), st);
            cmp = back.data();
        }
        vgpu::launch_row_l2(cmp, d_res, (long long)n, (int)dim, l2.data(), st);
        return ordered_sum(l2.data(), n) / (double)n;
    }

    // learn_opq_rotation (src/index/ivf_pq.cpp:2769-2945) on device residual rows.
    std::expected<void, error> learn_opq_rotation(const float* d_x, size_t n) {
        if (n < dim * 2)
            return fail(error_code::precondition_failed, "Not enough data for OPQ rotation learning");
        const int d = (int)dim;
        DeviceBuffer<double> mean(dim), cov(dim * dim), E(dim * dim), work(3 * dim + 4);
        vgpu::launch_col_mean(d_x, (long long)n, d, mean.data(), st);
        vgpu::launch_cross_fp64(d_x, d_x, (long long)n, d, mean.data(), mean.data(), cov.data(), st);
        vgpu::launch_daxpby(cov.data(), cov.data(), (long long)dim * dim, 0.0, 1.0 / (double)(n - 1), st);
        vgpu::power_iteration_pca(cov.data(), d, 100, 1e-6, E.data(), work.data(), st);
        std::vector<double> hE(dim * dim);
        d2h(hE.data(), E.data(), dim * dim, st);
        sync(st);
        h_rot.assign(dim * dim, 0.0f);
        for (size_t i = 0; i < dim * dim; ++i) h_rot[i] = (float)hE[i];
        // Orthogonality check with identity fallback (:2924-2942).
        bool bad = false;
        for (size_t i = 0; i < dim && !bad; ++i)
            for (size_t j = i + 1; j < dim; ++j) {
                double dot = 0.0;
                for (size_t k = 0; k < dim; ++k) dot += h_rot[i * dim + k] * h_rot[j * dim + k];
                if (std::abs(dot) > 0.01) { bad = true; break; }
            }
        if (bad) {
            std::fill(h_rot.begin(), h_rot.end(), 0.0f);
            for (size_t k = 0; k < dim; ++k) h_rot[k * dim + k] = 1.0f;
        }
        return {};
    }

    // The Procrustes rotation as the reference computes it (src/index/ivf_pq.cpp:2636-2698):
    // one-sided Jacobi sweeps on the columns of A = C (at most 20, stopping when the sum of
    // squared column inner products falls below 1e-10 d^2; pairs with |<a_p, a_q>| < 1e-10
    // are left alone), U = A's columns normalised, R = U V^T.  Host fp64, every sum in the
    // reference's order and no fused multiply-add, so R equals the reference's bit for
    // bit given the same C.  O(20 d^3): used up to kJacobiMaxDim.
    std::vector<float> jacobi_polar(const std::vector<double>& C) const {
        const size_t d = dim;
        const double tol = 1e-10;
        std::vector<double> A = C, V(d * d, 0.0), U(d * d, 0.0);
        for (size_t i = 0; i < d; ++i) { U[i * d + i] = 1.0; V[i * d + i] = 1.0; }
        auto rotate_cols = [d](std::vector<double>& M, size_t p, size_t q, double c, double s) {
            for (size_t i = 0; i < d; ++i) {
                const double mp = M[i * d + p], mq = M[i * d + q];
                M[i * d + p] = c * mp - s * mq;
                M[i * d + q] = s * mp + c * mq;
            }
        };
        for (int sweep = 0; sweep < 20; ++sweep) {
            double off = 0.0;
            for (size_t p = 0; p + 1 < d; ++p)
                for (size_t q = p + 1; q < d; ++q) {
                    double app = 0.0, aqq = 0.0, apq = 0.0;
                    for (size_t i = 0; i < d; ++i) {
                        const double ap = A[i * d + p], aq = A[i * d + q];
                        app += ap * ap;
                        aqq += aq * aq;
                        apq += ap * aq;
                    }
                    off += apq * apq;
                    if (std::abs(apq) < tol) continue;
                    const double tau = (aqq - app) / (2.0 * apq);
                    const double t = tau >= 0 ? 1.0 / (tau + std::sqrt(1.0 + tau * tau))
                                              : -1.0 / (-tau + std::sqrt(1.0 + tau * tau));
                    const double c = 1.0 / std::sqrt(1.0 + t * t);
                    const double s = t * c;
                    rotate_cols(A, p, q, c, s);
                    rotate_cols(V, p, q, c, s);
                }
            if (off < tol * (double)d * (double)d) break;
        }
        for (size_t i = 0; i < d; ++i) {
            double norm = 0.0;
            for (size_t j = 0; j < d; ++j) norm += A[j * d + i] * A[j * d + i];
            norm = std::sqrt(norm);
            if (norm > tol)
                for (size_t j = 0; j < d; ++j) U[j * d + i] = A[j * d + i] / norm;
        }
        std::vector<float> R(d * d);
        for (size_t i = 0; i < d; ++i)
            for (size_t j = 0; j < d; ++j) {
                double sum = 0.0;
                for (size_t k = 0; k < d; ++k) sum += U[i * d + k] * V[j * d + k];
                R[i * d + j] = (float)sum;
            }
        return R;
    }

    // Orthogonal polar factor of C (d x d, fp64, device) by Newton-Schulz; result in
    // float R (host).
    std::vector<float> polar_factor(DeviceBuffer<double>& C) {
        const int d = (int)dim;
        std::vector<double> hC(dim * dim);
        d2h(hC.data(), C.data(), dim * dim, st);
        sync(st);
        double fro = 0.0;
        for (double v : hC) fro += v * v;
        fro = std::sqrt(fro);
        std::vector<float> R(dim * dim, 0.0f);
        if (!(fro > 0.0)) {
            for (size_t k = 0; k < dim; ++k) R[k * dim + k] = 1.0f;
            return R;
        }
        DeviceBuffer<double> X(dim * dim), T(dim * dim), Y(dim * dim);
        d2d(X.data(), C.data(), dim * dim, st);
        vgpu::launch_daxpby(X.data(), X.data(), (long long)dim * dim, 0.0, 1.0 / fro, st);
        for (int it = 0; it < 80; ++it) {
            vgpu::launch_dgemm(X.data(), X.data(), T.data(), d, 1, 0, 1.0, 0.0, st);   // T = X^T X
            d2d(Y.data(), X.data(), dim * dim, st);
            vgpu::launch_dgemm(X.data(), T.data(), Y.data(), d, 0, 0, -0.5, 1.5, st);  // Y = 1.5X - 0.5 X T
            std::swap(X, Y);
        }
        std::vector<double> hX(dim * dim);
        d2h(hX.data(), X.data(), dim * dim, st);
        sync(st);
        for (size_t i = 0; i < dim * dim; ++i) R[i] = (float)hX[i];
        return R;
    }

    std::expected<IvfPqTrainStats, error> train(const float* data, size_t dim_, size_t n,
                                                const IvfPqTrainParams& p, bool on_device) {
        if (n < p.nlist)
            return fail(error_code::precondition_failed, "Not enough training data for nlist centroids");
        if (p.m == 0 || dim_ % p.m != 0)
            return fail(error_code::precondition_failed, "Dimension must be divisible by number of subquantizers");
        if (p.nbits == 0 || p.nbits > 8)
            return fail(error_code::precondition_failed, "nbits must be in [1, 8] (codes are stored as bytes)");
        if (p.nlist == 0)
            return fail(error_code::precondition_failed, "nlist must be > 0");
        const auto t0 = std::chrono::steady_clock::now();
        trained = false;
        params = p;
        dim = dim_;
        dsub = dim / p.m;
        ksub = 1u << p.nbits;
        has_rot = false;
        h_rot.clear();
        if (params.nlist < 1024 && params.use_centroid_ann) params.use_centroid_ann = false;

        DeviceBuffer<float> x_own;
        const float* xp = data;
        if (!on_device) {
            x_own.resize(n * dim);
            h2d(x_own.data(), data, n * dim, st);
            xp = x_own.data();
        }
        d_cent.resize((size_t)nlist() * dim);
        DeviceBuffer<uint32_t> assign(n);
        IvfPqTrainStats stats;
        // Step 1: coarse quantizer (train_coarse_quantizer, :561-671).
        auto km = kmeans_engine().fit(xp, n, (int)dim, nlist(), p.max_iter, p.epsilon, p.seed, true,
                                      d_cent.data(), assign.data());
        stats.coarse_iterations = km.iterations;
        h_cent.resize((size_t)nlist() * dim);
        d2h(h_cent.data(), d_cent.data(), h_cent.size(), st);

        // Residuals of the training data w.r.t. the nearest centroid (:477-494, :2414-2432).
        DeviceBuffer<float> res(n * dim);
        assign_rows(xp, n, (int)dim, d_cent.data(), nlist(), assign.data());
        vgpu::launch_residual_rotate(xp, nullptr, d_cent.data(), assign.data(), (long long)n, (int)dim,
                                     nullptr, res.data(), st);
        x_own.release();

        // Step 2: OPQ PCA initialisation (:457-519).
        if (p.use_opq && p.opq_init == OpqInit::PCA) {
            const size_t cap = p.opq_sample_n > 0 ? p.opq_sample_n : 50000;
            const size_t n_pca = std::min(n, cap);
            if (n_pca == n) {
                if (auto r = learn_opq_rotation(res.data(), n); !r) return std::unexpected(r.error());
            } else {
                std::vector<uint32_t> idx(n_pca);
                const double stride = (double)n / (double)n_pca;
                for (size_t i = 0; i < n_pca; ++i) {
                    size_t j = (size_t)(i * stride);
                    if (j >= n) j = n - 1;
                    idx[i] = (uint32_t)j;
                }
                DeviceBuffer<uint32_t> d_idx(n_pca);
                DeviceBuffer<float> samp(n_pca * dim);
                h2d(d_idx.data(), idx.data(), n_pca, st);
                vgpu::launch_gather_rows(res.data(), (int)dim, d_idx.data(), (long long)n_pca, samp.data(), st);
                if (auto r = learn_opq_rotation(samp.data(), n_pca); !r) return std::unexpected(r.error());
            }
        }

        // Step 3: product quantizer (+ OPQ alternation) (:2398-2767).
        d_cb.resize((size_t)m() * ksub * dsub);
        DeviceBuffer<float> cb_unrot((size_t)m() * ksub * dsub);
        pq_train(res.data(), n, cb_unrot.data());
        const double err_unrot = recon_error(res.data(), res.data(), n, cb_unrot.data(), nullptr);
        stats.err_unrot = err_unrot;
        double err_best = std::numeric_limits<double>::infinity();
        DeviceBuffer<float> cb_opq;
        std::vector<float> R_best;
        if (p.use_opq) {
            if (h_rot.empty()) {
                h_rot.assign(dim * dim, 0.0f);
                for (size_t k = 0; k < dim; ++k) h_rot[k * dim + k] = 1.0f;
            }
            const uint32_t iters = std::max<uint32_t>(1, std::min<uint32_t>(p.opq_iter, 3));
            const size_t cap = p.opq_sample_n > 0 ? p.opq_sample_n : 20000;
            const size_t n_opq = std::min(n, cap);
            DeviceBuffer<float> R(dim * dim), RT(dim * dim), rot(n_opq * dim), cbt((size_t)m() * ksub * dsub),
                Y(n_opq * dim), Yb(n_opq * dim), l2(n_opq);
            DeviceBuffer<uint8_t> codes(n_opq * m());
            DeviceBuffer<double> C(dim * dim);
            const auto topq = std::chrono::steady_clock::now();
            double prev_err = std::numeric_limits<double>::infinity();
            uint32_t stall = 0;
            for (uint32_t it = 0; it < iters; ++it) {
                h2d(R.data(), h_rot.data(), dim * dim, st);
                vgpu::launch_transpose(R.data(), (int)dim, RT.data(), st);
                vgpu::launch_residual_rotate(res.data(), nullptr, nullptr, nullptr, (long long)n_opq, (int)dim,
                                             R.data(), rot.data(), st);
                pq_train(rot.data(), n_opq, cbt.data());
                vgpu::launch_pq_encode(rot.data(), (long long)n_opq, (int)m(), (int)ksub, (int)dsub, cbt.data(),
                                       codes.data(), st);
                vgpu::launch_pq_decode(codes.data(), (long long)n_opq, (int)m(), (int)ksub, (int)dsub, cbt.data(),
                                       Y.data(), st);
                vgpu::launch_residual_rotate(Y.data(), nullptr, nullptr, nullptr, (long long)n_opq, (int)dim,
                                             RT.data(), Yb.data(), st);
                vgpu::launch_row_l2(Yb.data(), res.data(), (long long)n_opq, (int)dim, l2.data(), st);
                const double err_it = ordered_sum(l2.data(), n_opq) / (double)n_opq;
                stats.errors.push_back((float)err_it);
                if (err_it < err_best) { err_best = err_it; R_best = h_rot; }
                if (std::isfinite(prev_err)) {
                    const double denom = std::max(prev_err, 1e-12);
                    if ((prev_err - err_it) / denom < 1e-4) ++stall; else stall = 0;
                }
                prev_err = err_it;
                if (stall >= 2) break;
                const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                                    std::chrono::steady_clock::now() - topq).count();
                if (el > 120000) break;
                // Procrustes on the sample: C = X^T Y / n, R = polar(C): the reference's
                // Jacobi iteration up to kJacobiMaxDim, a Newton-Schulz polar factor on the
                // GPU above (the host sweeps are O(20 d^3)).
                if (dim <= kJacobiMaxDim) {
                    vgpu::launch_cross_fp64_unfused(res.data(), Y.data(), (long long)n_opq, (int)dim, C.data(), st);
                    std::vector<double> hC(dim * dim);
                    d2h(hC.data(), C.data(), dim * dim, st);
                    sync(st);
                    const double invn = 1.0 / (double)n_opq;
                    for (double& v : hC) v *= invn;
                    h_rot = jacobi_polar(hC);
                } else {
                    vgpu::launch_cross_fp64(res.data(), Y.data(), (long long)n_opq, (int)dim, nullptr, nullptr,
                                            C.data(), st);
                    vgpu::launch_daxpby(C.data(), C.data(), (long long)dim * dim, 0.0, 1.0 / (double)n_opq, st);
                    h_rot = polar_factor(C);
                }
            }
            if (!R_best.empty()) h_rot = R_best;
            if (err_best < std::numeric_limits<double>::infinity()) {
                DeviceBuffer<float> rot_full(n * dim);
                h2d(R.data(), h_rot.data(), dim * dim, st);
                vgpu::launch_residual_rotate(res.data(), nullptr, nullptr, nullptr, (long long)n, (int)dim,
                                             R.data(), rot_full.data(), st);
                cb_opq.resize((size_t)m() * ksub * dsub);
                pq_train(rot_full.data(), n, cb_opq.data());
            }
        }
        stats.err_opq = err_best;
        const bool force = env_flag("VESPER_IVFPQ_FORCE_OPQ");
        if ((force && p.use_opq && !h_rot.empty() && cb_opq.size()) || err_best < err_unrot) {
            d2d(d_cb.data(), cb_opq.data(), d_cb.size(), st);
            has_rot = true;
        } else {
            d2d(d_cb.data(), cb_unrot.data(), d_cb.size(), st);
            h_rot.clear();
            has_rot = false;
        }
        stats.opq_kept = has_rot;
        h_cb.resize(d_cb.size());
        d2h(h_cb.data(), d_cb.data(), h_cb.size(), st);
        sync(st);
        upload_model();
        reset_lists();
        sync(st);
        trained = true;
        stats.iterations = 25;
        stats.train_time_sec = std::chrono::duration<float>(std::chrono::steady_clock::now() - t0).count();
        return stats;
    }

    // ------------------------------------------------------------------ add
    std::expected<void, error> add(const uint64_t* ids, const float* data, size_t n, bool on_device) {
        if (!trained) return fail(error_code::precondition_failed, "Index must be trained before adding vectors");
        if (n == 0) return {};
        const auto ta = std::chrono::steady_clock::now();
        const size_t M = m();
        DeviceBuffer<uint32_t> assign(n);
        DeviceBuffer<uint8_t> new_codes(n * M);
        {
            // Row chunks bounded by the residual buffer, and by the distance matrix when
            // the assignment writes one (the fused tensor-core arg-min does not).
            const bool fused = vgpu::use_tensor_cores(on_device ? data : d_cent.data(), d_cent.data(), (int)dim,
                                                      nlist()) && !vgpu::screen_all_columns();
            const size_t width = fused ? dim : std::max<size_t>(nlist(), dim);
            const size_t rows = std::max<size_t>(1, std::min<size_t>(n, kDistBudget / (sizeof(float) * width)));
            DeviceBuffer<float> x(on_device ? 0 : rows * dim), res(rows * dim);
            for (size_t r0 = 0; r0 < n; r0 += rows) {
                const size_t nr = std::min(rows, n - r0);
                const float* xr = data + r0 * dim;
                if (!on_device) {
                    h2d(x.data(), xr, nr * dim, st);
                    xr = x.data();
                }
                assign_rows(xr, nr, (int)dim, d_cent.data(), nlist(), assign.data() + r0);
                vgpu::launch_residual_rotate(xr, nullptr, d_cent.data(), assign.data() + r0, (long long)nr,
                                             (int)dim, has_rot ? d_rot.data() : nullptr, res.data(), st);
                vgpu::launch_pq_encode(res.data(), (long long)nr, (int)M, (int)ksub, (int)dsub, d_cb.data(),
                                       new_codes.data() + r0 * M, st);
            }
        }
        sync(st);
        const auto tb = std::chrono::steady_clock::now();
        // Append to the lists in input order (:3410-3427): stable destinations on host.
        std::vector<uint32_t> ha(n);
        d2h(ha.data(), assign.data(), n, st);
        sync(st);
        const uint32_t L = nlist();
        std::vector<uint64_t> cnt(L, 0);
        for (size_t i = 0; i < n; ++i) cnt[ha[i]]++;
        std::vector<uint64_t> new_offs(L + 1, 0);
        for (uint32_t l = 0; l < L; ++l) new_offs[l + 1] = new_offs[l] + (h_offs[l + 1] - h_offs[l]) + cnt[l];
        std::vector<uint64_t> cursor(L);
        for (uint32_t l = 0; l < L; ++l) cursor[l] = new_offs[l] + (h_offs[l + 1] - h_offs[l]);
        std::vector<uint64_t> dest(n);
        for (size_t i = 0; i < n; ++i) dest[i] = cursor[ha[i]]++;
        const size_t total = n_vectors + n;
        DeviceBuffer<uint8_t> codes(total * M);
        DeviceBuffer<uint64_t> allids(total), d_new_offs(L + 1), d_dest(n), d_newids(n);
        h2d(d_new_offs.data(), new_offs.data(), L + 1, st);
        h2d(d_dest.data(), dest.data(), n, st);
        if (on_device) d2d(d_newids.data(), ids, n, st); else h2d(d_newids.data(), ids, n, st);
        if (n_vectors)
            vgpu::launch_csr_move(d_codes.data(), d_ids.data(), d_offs.data(), d_new_offs.data(), (int)L, (int)M,
                                  codes.data(), allids.data(), st);
        vgpu::launch_csr_scatter(new_codes.data(), d_newids.data(), d_dest.data(), (long long)n, (int)M,
                                 codes.data(), allids.data(), st);
        d_codes = std::move(codes);
        d_ids = std::move(allids);
        d_offs = std::move(d_new_offs);
        h_offs = std::move(new_offs);
        n_vectors = total;
        recompute_vterms();
        rebuild_blocks();
        sync(st);
        const auto tc = std::chrono::steady_clock::now();
        if (params.timings_enabled || params.verbose || env_flag("VESPER_TIMING")) {
            t_assign_ms += std::chrono::duration<double, std::milli>(tb - ta).count();
            t_lists_ms += std::chrono::duration<double, std::milli>(tc - tb).count();
        }
        return {};
    }

    // ------------------------------------------------------------------ search
    std::expected<void, error> search_flat(const float* queries, size_t nq, const IvfPqSearchParams& sp,
                                           uint64_t* out_ids, float* out_d, uint32_t* out_n,
                                           bool on_device) const {
        // VESPER_IVFPQ_RERANK=1 forces the rerank as in the reference (ivf_pq.cpp:3543).
        if (sp.use_exact_rerank || env_flag("VESPER_IVFPQ_RERANK"))
            return search_rerank(queries, nq, sp, out_ids, out_d, out_n, on_device);
        return search_adc(queries, nq, sp, out_ids, out_d, out_n, on_device);
    }

    // ------------------------------------------------------------------ exact rerank
    // Impl::search with use_exact_rerank (src/index/ivf_pq.cpp:3544-3552, 3995-4091):
    // the ADC pool of pool_k = max(k, cand_k or k, rerank_k or max(3k, 1000)) candidates,
    // then the first min(rerank_k or pool_k, pool size) re-scored exactly and re-sorted.
    std::expected<void, error> search_rerank(const float* queries, size_t nq, const IvfPqSearchParams& sp,
                                             uint64_t* out_ids, float* out_d, uint32_t* out_n,
                                             bool on_device) const {
        if (!trained) return fail(error_code::precondition_failed, "Index must be trained before searching");
        if (sp.k == 0) return fail(error_code::invalid_argument, "k must be > 0");
        if (nq == 0) return {};
        const uint32_t k = sp.k;
        size_t pool = std::max<uint32_t>(k, sp.cand_k > 0 ? sp.cand_k : k);
        pool = std::max<size_t>(pool, sp.rerank_k > 0 ? sp.rerank_k : std::max<uint32_t>(k * 3, 1000));
        if (pool > (size_t)vgpu::kMaxK)
            return fail(error_code::unsupported, "the rerank candidate pool (" + std::to_string(pool) +
                                                     " = max(k, cand_k, rerank_k or max(3k, 1000))) exceeds 1024, "
                                                     "the GPU path's limit");
        const int head_cap = sp.rerank_k > 0 ? (int)sp.rerank_k : (int)pool;
        IvfPqSearchParams ap = sp;
        ap.k = (uint32_t)pool;
        ap.cand_k = 0;
        ap.use_exact_rerank = false;
        ap.rerank_k = 0;
        const size_t per_q = has_rot ? 2 * pool * dim * sizeof(float) : 0;
        size_t qc = std::min<size_t>(nq, 16384);
        if (per_q) qc = std::min(qc, std::max<size_t>(1, kDistBudget / per_q));
        SearchTimings acc;
        float rerank_ms = 0.0f;
        for (size_t q0 = 0; q0 < nq; q0 += qc) {
            const size_t nc = std::min(qc, nq - q0);
            const float* dq = queries + q0 * dim;
            if (!on_device) {
                std::lock_guard<std::mutex> lock(mu);
                w_rr_q.reserve(qc * dim);
                h2d(w_rr_q.data(), queries + q0 * dim, nc * dim, st);
                dq = w_rr_q.data();
            }
            {
                std::lock_guard<std::mutex> lock(mu);
                w_pool_ids.reserve(qc * pool);
                w_pool_d.reserve(qc * pool);
                w_pool_n.reserve(qc);
            }
            auto r = search_adc(dq, nc, ap, w_pool_ids.data(), w_pool_d.data(), w_pool_n.data(), true);
            if (!r) return r;
            std::lock_guard<std::mutex> lock(mu);
            acc.coarse_ms += timings.coarse_ms; acc.select_ms += timings.select_ms;
            acc.rotate_ms += timings.rotate_ms; acc.scan_ms += timings.scan_ms; acc.merge_ms += timings.merge_ms;
            acc.total_ms += timings.total_ms; acc.scanned_entries += timings.scanned_entries;
            acc.kernel_launches += timings.kernel_launches + 3 + (has_rot ? 1 : 0);
            acc.scan_variant = timings.scan_variant; acc.coarse_variant = timings.coarse_variant;
            acc.list_kernel_ms += timings.list_kernel_ms; acc.list_candidates += timings.list_candidates;
            acc.list_fallback_queries += timings.list_fallback_queries;
            acc.list_threshold_ms += timings.list_threshold_ms; acc.list_prep_ms += timings.list_prep_ms;
            acc.list_refine_ms += timings.list_refine_ms; acc.list_fallback_ms += timings.list_fallback_ms;
            if (!id_map_ok) acc.kernel_launches += 3;
            ensure_id_map();
            w_rr_ent.reserve(qc * pool);
            w_rr_lst.reserve(qc * pool);
            w_rr_exact.reserve(qc * pool);
            if (has_rot) {
                w_rr_dec.reserve(qc * pool * dim);
                w_rr_rot.reserve(qc * pool * dim);
            }
            uint64_t* oid = out_ids + q0 * k;
            float* od = out_d + q0 * k;
            uint32_t* on = out_n ? out_n + q0 : nullptr;
            if (!on_device) {
                w_out_ids.reserve(qc * k);
                w_out_d.reserve(qc * k);
                w_out_n.reserve(qc);
                oid = w_out_ids.data();
                od = w_out_d.data();
                on = w_out_n.data();
            }
            cudaEventRecord(ev[0], st);
            vgpu::RerankArgs a{};
            a.q = dq; a.pool_ids = w_pool_ids.data(); a.pool_d = w_pool_d.data(); a.pool_n = w_pool_n.data();
            a.nq = (long long)nc; a.P = (int)pool; a.head_cap = head_cap; a.k = (int)k;
            a.sid = d_sid.data(); a.sent = d_sent.data(); a.n = (long long)n_vectors;
            a.offs = d_offs.data(); a.nlist = (int)nlist(); a.codes = d_codes.data();
            a.m = (int)m(); a.ksub = (int)ksub; a.dsub = (int)dsub; a.cb = d_cb.data(); a.cent = d_cent.data();
            a.rotT = has_rot ? d_rotT.data() : nullptr;
            a.ent = w_rr_ent.data(); a.lst = w_rr_lst.data();
            a.dec = has_rot ? w_rr_dec.data() : nullptr; a.rot_out = has_rot ? w_rr_rot.data() : nullptr;
            a.exact_d = w_rr_exact.data(); a.out_ids = oid; a.out_d = od; a.out_n = on;
            vgpu::launch_rerank(a, st);
            cudaEventRecord(ev[1], st);
            if (!on_device) {
                d2h(out_ids + q0 * k, oid, nc * k, st);
                d2h(out_d + q0 * k, od, nc * k, st);
                if (out_n) d2h(out_n + q0, on, nc, st);
            }
            sync(st);
            float t = 0.0f;
            cudaEventElapsedTime(&t, ev[0], ev[1]);
            rerank_ms += t;
        }
        std::lock_guard<std::mutex> lock(mu);
        acc.rerank_ms = rerank_ms;
        acc.total_ms += rerank_ms;
        timings = acc;
        return {};
    }

    // ext_probe / ext_probe_d (device, [nq x min(nprobe, nlist)]): probe lists computed
    // elsewhere (probe_device, e.g. by another rank); the coarse stage is skipped.
    // id -> first entry in list order (stable radix sort of the ids); caller holds mu.
    void ensure_id_map() const {
        if (id_map_ok) return;
        d_sid.reserve(std::max<size_t>(n_vectors, 1));
        d_sent.reserve(std::max<size_t>(n_vectors, 1));
        vgpu::launch_id_map_build(d_ids.data(), (long long)n_vectors, d_sid.data(), d_sent.data(), w_iota, w_cub, st);
        id_map_ok = true;
    }

    // ------------------------------------------------------------------ maintenance / inspection
    // (src/index/ivf_pq.cpp:4997-5541).  Caller holds mu.
    // The first entry holding id and its list; false if absent.
    bool find_entry(uint64_t id, uint32_t& e, uint32_t& l) const {
        if (n_vectors == 0) return false;
        ensure_id_map();
        w_lookup.reserve(2);
        vgpu::launch_id_lookup(d_sid.data(), d_sent.data(), (long long)n_vectors, id, d_offs.data(), (int)nlist(),
                               w_lookup.data(), st);
        uint32_t h[2] = {0, 0};
        d2h(h, w_lookup.data(), 2, st);
        sync(st);
        e = h[0];
        l = h[1];
        return e != 0xffffffffu;
    }

    // Rebuild n entries (device entries/lists, or the range e0.. of one list) into d_out.
    void reconstruct_rows(const uint32_t* entries, uint64_t e0, const uint32_t* lists, uint32_t list0, size_t n,
                          float* d_out) const {
        w_rc_dec.reserve(std::max<size_t>(n * dim, 1));
        if (has_rot) w_rc_rot.reserve(std::max<size_t>(n * dim, 1));
        vgpu::launch_reconstruct_rows(entries, e0, lists, list0, (long long)n, d_codes.data(), (int)m(), (int)ksub,
                                      (int)dsub, d_cb.data(), d_cent.data(), has_rot ? d_rotT.data() : nullptr,
                                      w_rc_dec.data(), has_rot ? w_rc_rot.data() : nullptr, d_out, st);
    }

    std::expected<std::vector<float>, error> reconstruct(uint64_t id) const {
        if (!trained) return fail(error_code::precondition_failed, "Index not trained");
        std::lock_guard<std::mutex> lock(mu);
        uint32_t e = 0, l = 0;
        if (!find_entry(id, e, l)) return fail(error_code::not_found, "Vector ID not found");
        DeviceBuffer<float> out(dim);
        reconstruct_rows(nullptr, e, nullptr, l, 1, out.data());
        std::vector<float> h(dim);
        d2h(h.data(), out.data(), dim, st);
        sync(st);
        return h;
    }

    std::expected<void, error> reconstruct_cluster(uint32_t c, std::vector<uint64_t>& ids,
                                                   std::vector<float>& vectors) const {
        if (!trained) return fail(error_code::precondition_failed, "Index not trained");
        if (c >= nlist()) return fail(error_code::precondition_failed, "Invalid cluster ID");
        std::lock_guard<std::mutex> lock(mu);
        ids.clear();
        vectors.clear();
        const uint64_t e0 = h_offs[c], n = h_offs[c + 1] - e0;
        if (n == 0) return {};
        ids.resize(n);
        vectors.resize(n * dim);
        DeviceBuffer<float> out(n * dim);
        reconstruct_rows(nullptr, e0, nullptr, c, n, out.data());
        d2h(ids.data(), d_ids.data() + e0, n, st);
        d2h(vectors.data(), out.data(), n * dim, st);
        sync(st);
        return {};
    }

    std::expected<uint32_t, error> cluster_assignment(uint64_t id) const {
        if (!trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.get_cluster_assignment");
        std::lock_guard<std::mutex> lock(mu);
        uint32_t e = 0, l = 0;
        if (!find_entry(id, e, l)) return fail(error_code::not_found, "Vector ID not found", "ivf_pq.get_cluster_assignment");
        return l;
    }

    std::expected<void, error> update_centroid(uint32_t c, const float* centroid) {
        if (!trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.update_cluster_centroid");
        if (c >= nlist()) return fail(error_code::out_of_range, "Cluster ID out of range", "ivf_pq.update_cluster_centroid");
        if (!centroid) return fail(error_code::invalid_argument, "Null centroid pointer", "ivf_pq.update_cluster_centroid");
        std::lock_guard<std::mutex> lock(mu);
        std::copy(centroid, centroid + dim, h_cent.begin() + (size_t)c * dim);
        // the centroid and what the search derives from it: its norm, its rotation, and
        // the per-entry terms of the fast scan
        h2d(d_cent.data() + (size_t)c * dim, h_cent.data() + (size_t)c * dim, dim, st);
        vgpu::launch_row_norms(d_cent.data() + (size_t)c * dim, 1, (int)dim, d_cn.data() + c, st);
        if (has_rot)
            vgpu::launch_rotate_fast(d_cent.data() + (size_t)c * dim, 1, (int)dim, d_rot.data(),
                                     d_rc.data() + (size_t)c * dim, st);
        else
            d2d(d_rc.data() + (size_t)c * dim, d_cent.data() + (size_t)c * dim, dim, st);
        recompute_vterms();
        rebuild_blocks();
        sync(st);
        return {};
    }

    // Move entries so that the new order is `order` (old entry index per new position,
    // 0xffffffff = the single new entry taken from new_code / new_id); h_offs_new: the
    // new list offsets.  Codes, ids and everything derived from them are rebuilt.
    void relayout(const std::vector<uint32_t>& order, const std::vector<uint64_t>& h_offs_new,
                  const uint8_t* d_new_code, uint64_t new_id) {
        const size_t n = order.size();
        DeviceBuffer<uint32_t> d_order(std::max<size_t>(n, 1));
        h2d(d_order.data(), order.data(), n, st);
        DeviceBuffer<uint8_t> codes2(std::max<size_t>(n * m(), 1));
        DeviceBuffer<uint64_t> ids2(std::max<size_t>(n, 1));
        vgpu::launch_gather_entries(d_order.data(), (long long)n, d_codes.data(), d_ids.data(), (int)m(), d_new_code,
                                    new_id, codes2.data(), ids2.data(), st);
        sync(st);  // the old arrays are released below
        d_codes = std::move(codes2);
        d_ids = std::move(ids2);
        h_offs = h_offs_new;
        h2d(d_offs.data(), h_offs.data(), h_offs.size(), st);
        n_vectors = n;
        recompute_vterms();
        rebuild_blocks();
        id_map_ok = false;
        sync(st);
    }

    std::expected<void, error> reassign(uint64_t id, uint32_t nc) {
        if (!trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.reassign_vector");
        if (nc >= nlist()) return fail(error_code::out_of_range, "New cluster ID out of range", "ivf_pq.reassign_vector");
        std::lock_guard<std::mutex> lock(mu);
        uint32_t e = 0, lo = 0;
        if (!find_entry(id, e, lo)) return fail(error_code::not_found, "Vector ID not found", "ivf_pq.reassign_vector");
        // the stored vector rebuilt, its residual to the new centroid (rotated), encoded
        DeviceBuffer<float> vec(dim), res(dim);
        DeviceBuffer<uint32_t> d_nc(1);
        DeviceBuffer<uint8_t> code(m());
        reconstruct_rows(nullptr, e, nullptr, lo, 1, vec.data());
        h2d(d_nc.data(), &nc, 1, st);
        vgpu::launch_residual_rotate(vec.data(), nullptr, d_cent.data(), d_nc.data(), 1, (int)dim,
                                     has_rot ? d_rot.data() : nullptr, res.data(), st);
        vgpu::launch_pq_encode(res.data(), 1, (int)m(), (int)ksub, (int)dsub, d_cb.data(), code.data(), st);
        // new order: entry e removed, the new entry appended to list nc
        std::vector<uint32_t> order;
        order.reserve(n_vectors);
        std::vector<uint64_t> offs2(nlist() + 1, 0);
        for (uint32_t l = 0; l < nlist(); ++l) {
            for (uint64_t i = h_offs[l]; i < h_offs[l + 1]; ++i)
                if (i != e) order.push_back((uint32_t)i);
            if (l == nc) order.push_back(0xffffffffu);
            offs2[l + 1] = order.size();
        }
        relayout(order, offs2, code.data(), id);
        return {};
    }

    std::expected<size_t, error> compact_list(uint32_t c, const uint32_t* deleted, size_t n_del) {
        if (!trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.compact_inverted_list");
        if (c >= nlist()) return fail(error_code::out_of_range, "Cluster ID out of range", "ivf_pq.compact_inverted_list");
        std::lock_guard<std::mutex> lock(mu);
        const uint64_t e0 = h_offs[c], n = h_offs[c + 1] - e0;
        if (n == 0 || n_del == 0 || !deleted) return (size_t)0;
        std::vector<uint64_t> lid(n);
        d2h(lid.data(), d_ids.data() + e0, n, st);
        sync(st);
        std::vector<uint32_t> del(deleted, deleted + n_del);
        std::sort(del.begin(), del.end());
        std::vector<uint32_t> order;
        order.reserve(n_vectors);
        std::vector<uint64_t> offs2(nlist() + 1, 0);
        size_t removed = 0;
        for (uint32_t l = 0; l < nlist(); ++l) {
            for (uint64_t i = h_offs[l]; i < h_offs[l + 1]; ++i) {
                if (l == c && std::binary_search(del.begin(), del.end(), static_cast<uint32_t>(lid[i - e0]))) {
                    ++removed;
                    continue;
                }
                order.push_back((uint32_t)i);
            }
            offs2[l + 1] = order.size();
        }
        if (removed) relayout(order, offs2, nullptr, 0);
        return removed;
    }

    std::expected<std::pair<size_t, uint32_t>, error> centroid_rank(const float* query, uint64_t id) const {
        if (!env_flag("VESPER_IVFPQ_DEBUG"))
            return fail(error_code::precondition_failed, "debug_explain_centroid_rank requires VESPER_IVFPQ_DEBUG=1");
        if (!trained || n_vectors == 0) return fail(error_code::precondition_failed, "Index must be trained and non-empty");
        std::lock_guard<std::mutex> lock(mu);
        uint32_t e = 0, l = 0;
        if (!find_entry(id, e, l)) return fail(error_code::not_found, "Target ID not found in index");
        DeviceBuffer<float> q(dim), d(nlist());
        h2d(q.data(), query, dim, st);
        vgpu::launch_l2_dist(q.data(), 1, d_cent.data(), (int)nlist(), (int)dim, d.data(), (long long)nlist(), st);
        w_count.reserve(1);
        vgpu::check(cudaMemsetAsync(w_count.data(), 0, sizeof(unsigned long long), st), "memset");
        vgpu::launch_count_less(d.data(), (long long)nlist(), (long long)l, w_count.data(), st);
        unsigned long long cnt = 0;
        d2h(&cnt, w_count.data(), 1, st);
        sync(st);
        return std::make_pair((size_t)cnt + 1, l);
    }

    std::expected<std::pair<size_t, float>, error> adc_rank(const float* query, uint64_t id) const {
        if (!env_flag("VESPER_IVFPQ_DEBUG"))
            return fail(error_code::precondition_failed, "debug_explain_adc_rank requires VESPER_IVFPQ_DEBUG=1");
        if (!trained || n_vectors == 0) return fail(error_code::precondition_failed, "Index must be trained and non-empty");
        std::lock_guard<std::mutex> lock(mu);
        uint32_t e = 0, l = 0;
        if (!find_entry(id, e, l)) return fail(error_code::not_found, "Target ID not found in index");
        // every list's (rotated) query residual in the search's exact order, then every
        // entry's exact ADC distance
        DeviceBuffer<float> q(dim), rres((size_t)nlist() * dim), adc(n_vectors);
        DeviceBuffer<uint32_t> qidx(nlist()), lidx(nlist());
        h2d(q.data(), query, dim, st);
        vgpu::check(cudaMemsetAsync(qidx.data(), 0, nlist() * sizeof(uint32_t), st), "memset");
        vgpu::launch_iota(lidx.data(), nlist(), st);
        vgpu::launch_residual_rotate(q.data(), qidx.data(), d_cent.data(), lidx.data(), nlist(), (int)dim,
                                     has_rot ? d_rot.data() : nullptr, rres.data(), st);
        vgpu::launch_adc_all(rres.data(), (int)dim, (int)nlist(), d_cb.data(), (int)m(), (int)ksub, (int)dsub,
                             d_offs.data(), d_codes.data(), adc.data(), st);
        w_count.reserve(1);
        vgpu::check(cudaMemsetAsync(w_count.data(), 0, sizeof(unsigned long long), st), "memset");
        vgpu::launch_count_less(adc.data(), (long long)n_vectors, (long long)e, w_count.data(), st);
        unsigned long long cnt = 0;
        float dist = 0.0f;
        d2h(&cnt, w_count.data(), 1, st);
        d2h(&dist, adc.data() + e, 1, st);
        sync(st);
        return std::make_pair((size_t)cnt + 1, dist);
    }

    std::expected<void, error> search_adc(const float* queries, size_t nq, const IvfPqSearchParams& sp,
                                          uint64_t* out_ids, float* out_d, uint32_t* out_n,
                                          bool on_device, const uint32_t* ext_probe = nullptr,
                                          const float* ext_probe_d = nullptr) const {
        if (!trained) return fail(error_code::precondition_failed, "Index must be trained before searching");
        if (sp.k == 0) return fail(error_code::invalid_argument, "k must be > 0");
        if (sp.k > (uint32_t)vgpu::kMaxK) return fail(error_code::unsupported, "k above 1024 is not supported by the GPU path");
        if (nq == 0) return {};
        uint32_t np = std::min(sp.nprobe, nlist());
        if (env_flag("VESPER_IVFPQ_PROBE_ALL")) np = nlist();
        if (np == 0) {  // nothing probed: every result is padding
            if (on_device) {
                vgpu::check(cudaMemsetAsync(out_ids, 0, nq * sp.k * sizeof(uint64_t), st), "memset");
                vgpu::check(cudaMemsetAsync(out_d, 0, nq * sp.k * sizeof(float), st), "memset");
                if (out_n) vgpu::check(cudaMemsetAsync(out_n, 0, nq * sizeof(uint32_t), st), "memset");
                sync(st);
            } else {
                std::fill(out_ids, out_ids + nq * sp.k, 0);
                std::fill(out_d, out_d + nq * sp.k, 0.0f);
                if (out_n) std::fill(out_n, out_n + nq, 0u);
            }
            return {};
        }
        if (np > (uint32_t)vgpu::kMaxK) return fail(error_code::unsupported, "nprobe above 1024 is not supported by the GPU path");
        std::lock_guard<std::mutex> lock(mu);
        const uint32_t k = sp.k;
        const bool exact = sp.mode == SearchMode::Exact;
        // Chunk queries so the coarse distance tile (when one is written), the tables and
        // the exact-path buffers stay bounded.  Device queries keep their alignment per
        // chunk (rows of dim floats, dim % 4 == 0 on the tensor-core path); host queries
        // are copied into w_q.
        const bool filt = !ext_probe && filter_probe(on_device ? queries : d_cent.data());  // w_q is cudaMalloc'd
        // No distance matrix when the probe lists are given or come from the filter path.
        const bool no_dist = filt || ext_probe;
        size_t qc = no_dist ? std::max<size_t>(1, kSearchTableBudget / (sizeof(float) * (size_t)m() * ksub))
                            : std::max<size_t>(1, kSearchDistBudget / (sizeof(float) * (size_t)nlist()));
        if (exact && has_rot) qc = std::min(qc, std::max<size_t>(1, kDistBudget / (sizeof(float) * np * dim)));
        qc = std::min(qc, nq);
        if (!filt && !ext_probe) w_D.reserve(qc * nlist());
        w_probe.reserve(qc * np);
        w_probe_d.reserve(qc * np);
        if (!on_device) {
            w_q.reserve(qc * dim);
            w_out_ids.reserve(qc * k);
            w_out_d.reserve(qc * k);
            w_out_n.reserve(qc);
        }
        if (exact) {
            w_cand_d.reserve(qc * np * k);
            w_cand_pos.reserve(qc * np * k);
            w_cand_n.reserve(qc * np);
            if (has_rot) {
                w_rres.reserve(qc * np * dim);
                w_pair_q.reserve(qc * np);
            }
        } else {
            w_rq.reserve(qc * dim);
            w_T.reserve(qc * (size_t)m() * ksub);
            w_pbase.reserve(qc * np);
        }
        // FAST search rotates the queries with one tensor-core GEMM (3xTF32); EXACT
        // search keeps the reference's sequential rotation.
        const bool rot_gemm = !exact && has_rot && use_rotation_gemm();
        if (rot_gemm) {
            w_rq3.reserve(qc * dim * 3);
            reset_err();
        }
        const bool list_scan = !exact && use_list_scan(nq, np);
        const bool split_scan = !exact && !list_scan && has_blocks && use_split_scan();
        if (list_scan) {
            int cap = kListScanCap;
            if (const char* v = std::getenv("VGPU_LIST_CAP")) cap = std::clamp(std::atoi(v), 256, 4096);
            tlw.reserve((long long)qc, (int)np, (int)nlist(), (int)dim, (int)k, cap, n_vectors);
            vgpu::check(cudaMemsetAsync(tlw.stats.data(), 0, 2 * sizeof(unsigned long long), st), "memset");
            reset_err();
        }
        SearchTimings tm;
        const unsigned long long launches0 = vgpu::thread_launches();
        w_scanned.reserve(1);
        vgpu::check(cudaMemsetAsync(w_scanned.data(), 0, sizeof(unsigned long long), st), "memset");
        for (size_t q0 = 0; q0 < nq; q0 += qc) {
            const size_t nc = std::min(qc, nq - q0);
            const float* dq;
            uint64_t* oid;
            float* od;
            uint32_t* on;
            if (on_device) {
                dq = queries + q0 * dim;
                oid = out_ids + q0 * k;
                od = out_d + q0 * k;
                on = out_n ? out_n + q0 : nullptr;
            } else {
                h2d(w_q.data(), queries + q0 * dim, nc * dim, st);
                dq = w_q.data();
                oid = w_out_ids.data();
                od = w_out_d.data();
                on = w_out_n.data();
            }
            const bool tc = !ext_probe && vgpu::use_tensor_cores(dq, d_cent.data(), (int)dim, nlist());
            const uint32_t* probe = ext_probe ? ext_probe + q0 * np : w_probe.data();
            const float* probe_d = ext_probe ? ext_probe_d + q0 * np : w_probe_d.data();
            cudaEventRecord(ev[0], st);
            if (ext_probe) {
                // probe lists given
            } else if (filt) {
                vgpu::launch_exact_nearest(dq, (long long)nc, d_cent.data(), nlist(), (int)dim, (int)np, nullptr,
                                           w_probe.data(), w_probe_d.data(), w_flat, st);
            } else if (tc) {
                w_xn.reserve(qc);
                reset_err();
                vgpu::launch_row_norms(dq, (long long)nc, (int)dim, w_xn.data(), st);
                vgpu::launch_tc_screen(dq, (long long)nc, d_cent.data(), (int)nlist(), (int)dim, w_xn.data(),
                                       d_cn.data(), w_D.data(), (long long)nlist(), d_err.data(), st);
            } else {
                vgpu::launch_l2_dist(dq, (long long)nc, d_cent.data(), (int)nlist(), (int)dim, w_D.data(),
                                     (long long)nlist(), st);
            }
            cudaEventRecord(ev[1], st);
            if (ext_probe || filt) {
                // probe lists given, or selected by the filter path
            } else if (tc) {
                vgpu::launch_screen_select(w_D.data(), (long long)nc, (long long)nlist(), (int)nlist(), dq, (int)dim,
                                           d_cent.data(), w_xn.data(), d_cn.data(), (int)np, nullptr, w_probe.data(),
                                           w_probe_d.data(), d_err.data(), st);
            } else {
                vgpu::launch_row_topk(w_D.data(), (long long)nc, (int)nlist(), (long long)nlist(), (int)np,
                                      w_probe.data(), w_probe_d.data(), st);
            }
            cudaEventRecord(ev[2], st);
            vgpu::launch_probe_sizes(probe, (long long)(nc * np), d_offs.data(), w_scanned.data(), st);
            if (exact) {
                const float* rres = nullptr;
                if (has_rot) {
                    std::vector<uint32_t> pq(nc * np);
                    for (size_t i = 0; i < nc * np; ++i) pq[i] = (uint32_t)(i / np);
                    h2d(w_pair_q.data(), pq.data(), pq.size(), st);
                    vgpu::launch_residual_rotate(dq, w_pair_q.data(), d_cent.data(), probe,
                                                 (long long)(nc * np), (int)dim, d_rot.data(), w_rres.data(), st);
                    rres = w_rres.data();
                }
                cudaEventRecord(ev[3], st);
                vgpu::launch_scan_exact(dq, (long long)nc, (int)dim, d_cent.data(), rres, probe, (int)np,
                                        d_cb.data(), (int)m(), (int)ksub, (int)dsub, d_offs.data(), d_codes.data(),
                                        (int)k, w_cand_d.data(), w_cand_pos.data(), w_cand_n.data(), st);
                cudaEventRecord(ev[4], st);
                vgpu::launch_merge(w_cand_d.data(), w_cand_pos.data(), w_cand_n.data(), (long long)nc, (int)np,
                                   (int)k, probe, d_offs.data(), d_ids.data(), oid, od, on, st);
            } else {
                const float* rq = dq;
                if (rot_gemm) {
                    vgpu::launch_rotate_3xtf32(dq, (long long)nc, (int)dim, d_rot3.data(), w_rq3.data(), w_rq.data(),
                                               d_err.data(), st);
                    rq = w_rq.data();
                } else if (has_rot) {
                    vgpu::launch_rotate_fast(dq, (long long)nc, (int)dim, d_rot.data(), w_rq.data(), st);
                    rq = w_rq.data();
                }
                if (has_blocks) {
                    vgpu::launch_lut_blocked(rq, (long long)nc, (int)dim, d_cb.data(), (int)m(), (int)dsub,
                                             w_T.data(), st);
                    vgpu::launch_probe_base(rq, (long long)nc, (int)dim, probe, probe_d,
                                            has_rot ? d_rc.data() : nullptr, (int)np, w_pbase.data(), st);
                    cudaEventRecord(ev[3], st);
                    if (list_scan) {
                        vgpu::TlScanArgs a{};
                        a.T = w_T.data(); a.rq = rq; a.pbase = w_pbase.data(); a.probe = probe;
                        a.nq = (long long)nc; a.nprobe = (int)np; a.nlist = (int)nlist(); a.dim = (int)dim;
                        a.m = (int)m(); a.k = (int)k; a.offs = d_offs.data(); a.codes = d_codes.data();
                        a.vterm = d_vterm.data(); a.xnorm = d_xnorm.data(); a.cbb = d_cbb.data(); a.cb = d_cb.data();
                        a.blk_off = d_blk_off.data(); a.bcodes = d_bcodes.data(); a.bvterm = d_bvterm.data();
                        a.ids = d_ids.data(); a.out_ids = oid; a.out_d = od; a.out_n = on; a.err = d_err.data();
                        a.tau_fn = tau_fn; a.tau_user = tau_user;
                        a.tau_shard = tau_shard; a.tau_shards = tau_shards;
                        vgpu::launch_tc_list_scan(a, tlw, st);
                    } else if (split_scan) {
                        vgpu::launch_scan_blocked_split(w_T.data(), (long long)nc, w_pbase.data(), probe,
                                                        (int)np, (int)np, (int)m(), d_offs.data(), d_blk_off.data(),
                                                        d_bcodes.data(), d_bvterm.data(), d_ids.data(), (int)k, oid,
                                                        od, on, nullptr, 0, tlw.split, st);
                    } else {
                        vgpu::launch_scan_blocked(w_T.data(), (long long)nc, w_pbase.data(), probe, (int)np,
                                                  (int)np, (int)m(), d_offs.data(), d_blk_off.data(),
                                                  d_bcodes.data(), d_bvterm.data(), d_ids.data(), (int)k, oid, od,
                                                  on, nullptr, 0, st);
                    }
                } else {
                    vgpu::launch_lut_fast(rq, (long long)nc, (int)dim, d_cb.data(), (int)m(), (int)ksub, (int)dsub,
                                          w_T.data(), st);
                    cudaEventRecord(ev[3], st);
                    vgpu::launch_scan_fast2(w_T.data(), rq, (long long)nc, (int)dim, probe, probe_d,
                                            has_rot ? d_rc.data() : nullptr, (int)np, (int)m(), (int)ksub,
                                            d_offs.data(), d_codes.data(), d_vterm.data(), d_ids.data(), (int)k,
                                            oid, od, on, st);
                }
                cudaEventRecord(ev[4], st);
            }
            if (tau_fn && !list_scan) {
                // this shard has no bound to offer, but the shards' calls must pair up
                w_tau_inf.reserve(qc);
                vgpu::launch_fill(w_tau_inf.data(), (long long)nc, __builtin_inff(), st);
                if (tau_fn(w_tau_inf.data(), nc, st, tau_user) != 0)
                    throw vgpu::CudaError("search: the threshold exchange failed");
            }
            cudaEventRecord(ev[5], st);
            tm.scan_variant = exact ? 1u : list_scan ? 4u : (has_blocks ? 3u : 2u);
            tm.coarse_variant = filt ? 3u : tc ? 2u : 1u;
            if (!on_device) {
                d2h(out_ids + q0 * k, oid, nc * k, st);
                d2h(out_d + q0 * k, od, nc * k, st);
                if (out_n) d2h(out_n + q0, on, nc, st);
            }
            sync(st);
            if ((tc && !filt) || list_scan || rot_gemm) check_err();
            float a = 0;
            cudaEventElapsedTime(&a, ev[0], ev[1]); tm.coarse_ms += a;
            cudaEventElapsedTime(&a, ev[1], ev[2]); tm.select_ms += a;
            cudaEventElapsedTime(&a, ev[2], ev[3]); tm.rotate_ms += a;
            cudaEventElapsedTime(&a, ev[3], ev[4]); tm.scan_ms += a;
            cudaEventElapsedTime(&a, ev[4], ev[5]); tm.merge_ms += a;
            cudaEventElapsedTime(&a, ev[0], ev[5]); tm.total_ms += a;
            if (list_scan) {
                cudaEventElapsedTime(&a, tlw.ev[0], tlw.ev[1]); tm.list_threshold_ms += a;
                cudaEventElapsedTime(&a, tlw.ev[1], tlw.ev[2]); tm.list_prep_ms += a;
                cudaEventElapsedTime(&a, tlw.ev[2], tlw.ev[3]); tm.list_kernel_ms += a;
                cudaEventElapsedTime(&a, tlw.ev[3], tlw.ev[4]); tm.list_refine_ms += a;
                cudaEventElapsedTime(&a, tlw.ev[4], tlw.ev[5]); tm.list_fallback_ms += a;
            }
        }
        if (list_scan) {
            unsigned long long s2[2] = {0, 0};
            d2h(s2, tlw.stats.data(), 2, st);
            sync(st);
            tm.list_candidates = s2[0];
            tm.list_fallback_queries = (uint32_t)s2[1];
        }
        unsigned long long scanned = 0;
        d2h(&scanned, w_scanned.data(), 1, st);
        sync(st);
        tm.scanned_entries = scanned;
        tm.kernel_launches = (uint32_t)(vgpu::thread_launches() - launches0);
        timings = tm;
        return {};
    }

    // ------------------------------------------------------------------ coarse stage only
    // The probe lists of search_adc's coarse stage (tensor-core screen + exact refine,
    // or CUDA-core distances): d_probe / d_probe_d [nq x min(nprobe, nlist)].
    std::expected<void, error> probe_only(const float* dq_all, size_t nq, uint32_t nprobe, uint32_t* d_probe,
                                          float* d_probe_d) const {
        if (!trained) return fail(error_code::precondition_failed, "Index must be trained before searching");
        const uint32_t np = std::min(nprobe, nlist());
        if (nq == 0 || np == 0) return {};
        if (np > (uint32_t)vgpu::kMaxK) return fail(error_code::unsupported, "nprobe above 1024 is not supported by the GPU path");
        std::lock_guard<std::mutex> lock(mu);
        if (filter_probe(dq_all)) {
            vgpu::launch_exact_nearest(dq_all, (long long)nq, d_cent.data(), nlist(), (int)dim, (int)np, nullptr,
                                       d_probe, d_probe_d, w_flat, st);
            sync(st);
            return {};
        }
        const size_t qc = std::min(nq, std::max<size_t>(1, kSearchDistBudget / (sizeof(float) * (size_t)nlist())));
        w_D.reserve(qc * nlist());
        for (size_t q0 = 0; q0 < nq; q0 += qc) {
            const size_t nc = std::min(qc, nq - q0);
            const float* dq = dq_all + q0 * dim;
            uint32_t* probe = d_probe + q0 * np;
            float* probe_d = d_probe_d + q0 * np;
            if (vgpu::use_tensor_cores(dq, d_cent.data(), (int)dim, nlist())) {
                w_xn.reserve(qc);
                reset_err();
                vgpu::launch_row_norms(dq, (long long)nc, (int)dim, w_xn.data(), st);
                vgpu::launch_tc_screen(dq, (long long)nc, d_cent.data(), (int)nlist(), (int)dim, w_xn.data(),
                                       d_cn.data(), w_D.data(), (long long)nlist(), d_err.data(), st);
                vgpu::launch_screen_select(w_D.data(), (long long)nc, (long long)nlist(), (int)nlist(), dq, (int)dim,
                                           d_cent.data(), w_xn.data(), d_cn.data(), (int)np, nullptr, probe, probe_d,
                                           d_err.data(), st);
                sync(st);
                check_err();
            } else {
                vgpu::launch_l2_dist(dq, (long long)nc, d_cent.data(), (int)nlist(), (int)dim, w_D.data(),
                                     (long long)nlist(), st);
                vgpu::launch_row_topk(w_D.data(), (long long)nc, (int)nlist(), (long long)nlist(), (int)np, probe,
                                      probe_d, st);
            }
        }
        sync(st);
        return {};
    }

    // ------------------------------------------------------------------ search without allocation
    // The FAST search of search_flat with every temporary buffer carved out of the
    // fixed device array of noalloc_search.cu instead of cudaMalloc'd workspace: no
    // allocation of any kind.  Queries are processed in chunks sized to the array.
    std::expected<void, error> search_noalloc(const float* dq_all, size_t nq, const IvfPqSearchParams& sp,
                                              uint64_t* out_ids, float* out_d, uint32_t* out_n) const {
        if (!trained) return fail(error_code::precondition_failed, "Index must be trained before searching");
        if (sp.mode != SearchMode::Fast)
            return fail(error_code::unsupported, "the allocation-free search supports the FAST mode only");
        if (sp.k == 0) return fail(error_code::invalid_argument, "k must be > 0");
        if (sp.k > (uint32_t)vgpu::kMaxK) return fail(error_code::unsupported, "k above 1024 is not supported by the GPU path");
        if (nq == 0) return {};
        const uint32_t np = std::min(sp.nprobe, nlist());
        if (np == 0 || np > (uint32_t)vgpu::kMaxK)
            return fail(error_code::unsupported, "nprobe must be in [1, 1024] for the allocation-free search");
        auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
        const size_t per_q = (size_t)nlist() * 4 + (size_t)np * 8 + (has_rot ? dim * 4 : 0) + (size_t)m() * ksub * 4;
        const size_t slack = 4 * 256;
        if (per_q + slack > vgpu::kNoAllocScratchBytes)
            return fail(error_code::out_of_range,
                        "allocation-free search: one query needs " + std::to_string(per_q) +
                        " bytes of scratch, more than the fixed " + std::to_string(vgpu::kNoAllocScratchBytes) +
                        "-byte device buffer (nlist or m * 2^nbits too large)");
        // Every launch limit is checked before anything is queued on the shared array, so
        // a rejected call never leaves scratch work in flight behind the released lock.
        if (!vgpu::lut_fast_fits((int)ksub, (int)dsub) || !vgpu::scan_fast2_fits((int)m(), (int)ksub, (int)sp.k, (int)np))
            return fail(error_code::out_of_range,
                        "allocation-free search: the per-query lookup table (m * 2^nbits floats) or the top-k "
                        "merge buffer exceeds the shared memory of its kernels");
        std::lock_guard<std::mutex> call_lock(vgpu::noalloc_call_mutex());
        std::lock_guard<std::mutex> lock(mu);
        unsigned char* base = static_cast<unsigned char*>(vgpu::noalloc_scratch_device_address(dev));
        const size_t qc = std::min(nq, (vgpu::kNoAllocScratchBytes - slack) / per_q);
        unsigned char* p = base;
        float* D = reinterpret_cast<float*>(p); p += al(qc * nlist() * 4);
        uint32_t* probe = reinterpret_cast<uint32_t*>(p); p += al(qc * np * 4);
        float* probe_d = reinterpret_cast<float*>(p); p += al(qc * np * 4);
        float* rq = has_rot ? reinterpret_cast<float*>(p) : nullptr; p += has_rot ? al(qc * dim * 4) : 0;
        float* T = reinterpret_cast<float*>(p);
        const uint32_t k = sp.k;
        try {
        for (size_t q0 = 0; q0 < nq; q0 += qc) {
            const size_t nc = std::min(qc, nq - q0);
            const float* dq = dq_all + q0 * dim;
            vgpu::launch_l2_dist(dq, (long long)nc, d_cent.data(), (int)nlist(), (int)dim, D, (long long)nlist(), st);
            vgpu::launch_row_topk(D, (long long)nc, (int)nlist(), (long long)nlist(), (int)np, probe, probe_d, st);
            const float* qrot = dq;
            if (has_rot) {
                vgpu::launch_rotate_fast(dq, (long long)nc, (int)dim, d_rot.data(), rq, st);
                qrot = rq;
            }
            vgpu::launch_lut_fast(qrot, (long long)nc, (int)dim, d_cb.data(), (int)m(), (int)ksub, (int)dsub, T, st);
            vgpu::launch_scan_fast2(T, qrot, (long long)nc, (int)dim, probe, probe_d, has_rot ? d_rc.data() : nullptr,
                                    (int)np, (int)m(), (int)ksub, d_offs.data(), d_codes.data(), d_vterm.data(),
                                    d_ids.data(), (int)k, out_ids + q0 * k, out_d + q0 * k,
                                    out_n ? out_n + q0 : nullptr, st);
        }
        } catch (...) {
            // kernels already queued still use the array: drain them before the lock goes
            cudaStreamSynchronize(st);
            throw;
        }
        sync(st);
        return {};
    }
};

// ====================================================================== public API
IvfPqIndex::IvfPqIndex() : impl_(std::make_unique<Impl>()) {}
IvfPqIndex::~IvfPqIndex() = default;
IvfPqIndex::IvfPqIndex(IvfPqIndex&&) noexcept = default;
IvfPqIndex& IvfPqIndex::operator=(IvfPqIndex&&) noexcept = default;

auto IvfPqIndex::train(const float* data, std::size_t dim, std::size_t n, const IvfPqTrainParams& params)
    -> std::expected<IvfPqTrainStats, core::error> {
    return train_device(data, dim, n, params, false);
}

auto IvfPqIndex::train_device(const float* data, std::size_t dim, std::size_t n,
                              const IvfPqTrainParams& params, bool on_device)
    -> std::expected<IvfPqTrainStats, core::error> {
    DeviceGuard g(impl_->dev);
    try {
        std::lock_guard<std::mutex> lock(impl_->mu);
        return impl_->train(data, dim, n, params, on_device);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    } catch (const std::bad_alloc&) {
        return fail(error_code::out_of_memory, "bad_alloc in train");
    }
}

auto IvfPqIndex::add(const std::uint64_t* ids, const float* data, std::size_t n)
    -> std::expected<void, core::error> {
    return add_device(ids, data, n, false);
}

auto IvfPqIndex::add_device(const std::uint64_t* ids, const float* data, std::size_t n, bool on_device)
    -> std::expected<void, core::error> {
    DeviceGuard g(impl_->dev);
    try {
        std::lock_guard<std::mutex> lock(impl_->mu);
        return impl_->add(ids, data, n, on_device);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    } catch (const std::bad_alloc&) {
        return fail(error_code::out_of_memory, "bad_alloc in add() residuals/rotation");
    }
}

auto IvfPqIndex::search_batch_flat(const float* queries, std::size_t n_queries,
                                   const IvfPqSearchParams& params, std::uint64_t* out_ids,
                                   float* out_dist, std::uint32_t* out_counts, bool on_device) const
    -> std::expected<void, core::error> {
    DeviceGuard g(impl_->dev);
    try {
        return impl_->search_flat(queries, n_queries, params, out_ids, out_dist, out_counts, on_device);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
}

void IvfPqIndex::set_threshold_exchange(ThresholdExchangeFn fn, void* user, std::uint32_t shard,
                                        std::uint32_t shards) {
    if (shards == 0 || shard >= shards) throw vgpu::CudaError("set_threshold_exchange: shard must be below shards");
    std::lock_guard<std::mutex> lk(impl_->mu);
    impl_->tau_fn = fn;
    impl_->tau_user = fn ? user : nullptr;
    impl_->tau_shard = fn ? shard : 0;
    impl_->tau_shards = fn ? shards : 1;
}

auto IvfPqIndex::probe_device(const float* d_queries, std::size_t n_queries, std::uint32_t nprobe,
                              std::uint32_t* d_probe, float* d_probe_d) const -> std::expected<void, core::error> {
    DeviceGuard g(impl_->dev);
    try {
        return impl_->probe_only(d_queries, n_queries, nprobe, d_probe, d_probe_d);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
}

auto IvfPqIndex::search_batch_device_probed(const float* d_queries, std::size_t n_queries,
                                            const IvfPqSearchParams& params, const std::uint32_t* d_probe,
                                            const float* d_probe_d, std::uint64_t* d_out_ids, float* d_out_dist,
                                            std::uint32_t* d_out_counts) const -> std::expected<void, core::error> {
    DeviceGuard g(impl_->dev);
    if (params.use_exact_rerank)
        return fail(error_code::unsupported, "the search with given probe lists does not support the exact rerank");
    try {
        return impl_->search_adc(d_queries, n_queries, params, d_out_ids, d_out_dist, d_out_counts, true, d_probe,
                                 d_probe_d);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
}

auto IvfPqIndex::search_batch_device_noalloc(const float* d_queries, std::size_t n_queries,
                                              const IvfPqSearchParams& params, std::uint64_t* d_out_ids,
                                              float* d_out_dist, std::uint32_t* d_out_counts) const
    -> std::expected<void, core::error> {
    DeviceGuard g(impl_->dev);
    try {
        return impl_->search_noalloc(d_queries, n_queries, params, d_out_ids, d_out_dist, d_out_counts);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
}

auto IvfPqIndex::search_batch(const float* queries, std::size_t n_queries, const IvfPqSearchParams& params) const
    -> std::expected<std::vector<std::vector<std::pair<std::uint64_t, float>>>, core::error> {
    const size_t k = params.k;
    std::vector<uint64_t> ids(n_queries * k);
    std::vector<float> d(n_queries * k);
    std::vector<uint32_t> cnt(n_queries);
    auto r = search_batch_flat(queries, n_queries, params, ids.data(), d.data(), cnt.data(), false);
    if (!r) return std::unexpected(r.error());
    std::vector<std::vector<std::pair<std::uint64_t, float>>> out(n_queries);
    for (size_t q = 0; q < n_queries; ++q)
        for (uint32_t i = 0; i < cnt[q]; ++i) out[q].emplace_back(ids[q * k + i], d[q * k + i]);
    return out;
}

auto IvfPqIndex::search(const float* query, const IvfPqSearchParams& params) const
    -> std::expected<std::vector<std::pair<std::uint64_t, float>>, core::error> {
    auto r = search_batch(query, 1, params);
    if (!r) return std::unexpected(r.error());
    return std::move((*r)[0]);
}

void IvfPqIndex::set_metadata_json(std::string_view json) { impl_->metadata_json.assign(json); }
auto IvfPqIndex::get_metadata_json() const -> std::string { return impl_->metadata_json; }

auto IvfPqIndex::get_stats() const noexcept -> Stats {
    Stats s;
    const auto& I = *impl_;
    s.n_vectors = I.n_vectors;
    s.n_lists = I.params.nlist;
    s.m = I.params.m;
    s.code_size = I.params.m;
    s.memory_bytes = sizeof(Impl) + I.d_cent.bytes() + I.d_cb.bytes() + I.d_rot.bytes() + I.d_rotT.bytes() + I.d_rot3.bytes() +
                     I.d_rc.bytes() + I.d_offs.bytes() + I.d_ids.bytes() + I.d_codes.bytes() + I.d_vterm.bytes() +
                     I.d_blk_off.bytes() + I.d_bcodes.bytes() + I.d_bvterm.bytes() + I.d_cbb.bytes() +
                     I.d_xnorm.bytes();
    s.avg_list_size = I.n_vectors > 0 && I.params.nlist ? (float)I.n_vectors / (float)I.params.nlist : 0.0f;
    s.timings_enabled = I.params.verbose || I.params.timings_enabled || env_flag("VESPER_TIMING");
    if (s.timings_enabled) { s.t_assign_ms = I.t_assign_ms; s.t_encode_ms = I.t_encode_ms; s.t_lists_ms = I.t_lists_ms; }
    return s;
}

auto IvfPqIndex::is_trained() const noexcept -> bool { return impl_->trained; }
auto IvfPqIndex::dimension() const noexcept -> std::size_t { return impl_->dim; }
auto IvfPqIndex::last_search_timings() const -> SearchTimings { return impl_->timings; }
auto IvfPqIndex::params() const -> IvfPqTrainParams { return impl_->params; }

#define VGPU_GUARDED(expr)                                      \
    DeviceGuard g(impl_->dev);                                  \
    try {                                                       \
        return expr;                                            \
    } catch (const vgpu::CudaError& e) {                        \
        return fail(error_code::internal, e.what(), "ivf_pq.cuda"); \
    }

auto IvfPqIndex::reconstruct_cluster(std::uint32_t cluster_id, std::vector<std::uint64_t>& ids,
                                     std::vector<float>& vectors) const -> std::expected<void, core::error> {
    VGPU_GUARDED(impl_->reconstruct_cluster(cluster_id, ids, vectors))
}
auto IvfPqIndex::reconstruct(std::uint64_t id) const -> std::expected<std::vector<float>, core::error> {
    VGPU_GUARDED(impl_->reconstruct(id))
}
auto IvfPqIndex::get_num_clusters() const -> std::expected<std::uint32_t, core::error> {
    if (!impl_->trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.get_num_clusters");
    return impl_->nlist();
}
auto IvfPqIndex::get_dimension() const -> std::expected<std::size_t, core::error> {
    if (!impl_->trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.get_dimension");
    return impl_->dim;
}
auto IvfPqIndex::get_cluster_assignment(std::uint64_t id) const -> std::expected<std::uint32_t, core::error> {
    VGPU_GUARDED(impl_->cluster_assignment(id))
}
auto IvfPqIndex::get_cluster_centroid(std::uint32_t cluster_id) const
    -> std::expected<std::vector<float>, core::error> {
    if (!impl_->trained) return fail(error_code::not_initialized, "Index not trained", "ivf_pq.get_cluster_centroid");
    if (cluster_id >= impl_->nlist())
        return fail(error_code::out_of_range, "Cluster ID out of range", "ivf_pq.get_cluster_centroid");
    const float* c = impl_->h_cent.data() + (size_t)cluster_id * impl_->dim;
    return std::vector<float>(c, c + impl_->dim);
}
auto IvfPqIndex::update_cluster_centroid(std::uint32_t cluster_id, const float* centroid)
    -> std::expected<void, core::error> {
    VGPU_GUARDED(impl_->update_centroid(cluster_id, centroid))
}
auto IvfPqIndex::reassign_vector(std::uint64_t id, std::uint32_t new_cluster) -> std::expected<void, core::error> {
    VGPU_GUARDED(impl_->reassign(id, new_cluster))
}
auto IvfPqIndex::compact_inverted_list(std::uint32_t cluster_id, const std::uint32_t* deleted_ids,
                                       std::size_t n_deleted) -> std::expected<std::size_t, core::error> {
    VGPU_GUARDED(impl_->compact_list(cluster_id, deleted_ids, n_deleted))
}
auto IvfPqIndex::debug_explain_centroid_rank(const float* query, std::uint64_t target_id) const
    -> std::expected<std::pair<std::size_t, std::uint32_t>, core::error> {
    VGPU_GUARDED(impl_->centroid_rank(query, target_id))
}
auto IvfPqIndex::debug_explain_adc_rank(const float* query, std::uint64_t target_id) const
    -> std::expected<std::pair<std::size_t, float>, core::error> {
    VGPU_GUARDED(impl_->adc_rank(query, target_id))
}
#undef VGPU_GUARDED

auto IvfPqIndex::clear() -> void {
    DeviceGuard g(impl_->dev);
    std::lock_guard<std::mutex> lock(impl_->mu);
    if (impl_->trained) { impl_->reset_lists(); sync(impl_->st); }
}

auto IvfPqIndex::reset() -> void {
    DeviceGuard g(impl_->dev);
    impl_ = std::make_unique<Impl>();
}

auto IvfPqIndex::centroids() const -> std::vector<float> { return impl_->h_cent; }
auto IvfPqIndex::codebooks() const -> std::vector<float> { return impl_->h_cb; }
auto IvfPqIndex::rotation() const -> std::vector<float> { return impl_->h_rot; }
auto IvfPqIndex::list_offsets() const -> std::vector<std::uint64_t> { return impl_->h_offs; }

auto IvfPqIndex::list_ids() const -> std::vector<std::uint64_t> {
    DeviceGuard g(impl_->dev);
    std::vector<uint64_t> v(impl_->n_vectors);
    d2h(v.data(), impl_->d_ids.data(), v.size(), impl_->st);
    sync(impl_->st);
    return v;
}

auto IvfPqIndex::list_codes() const -> std::vector<std::uint8_t> {
    DeviceGuard g(impl_->dev);
    std::vector<uint8_t> v(impl_->n_vectors * impl_->params.m);
    d2h(v.data(), impl_->d_codes.data(), v.size(), impl_->st);
    sync(impl_->st);
    return v;
}

auto IvfPqIndex::set_model(std::size_t dim, std::uint32_t nlist, std::uint32_t m, std::uint32_t nbits,
                           const float* cent, const float* cb, const float* rot)
    -> std::expected<void, core::error> {
    if (dim == 0 || nlist == 0 || m == 0 || dim % m != 0 || nbits == 0 || nbits > 8)
        return fail(error_code::invalid_argument, "invalid model shape");
    DeviceGuard g(impl_->dev);
    try {
        auto& I = *impl_;
        std::lock_guard<std::mutex> lock(I.mu);
        I.params = IvfPqTrainParams{};
        I.params.nlist = nlist;
        I.params.m = m;
        I.params.nbits = nbits;
        I.params.use_opq = rot != nullptr;
        I.dim = dim;
        I.dsub = dim / m;
        I.ksub = 1u << nbits;
        I.h_cent.assign(cent, cent + (size_t)nlist * dim);
        I.h_cb.assign(cb, cb + (size_t)m * I.ksub * I.dsub);
        I.has_rot = rot != nullptr;
        if (rot) I.h_rot.assign(rot, rot + dim * dim); else I.h_rot.clear();
        I.upload_model();
        I.reset_lists();
        sync(I.st);
        I.trained = true;
        return {};
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
}

// ---------------------------------------------------------------------- persistence
namespace {
struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void update(const void* p, size_t n) {
        const auto* b = static_cast<const uint8_t*>(p);
        for (size_t i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ull; }
    }
};


// IvfPqIndex::save v1.0 layout (src/index/ivf_pq.cpp:4412-4490): magic, version,
// flags, dims, centroids, codebooks, optional R, lists as (id, code) entries, FNV-1a
// trailer.  The directory is created; the file is <path>/ivfpq.bin.
// Byte offsets of each list's size field inside the inverted-list section (after the
// u32 list count) for list sizes offs.
std::vector<uint64_t> list_byte_offsets(const std::vector<uint64_t>& offs, uint32_t m) {
    const size_t nlist = offs.size() - 1;
    std::vector<uint64_t> lb(nlist + 1);
    uint64_t p = 4;
    for (size_t l = 0; l < nlist; ++l) {
        lb[l] = p;
        p += 8 + (offs[l + 1] - offs[l]) * (8 + (uint64_t)m);
    }
    lb[nlist] = p;
    return lb;
}

// Metadata JSON check used by the v1.1 writer and reader (validate_json_structure,
// src/index/ivf_pq.cpp:113-160): well-formed UTF-8, one JSON value by the RFC 8259
// grammar with nothing after it, nesting depth <= 64 and at most 4096 object keys.
class JsonCheck {
public:
    explicit JsonCheck(std::string_view s) : s_(s) {}
    // empty string = valid, else the reason
    std::string run() {
        if (!utf8_ok()) return "Metadata JSON is not valid UTF-8";
        ws();
        if (!value()) return "Metadata JSON is structurally invalid";
        ws();
        if (i_ != s_.size()) return "Trailing characters after JSON";
        return {};
    }

private:
    std::string_view s_;
    size_t i_ = 0, depth_ = 0, keys_ = 0;

    bool utf8_ok() const {
        const auto* p = reinterpret_cast<const uint8_t*>(s_.data());
        const size_t n = s_.size();
        for (size_t i = 0; i < n;) {
            const uint8_t c = p[i];
            int len = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
            if (len == 0 || i + len > n) return false;
            uint32_t cp = len == 1 ? c : len == 2 ? (c & 0x1f) : len == 3 ? (c & 0x0f) : (c & 0x07);
            for (int k = 1; k < len; ++k) {
                if ((p[i + k] & 0xc0) != 0x80) return false;
                cp = (cp << 6) | (p[i + k] & 0x3f);
            }
            static constexpr uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
            if (cp < kMin[len] || cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff)) return false;
            i += len;
        }
        return true;
    }
    bool more() const { return i_ < s_.size(); }
    void ws() {
        while (more() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    bool lit(std::string_view w) {
        if (s_.substr(i_, w.size()) != w) return false;
        i_ += w.size();
        return true;
    }
    static bool digit(char c) { return c >= '0' && c <= '9'; }
    bool digits() {
        const size_t b = i_;
        while (more() && digit(s_[i_])) ++i_;
        return i_ > b;
    }
    bool number() {
        if (more() && s_[i_] == '-') ++i_;
        if (!more()) return false;
        if (s_[i_] == '0') ++i_;
        else if (!digits()) return false;
        if (more() && s_[i_] == '.') { ++i_; if (!digits()) return false; }
        if (more() && (s_[i_] == 'e' || s_[i_] == 'E')) {
            ++i_;
            if (more() && (s_[i_] == '+' || s_[i_] == '-')) ++i_;
            if (!digits()) return false;
        }
        return true;
    }
    bool string() {
        if (!more() || s_[i_] != '"') return false;
        ++i_;
        while (more()) {
            const char c = s_[i_++];
            if (c == '"') return true;
            if (c != '\\') continue;
            if (!more()) return false;
            const char e = s_[i_++];
            if (e == 'u') {
                for (int k = 0; k < 4; ++k, ++i_)
                    if (!more() || !std::isxdigit(static_cast<unsigned char>(s_[i_]))) return false;
            } else if (std::string_view("\"\\/bfnrt").find(e) == std::string_view::npos) {
                return false;
            }
        }
        return false;
    }
    // '[' or '{' already current; close = ']' or '}'
    bool container(char close, bool object) {
        ++i_;
        if (++depth_ > 64) return false;
        ws();
        if (more() && s_[i_] == close) { ++i_; --depth_; return true; }
        while (more()) {
            if (object) {
                if (!string() || ++keys_ > 4096) return false;
                ws();
                if (!more() || s_[i_] != ':') return false;
                ++i_;
            }
            if (!value()) return false;
            ws();
            if (!more()) return false;
            if (s_[i_] == ',') { ++i_; ws(); continue; }
            if (s_[i_] == close) { ++i_; --depth_; return true; }
            return false;
        }
        return false;
    }
    bool value() {
        ws();
        if (!more()) return false;
        switch (s_[i_]) {
            case '"': return string();
            case '{': return container('}', true);
            case '[': return container(']', false);
            case 't': return lit("true");
            case 'f': return lit("false");
            case 'n': return lit("null");
            default: return number();
        }
    }
};
}  // namespace

// IvfPqIndex::save (src/index/ivf_pq.cpp:4241-4491): the v1.0 monolithic layout, or the
// v1.1 sectioned layout with VESPER_IVFPQ_SAVE_V11=1 (sections stored uncompressed:
// compressed size = uncompressed size).  The inverted-list section is packed on the device.
auto IvfPqIndex::save(const std::string& path) const -> std::expected<void, core::error> {
    namespace fs = std::filesystem;
    const auto& I = *impl_;
    if (!I.trained) return fail(error_code::internal, "PQ not trained", "ivf_pq.save");
    const bool v11 = env_flag("VESPER_IVFPQ_SAVE_V11");
    if (v11 && !I.metadata_json.empty()) {
        if (I.metadata_json.size() > 64u * 1024u)
            return fail(error_code::config_invalid, "Metadata JSON too large (limit 64 KiB)", "ivf_pq.save");
        const std::string why = JsonCheck(I.metadata_json).run();
        if (!why.empty()) return fail(error_code::config_invalid, "Metadata JSON invalid: " + why, "ivf_pq.save");
    }
    std::error_code fec;
    fs::create_directories(path, fec);
    if (fec) return fail(error_code::io_failed, "Failed to create directory: " + path, "ivf_pq.save");
    const std::string file_path = path + "/ivfpq.bin";
    std::ofstream f(file_path, std::ios::binary);
    if (!f) return fail(error_code::io_failed, "Failed to open file for writing: " + file_path, "ivf_pq.save");
    const uint32_t dim = (uint32_t)I.dim, nlist = I.params.nlist, m = I.params.m, nbits = I.params.nbits,
                   dsub = (uint32_t)I.dsub, code_size = m;
    // the inverted-list section, packed on the device
    const std::vector<uint64_t> lb = list_byte_offsets(I.h_offs, m);
    std::vector<uint8_t> inv(lb[nlist]);
    std::memcpy(inv.data(), &nlist, 4);
    {
        DeviceGuard g(I.dev);
        try {
            vgpu::DeviceBuffer<uint64_t> d_lb(nlist + 1);
            vgpu::DeviceBuffer<uint8_t> d_raw(inv.size());
            h2d(d_lb.data(), lb.data(), lb.size(), I.st);
            vgpu::launch_pack_lists(I.d_ids.data(), I.d_codes.data(), I.d_offs.data(), (int)nlist, (int)m,
                                    d_lb.data(), d_raw.data(), I.st);
            d2h(inv.data() + 4, d_raw.data() + 4, inv.size() - 4, I.st);
            sync(I.st);
        } catch (const vgpu::CudaError& e) {
            return fail(error_code::internal, e.what(), "ivf_pq.cuda");
        }
    }
    Fnv fnv;
    auto put = [&](const void* p, size_t n) {
        fnv.update(p, n);
        f.write(static_cast<const char*>(p), (std::streamsize)n);
    };
    const char magic[8] = {'I', 'V', 'F', 'P', 'Q', 'v', '1', v11 ? '1' : '0'};
    put(magic, 8);
    const uint16_t vmaj = 1, vmin = v11 ? 1 : 0;
    put(&vmaj, 2);
    put(&vmin, 2);
    const uint32_t flags = (I.params.use_opq && I.has_rot) ? 1u : 0u;
    put(&flags, 4);
    const uint64_t nvec = I.n_vectors;
    const uint64_t ts = (uint64_t)std::chrono::system_clock::to_time_t(std::chrono::system_clock::now());
    put(&dim, 4); put(&nlist, 4); put(&m, 4); put(&nbits, 4); put(&dsub, 4);
    put(&nvec, 8); put(&code_size, 4); put(&ts, 8);
    const uint32_t meta_len = 0;
    put(&meta_len, 4);
    if (v11) {
        // section header: type u32, uncompressed u64, stored u64, FNV-1a of the payload u64
        auto section = [&](uint32_t type, const void* data, uint64_t bytes) {
            Fnv sh;
            sh.update(data, bytes);
            put(&type, 4); put(&bytes, 8); put(&bytes, 8); put(&sh.h, 8);
            if (bytes) put(data, bytes);
        };
        section(1, I.h_cent.data(), I.h_cent.size() * 4);
        section(2, I.h_cb.data(), I.h_cb.size() * 4);
        if (flags & 1u) section(4, I.h_rot.data(), I.h_rot.size() * 4);
        if (!I.metadata_json.empty()) section(5, I.metadata_json.data(), I.metadata_json.size());
        section(3, inv.data(), inv.size());
    } else {
        put(I.h_cent.data(), I.h_cent.size() * 4);
        put(I.h_cb.data(), I.h_cb.size() * 4);
        if (flags & 1u) put(I.h_rot.data(), I.h_rot.size() * 4);
        put(inv.data(), inv.size());
    }
    const char tail[4] = {'C', 'H', 'K', 'S'};
    f.write(tail, 4);
    f.write(reinterpret_cast<const char*>(&fnv.h), 8);
    if (!f) return fail(error_code::io_failed, "Failed writing " + file_path, "ivf_pq.save");
    return {};
}

// IvfPqIndex::load (src/index/ivf_pq.cpp:4493-4966): v1.0 monolithic or v1.1 sectioned.
// Sections are checked as the reference's mapped-file reader checks them (4565-4690):
// every section's FNV-1a checksum, including unknown types, which are then skipped; a
// compressed section is refused (this build has no Zstandard).  The file checksum is
// verified first, and the inverted-list section is uploaded once and unpacked on the
// device.
auto IvfPqIndex::load(const std::string& path) -> std::expected<IvfPqIndex, core::error> {
    const std::string file_path = path + "/ivfpq.bin";
    std::ifstream f(file_path, std::ios::binary);
    if (!f) return fail(error_code::not_found, "Index file not found: " + file_path, "ivf_pq.load");
    f.seekg(0, std::ios::end);
    const std::streamoff fsize = f.tellg();
    if (fsize < 64) return fail(error_code::config_invalid, "File too small", "ivf_pq.load");
    f.seekg(0, std::ios::beg);
    std::vector<char> raw((size_t)fsize);
    f.read(raw.data(), fsize);
    if (f.gcount() != fsize) return fail(error_code::io_failed, "Failed reading file", "ivf_pq.load");
    const size_t body_end = (size_t)fsize - 12;
    if (std::memcmp(raw.data() + body_end, "CHKS", 4) != 0)
        return fail(error_code::config_invalid, "Missing checksum trailer", "ivf_pq.load");
    uint64_t chk = 0;
    std::memcpy(&chk, raw.data() + body_end + 4, 8);
    {
        Fnv fnv;
        fnv.update(raw.data(), body_end);
        if (chk != fnv.h) return fail(error_code::config_invalid, "Checksum mismatch", "ivf_pq.load");
    }
    size_t off = 0;
    auto get = [&](void* p, size_t n) -> bool {
        if (off + n > body_end) return false;
        std::memcpy(p, raw.data() + off, n);
        off += n;
        return true;
    };
    char magic[8];
    if (!get(magic, 8)) return fail(error_code::io_failed, "Failed reading magic", "ivf_pq.load");
    const bool v11 = std::string_view(magic, 8) == std::string_view("IVFPQv11", 8);
    if (!v11 && std::string_view(magic, 8) != std::string_view("IVFPQv10", 8))
        return fail(error_code::config_invalid, "Magic mismatch", "ivf_pq.load");
    uint16_t vmaj = 0, vmin = 0;
    if (!get(&vmaj, 2) || !get(&vmin, 2)) return fail(error_code::io_failed, "Failed reading version", "ivf_pq.load");
    if (vmaj != 1) return fail(error_code::config_invalid, "Unsupported version", "ivf_pq.load");
    uint32_t flags = 0, dim = 0, nlist = 0, m = 0, nbits = 0, dsub = 0, code_size = 0, meta_len = 0;
    uint64_t nvec = 0, ts = 0;
    if (!get(&flags, 4) || !get(&dim, 4) || !get(&nlist, 4) || !get(&m, 4) || !get(&nbits, 4) || !get(&dsub, 4) ||
        !get(&nvec, 8) || !get(&code_size, 4) || !get(&ts, 8) || !get(&meta_len, 4))
        return fail(error_code::io_failed, "Failed reading header", "ivf_pq.load");
    if (dim == 0 || m == 0 || nlist == 0 || nbits == 0 || nbits > 8 || dsub * m != dim)
        return fail(error_code::config_invalid, "Invalid header dimensions", "ivf_pq.load");
    if (meta_len > 64u * 1024u) return fail(error_code::config_invalid, "Metadata too large", "ivf_pq.load");
    std::string meta(meta_len, '\0');
    if (meta_len && !get(meta.data(), meta_len)) return fail(error_code::io_failed, "Failed reading metadata", "ivf_pq.load");
    if (meta_len) {
        const std::string why = JsonCheck(meta).run();
        if (!why.empty()) return fail(error_code::config_invalid, "Metadata JSON invalid (header): " + why, "ivf_pq.load");
    }
    const uint32_t ksub = 1u << nbits;
    std::vector<float> cent((size_t)nlist * dim), cb((size_t)m * ksub * dsub), rot;
    size_t inv_off = 0, inv_len = 0;
    bool have_cent = false, have_cb = false, have_inv = false;
    if (v11) {
        while (off < body_end) {
            uint32_t type = 0;
            uint64_t unc = 0, comp = 0, shash = 0;
            if (!get(&type, 4) || !get(&unc, 8) || !get(&comp, 8) || !get(&shash, 8)) break;
            if (comp > body_end - off) return fail(error_code::io_failed, "Failed reading section payload", "ivf_pq.load");
            const char* payload = raw.data() + off;
            off += comp;
            if (unc == 0 && comp == 0) continue;
            if (comp != unc && unc != 0)
                return fail(error_code::config_invalid, "Decompression failed (compressed sections need Zstandard)",
                            "ivf_pq.load");
            if (unc) {
                Fnv sh;
                sh.update(payload, unc);
                if (sh.h != shash) return fail(error_code::config_invalid, "Section checksum mismatch", "ivf_pq.load");
            }
            switch (type) {
                case 1:
                    if (unc != cent.size() * 4) return fail(error_code::config_invalid, "Centroids size mismatch", "ivf_pq.load");
                    std::memcpy(cent.data(), payload, unc);
                    have_cent = true;
                    break;
                case 2:
                    if (unc != cb.size() * 4) return fail(error_code::config_invalid, "Codebooks size mismatch", "ivf_pq.load");
                    std::memcpy(cb.data(), payload, unc);
                    have_cb = true;
                    break;
                case 4:
                    if (unc != (uint64_t)dim * dim * 4) return fail(error_code::config_invalid, "OPQ size mismatch", "ivf_pq.load");
                    rot.resize((size_t)dim * dim);
                    std::memcpy(rot.data(), payload, unc);
                    flags |= 1u;
                    break;
                case 5: {
                    if (unc > 64u * 1024u) return fail(error_code::config_invalid, "Metadata too large", "ivf_pq.load");
                    std::string sec(payload, unc);
                    const std::string why = JsonCheck(sec).run();
                    if (!why.empty())
                        return fail(error_code::config_invalid, "Metadata JSON invalid (section): " + why, "ivf_pq.load");
                    meta = std::move(sec);
                    break;
                }
                case 3:
                    inv_off = (size_t)(payload - raw.data());
                    inv_len = unc;
                    have_inv = true;
                    break;
                default:
                    break;  // unknown sections are skipped
            }
        }
        if (!have_cent || !have_cb) return fail(error_code::config_invalid, "Missing centroid or codebook section", "ivf_pq.load");
    } else {
        if (!get(cent.data(), cent.size() * 4)) return fail(error_code::io_failed, "Failed reading centroid row", "ivf_pq.load");
        if (!get(cb.data(), cb.size() * 4)) return fail(error_code::io_failed, "Failed reading PQ codebooks", "ivf_pq.load");
        if (flags & 1u) {
            rot.resize((size_t)dim * dim);
            if (!get(rot.data(), rot.size() * 4)) return fail(error_code::io_failed, "Failed reading OPQ rotation", "ivf_pq.load");
        }
        inv_off = off;
        inv_len = body_end - off;
        have_inv = true;
    }
    // list sizes from the inverted-list section's headers (error texts: v1.1 section
    // parser, src/index/ivf_pq.cpp:4839-4857; v1.0 stream reader, 4939-4949)
    std::vector<uint64_t> offs(nlist + 1, 0), lb(nlist + 1, 0);
    if (have_inv) {
        const char* q = raw.data() + inv_off;
        const uint64_t rec = 8 + (uint64_t)m;
        uint32_t lists_count = 0;
        if (inv_len < 4)
            return v11 ? fail(error_code::config_invalid, "Inverted too small", "ivf_pq.load")
                       : fail(error_code::io_failed, "Failed reading lists_count", "ivf_pq.load");
        std::memcpy(&lists_count, q, 4);
        if (lists_count != nlist) return fail(error_code::config_invalid, "lists_count mismatch", "ivf_pq.load");
        uint64_t p = 4;
        for (uint32_t l = 0; l < nlist; ++l) {
            uint64_t sz = 0;
            if (inv_len - p < 8)
                return v11 ? fail(error_code::config_invalid, "List header truncated", "ivf_pq.load")
                           : fail(error_code::io_failed, "Failed reading list size", "ivf_pq.load");
            std::memcpy(&sz, q + p, 8);
            if (sz > (inv_len - p - 8) / rec)
                return v11 ? fail(error_code::config_invalid, "Entry truncated", "ivf_pq.load")
                           : fail(error_code::io_failed, "Failed reading id", "ivf_pq.load");
            lb[l] = p;
            offs[l + 1] = offs[l] + sz;
            p += 8 + sz * rec;
        }
        if (p != inv_len)
            return fail(error_code::config_invalid, v11 ? "Inverted section extra bytes" : "Missing checksum trailer",
                        "ivf_pq.load");
    }
    const uint64_t n_entries = offs[nlist];

    IvfPqIndex index;
    auto r = index.set_model(dim, nlist, m, nbits, cent.data(), cb.data(), rot.empty() ? nullptr : rot.data());
    if (!r) return std::unexpected(r.error());
    auto& I = *index.impl_;
    DeviceGuard g(I.dev);
    try {
        I.params.use_opq = (flags & 1u) != 0;
        I.metadata_json = meta;
        I.h_offs = offs;
        I.n_vectors = n_entries;
        I.d_offs.resize(nlist + 1);
        h2d(I.d_offs.data(), offs.data(), offs.size(), I.st);
        I.d_ids.resize(std::max<size_t>(n_entries, 1));
        I.d_codes.resize(std::max<size_t>(n_entries * m, 1));
        if (n_entries) {
            vgpu::DeviceBuffer<uint8_t> d_raw(inv_len);
            vgpu::DeviceBuffer<uint64_t> d_lb(nlist + 1);
            h2d(d_raw.data(), reinterpret_cast<const uint8_t*>(raw.data() + inv_off), inv_len, I.st);
            h2d(d_lb.data(), lb.data(), lb.size(), I.st);
            vgpu::launch_unpack_lists(d_raw.data(), d_lb.data(), I.d_offs.data(), (int)nlist, (int)m, I.d_ids.data(),
                                      I.d_codes.data(), I.st);
            sync(I.st);
        }
        I.recompute_vterms();
        I.rebuild_blocks();
        sync(I.st);
    } catch (const vgpu::CudaError& e) {
        return fail(error_code::internal, e.what(), "ivf_pq.cuda");
    }
    return index;
}

}  // namespace vesper::index
