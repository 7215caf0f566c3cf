// Tensor-core screening + exact refine for nearest-centroid search (tc_coarse.cu).
#pragma once

#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace vgpu {

// tcgen05 needs dim % 4 == 0 (16-byte TMA rows) and at least one 32-wide K tile.
bool tc_screen_supported(int dim);
// Dt[i][j] = ||x_i||^2 + ||c_j||^2 - 2 <x_i, c_j> with tf32 tensor-core products.
// err receives a nonzero code if a bounded wait timed out.
void launch_tc_screen(const float* x, long long nx, const float* c, int nc, int dim, const float* xn,
                      const float* cn, float* Dt, long long ldd, int* err, cudaStream_t st);
// ip: Dt = -2 <x_i, c_j> instead (inner-product screen).  c_stride: row stride of c in
// elements (0 = dim), e.g. to screen a strided sample of a base set.
void launch_tc_screen_op(bool ip, const float* x, long long nx, const float* c, long long nc, long long c_stride,
                         int dim, const float* xn, const float* cn, float* Dt, long long ldd, int* err,
                         cudaStream_t st);
// Flat top-k filter: the same screen without storing it; column j of row i is appended
// to cand[i * cap + ...] as {j + col_off, screen value bits} (count in cand_cnt[i],
// which may exceed cap) when its lower bound is <= tau[i] (L2: distance; ip: -2 *
// inner product).
// cs: sqrt(cn), precomputed.
// c_stride: row stride of c in elements (0 = dim).
void launch_tc_filter(bool ip, const float* x, long long nx, const float* c, long long nc, long long c_stride,
                      int dim, const float* xn, const float* cn, const float* cs, const float* tau, uint32_t col_off,
                      uint2* cand, uint32_t* cand_cnt, int cap, int* err, cudaStream_t st);
// OPQ rotation of a query batch on the tensor cores (3xTF32, tc_coarse.cu): out[i][j] =
// sum_k x_i[k] W[j][k] to a few 1e-7 relative, W = R^T for the x R of apply_rotation
// (FAST search only; EXACT search, add() and training keep the sequential fp32
// rotation).  prepare_rotation_3xtf32 fills W3 [dim x 3 dim] from W once per model; x3
// is [n x 3 dim] scratch; err as for launch_tc_screen.
bool rotate_3xtf32_supported(int dim);
void prepare_rotation_3xtf32(const float* W, int dim, float* W3, cudaStream_t st);
void launch_rotate_3xtf32(const float* x, long long n, int dim, const float* R3, float* x3, float* out, int* err,
                          cudaStream_t st);
// out[i] = sqrt(in[i]).
void launch_sqrt(const float* in, long long n, float* out, cudaStream_t st);
// Exact flat top-k (flat_topk.cu).  Stage times of the last call, in ms.
struct FlatStats {
    float total_ms = 0, norms_ms = 0, sample_ms = 0, filter_ms = 0, refine_ms = 0, fallback_ms = 0;
    unsigned long long candidates = 0;  // kept columns over all queries (pass 2)
    uint32_t overflow_queries = 0;      // queries redone by the single-pass path
    int sample_stride = 0, cap = 0, single_pass = 0;
    uint32_t launches = 0;              // kernels launched by the call
};
struct FlatWork {
    static constexpr int kLevels = 4;   // sample levels of the threshold recursion
    struct Level {
        DeviceBuffer<float> cn, cs, s_val;
        DeviceBuffer<uint32_t> s_idx;
    } level[kLevels];
    DeviceBuffer<float> xn, cn, csq, tau, dt, oq, oxn, o_val, cmax, caug;
    DeviceBuffer<uint32_t> cand_cnt, over, o_idx, o_rows;
    DeviceBuffer<uint2> cand;
    DeviceBuffer<int> err;
    cudaEvent_t ev[7] = {};
    // host-resident base: copy stream, sample-rows event, per-chunk events
    cudaStream_t copy_st = nullptr;
    cudaEvent_t sample_ev = nullptr;
    DeviceBuffer<float> sample_rows;   // the threshold pass's rows, copied apart from the base
    std::vector<cudaEvent_t> chunk_ev;
    FlatStats last;
    int launches = 0;
    FlatWork() = default;
    FlatWork(const FlatWork&) = delete;
    FlatWork& operator=(const FlatWork&) = delete;
    ~FlatWork();
};
// ip: inner product (largest first), else squared L2 (smallest first).  q, base: device
// rows (16-byte aligned); out_idx/out_score: device [nq x k].  Synchronous on st.
void launch_flat_topk(bool ip, const float* q, long long nq, const float* base, long long nb, int dim, int k,
                      uint32_t* out_idx, float* out_score, FlatWork& w, cudaStream_t st);
// Exact k nearest rows of c [nc x dim] for every row of x [nx x dim] under squared L2
// (reference lane order; ties to the lowest index): launch_flat_topk's sampled-threshold
// filter path, which never writes an nx x nc matrix of screen values.  keep (device
// [nx], may be null, k == 1 only): where the row's current centroid ties the nearest,
// it stays (KmeansElkan::assign_with_bounds).  keep must not alias out_idx.  out_val
// receives the exact distances.  Synchronous on st.
void launch_exact_nearest(const float* x, long long nx, const float* c, long long nc, int dim, int k,
                          const uint32_t* keep, uint32_t* out_idx, float* out_val, FlatWork& w, cudaStream_t st);
// The same with the base in host memory (pinned for the copy to overlap): `dev_base`
// [nb x dim] receives it.  The threshold pass's sample rows are copied first; the rest
// arrives in chunks on a second stream while the sample pass runs, and each chunk is
// filtered as soon as it lands.  Results are those of launch_flat_topk on the copied base.
void launch_flat_topk_host(bool ip, const float* q, long long nq, const float* host_base, float* dev_base,
                           long long nb, int dim, int k, uint32_t* out_idx, float* out_score, FlatWork& w,
                           cudaStream_t st);

// Fused exact nearest centroid (k = 1) on the tensor cores (tc_argmin_kernel): x [nx x
// dim] against c [nc x dim] with row norms xn, column norms cn, their square roots cs
// and cmax = {max cn, max cs} (launch_col_max).  out_idx/out_val receive the reference
// lane-order arg-min (ties to the lowest index; with keep, to keep[row] -- keep must not
// alias out_idx).  Rows whose candidate list overflowed are appended to over[] with
// *n_over counting them (zero it first); they are left for the caller.  err receives a
// nonzero code if a bounded wait expired.
// caug: workspace of nc * aug_ld(dim) floats for the augmented centroid operand.
bool tc_argmin_supported(int dim);
void launch_col_max(const float* cn, const float* cs, int nc, float* cmax, cudaStream_t st);
void launch_tc_argmin(const float* x, long long nx, const float* c, int nc, int dim, const float* xn, const float* cn,
                      const float* cs, const float* cmax, const uint32_t* keep, uint32_t* out_idx, float* out_val,
                      uint32_t* over, uint32_t* n_over, float* caug, int* err, cudaStream_t st);
// The augmented centroid operand of the L2 screens (tc_argmin_kernel, tc_filter_kernel):
// row i = (c_i, zeros to a multiple of 32, -hi, -lo, zeros), aug_ld(dim) floats, with
// hi + lo the two-term tf32 split of ||c_i||^2 / 2 (cn[i] / 2); c's row i at c + i * c_ld.
int aug_ld(int dim);
void launch_aug_cols(const float* c, long long nc, int dim, long long c_ld, const float* cn, float* out,
                     cudaStream_t st);
void launch_scatter_top1(const uint32_t* rows, int n, const uint32_t* idx, const float* val, uint32_t* out_idx,
                         float* out_val, cudaStream_t st);
// launch_tc_filter's keep rule on the persistent pipeline of tc_argmin_kernel (each CTA
// walks a share of the column tiles for its 128 rows); cmax from launch_col_max over
// the same columns' cn / cs.  Same outputs and semantics as launch_tc_filter.  caug
// (L2 only, may be null): the same columns' augmented operand (launch_aug_cols), which
// moves ||c||^2 into the tensor-core product; the kept values are then ||x||^2 - 2 S'.
void launch_tc_filter_persistent(bool ip, const float* x, long long nx, const float* c, long long nc,
                                 long long c_stride, int dim, const float* xn, const float* cn, const float* cs,
                                 const float* cmax, const float* tau, uint32_t col_off, uint2* cand,
                                 uint32_t* cand_cnt, int cap, int* err, cudaStream_t st,
                                 const float* caug = nullptr);
// out[i] = ||x_i||^2 (fp64 accumulation); row i at x + i * ld (ld = dim by default).
void launch_row_norms(const float* x, long long n, int dim, float* out, cudaStream_t st, long long ld = 0);
// Per row: exact k nearest centroids (reference-order distances, ties to the lowest
// index; `keep` applies Elkan's keep-on-tie rule to the nearest).  Dt from
// launch_tc_screen bounds which centroids need the exact recomputation.
void launch_screen_select(const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                          const float* cent, const float* xn, const float* cn, int k, const uint32_t* keep,
                          uint32_t* out_idx, float* out_val, int* err, cudaStream_t st);
// The same for L2 or inner-product screens (ip: exact reference-order inner products,
// larger first); column j is row j * cent_ld of cent.
void launch_screen_select_op(bool ip, const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                             const float* cent, long long cent_ld, const float* xn, const float* cn, int k,
                             uint32_t* out_idx, float* out_val, int* err, cudaStream_t st);

}  // namespace vgpu

namespace vgpu {

// ---------------------------------------------------------------------------------
// List-major tensor-core FAST scan (tc_scan.cu).
// ---------------------------------------------------------------------------------
// Shapes the kernel handles: 256 codes per sub-space, dim a multiple of 64 up to 768,
// dim / m in {4, 8, 16}, and an m the blocked scan supports (it provides the
// thresholds and handles overflowed queries).
bool tc_list_scan_supported(int dim, int m, int ksub);

// Per-batch scratch, grown on demand and reused.  bf16 arrays are held as uint16_t.
struct TlWork {
    DeviceBuffer<uint16_t> rqb, qperm;
    DeviceBuffer<float> rqn, tau, tau_x, p1_d;
    DeviceBuffer<uint64_t> p1_ids;
    DeviceBuffer<uint32_t> p1_n, cnt, cursor, seg_off, units, unit_off, unit_list, seg_meta, cand_cnt, counter;
    DeviceBuffer<uint32_t> p0, mcount, mins_off, run_lut;   // threshold pass over long nearest lists
    DeviceBuffer<float> pbase0, mins;
    uint32_t* host_u32 = nullptr;                            // pinned
    DeviceBuffer<unsigned long long> cand;
    DeviceBuffer<unsigned char> scan_tmp;
    // stats[0] += candidates refined, stats[1] += queries left to the blocked scan
    // (zeroed by the caller); ev brackets the screening kernel of the last launch.
    DeviceBuffer<unsigned long long> stats;
    // ev[0..5]: start, threshold scan done, batch prep done, screen done, refine done,
    // fallback done (of the last launch)
    cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    SplitWork split;  // threshold scan and overflow fallback
    int cap = 0;
    bool pairs = false;  // screen on CTA pairs (tcgen05 cta_group::2) instead of single CTAs
    void reserve(long long nq, int nprobe, int nlist, int dim, int k, int cap, size_t n_vectors);
    TlWork() = default;
    TlWork(const TlWork&) = delete;
    TlWork& operator=(const TlWork&) = delete;
    ~TlWork() {
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        if (host_u32) cudaFreeHost(host_u32);
    }
};

struct TlScanArgs {
    const float* T;          // blocked lookup tables [nq x m x 256]
    const float* rq;         // rotated queries [nq x dim]
    const float* pbase;      // [nq x nprobe] (launch_probe_base)
    const uint32_t* probe;   // [nq x nprobe]
    long long nq;
    int nprobe, nlist, dim, m, k;
    const uint64_t* offs;    // CSR list offsets
    const uint8_t* codes;    // CSR codes
    const float* vterm;      // CSR per-entry terms
    const float* xnorm;      // CSR per-entry decoded norms
    const uint16_t* cbb;     // bf16 codebooks [m x 256 x dsub]
    const float* cb = nullptr;  // fp32 codebooks [m x 256 x dsub] (the refine's table entries)
    const uint64_t* blk_off; // blocked copy (threshold scan and overflow fallback)
    const uint8_t* bcodes;
    const float* bvterm;
    const uint64_t* ids;
    uint64_t* out_ids;
    float* out_d;
    uint32_t* out_n;
    int* err;
    // Optional exchange of the per-query thresholds between the shards of one database
    // (ThresholdExchangeFn, ivf_pq_gpu.hpp): called on the host after the threshold pass
    // with tau_x [nq] on the device (+inf where this shard has no bound) and the stream;
    // it must leave the element-wise minimum over every shard in tau_x, ordered on that
    // stream, and return 0.
    int (*tau_fn)(float* d_tau, size_t nq, void* stream, void* user) = nullptr;
    void* tau_user = nullptr;
    // With an exchange, this shard's own threshold pass covers only the queries q with
    // q mod tau_shards == tau_shard; the exchange brings the other queries' bounds.
    uint32_t tau_shard = 0, tau_shards = 1;
};

// FAST search results identical to launch_scan_blocked over all nprobe probes.
void launch_tc_list_scan(const TlScanArgs& a, TlWork& w, cudaStream_t st);
// out[i] = bf16(cb[i]).
void launch_codebook_bf16(const float* cb, long long n, uint16_t* out, cudaStream_t st);
// xnorm[e] = ||decoded entry e|| (rounded up), for the screen's error bound.
void launch_entry_norms(const uint8_t* codes, long long n, const float* cb, int m, int dsub, float* xnorm,
                        cudaStream_t st);
void launch_query_prep(const float* rq, long long nq, int dim, uint16_t* rqb, float* rqn, cudaStream_t st);

}  // namespace vgpu
