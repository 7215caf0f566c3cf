// B200 IVF-PQ index: the host-side mirror of the reference's IvfPqIndex
// (include/vesper/index/ivf_pq.hpp:140-386).  Same method names, argument meaning and
// error behaviour; the work runs in the CUDA kernels of this directory.
//
// Data layout in HBM (one index = one device):
//   centroids   float [nlist x dim]            coarse quantizer
//   codebooks   float [m x ksub x dsub]        PQ codebooks (export_codebooks layout)
//   rotation    float [dim x dim]              OPQ matrix R (row-vector convention x*R)
//   rot_T       float [dim x dim]              R transposed (apply_rotation_T)
//   rc          float [nlist x dim]            centroids * R (fast scan)
//   list_offs   u64   [nlist + 1]              CSR offsets of the inverted lists
//   codes       u8    [N x m]                  PQ codes, list-contiguous, insertion order
//   ids         u64   [N]                      user ids, same order
//   vterm       float [N]                      per-vector term of the fast scan
#pragma once

#include <cstddef>
#include <cstdint>
#include <expected>
#include <memory>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace vesper::core {

// Error taxonomy (include/vesper/error.hpp:19-44).
enum class error_code : std::uint32_t {
    ok = 0,
    io_failed = 1001,
    config_invalid = 2001,
    precondition_failed = 4001,
    out_of_memory = 5002,
    not_found = 6001,
    internal = 9001,
    invalid_argument = 9002,
    not_initialized = 9003,
    out_of_range = 9004,
    unsupported = 9005,
};

struct error {
    error_code code{error_code::internal};
    std::string message;
    std::string component;
};

}  // namespace vesper::core

namespace vesper::index {

enum class OpqInit { Identity, PCA };
enum class CoarseAssigner { Brute, HNSW, KDTree, Projection };
enum class KmeansInit { KMeansPlusPlus, KMeansParallel };

// Search arithmetic.  Exact: every distance, LUT and rotation in the reference's
// operation order (bit-identical results).  Fast: lookup table built once per query
// (distance = ||q - c||^2 + u(x) + sum_s T_q[s][code]); distances agree with Exact to
// fp32 rounding (well inside 1e-4 relative).
enum class SearchMode : std::uint32_t { Fast = 0, Exact = 1 };

// ivf_pq.hpp:59-106 (fields the GPU engine reads; the rest are accepted and ignored:
// every coarse assigner of the reference returns the exact nearest centroid, which
// is what the GPU computes by brute force).
struct IvfPqTrainParams {
    std::uint32_t nlist{256};
    std::uint32_t m{8};
    std::uint32_t nbits{8};
    std::uint32_t max_iter{25};
    float epsilon{1e-4f};
    bool verbose{false};
    bool use_opq{true};
    std::uint32_t opq_iter{10};
    std::size_t opq_sample_n{20000};
    OpqInit opq_init{OpqInit::PCA};
    std::uint32_t seed{42};
    KmeansInit kmeans_init_method{KmeansInit::KMeansPlusPlus};
    CoarseAssigner coarse_assigner{CoarseAssigner::KDTree};
    bool use_centroid_ann{true};
    bool timings_enabled{false};
};

// ivf_pq.hpp:109-117, plus the GPU search mode.
struct IvfPqSearchParams {
    std::uint32_t nprobe{8};
    std::uint32_t k{10};
    std::uint32_t cand_k{0};
    bool use_exact_rerank{false};
    std::uint32_t rerank_k{0};
    SearchMode mode{SearchMode::Fast};
};

struct IvfPqTrainStats {
    std::uint32_t iterations{0};
    float final_error{0.0f};
    float train_time_sec{0.0f};
    std::vector<float> errors;
    // GPU additions: what the trainer decided / measured.
    bool opq_kept{false};
    double err_unrot{0.0};
    double err_opq{0.0};
    std::uint32_t coarse_iterations{0};
};

// Per-stage device times of the last search_batch call (CUDA events, ms).
struct SearchTimings {
    float coarse_ms{0}, select_ms{0}, rotate_ms{0}, scan_ms{0}, merge_ms{0}, total_ms{0};
    std::uint64_t scanned_entries{0};   // sum over queries of the probed lists' sizes
    std::uint32_t kernel_launches{0};   // kernels this library launched for the call
    std::uint32_t scan_variant{0};      // 1 exact per-list LUT, 2 per-query LUT, 3 blocked per-query LUT,
                                        // 4 tensor-core list scan + refine
    std::uint32_t coarse_variant{0};    // 1 CUDA-core exact distances, 2 tensor-core screen + exact refine, 3 sampled-threshold filter + exact refine
    float list_kernel_ms{0};            // variant 4: device time of the tensor-core screening kernel
    std::uint64_t list_candidates{0};   // variant 4: pairs kept by the screen (refined)
    std::uint32_t list_fallback_queries{0};  // variant 4: queries handed to the blocked scan
    float list_threshold_ms{0};         // variant 4: nearest-list scan giving the thresholds
    float list_prep_ms{0};              // variant 4: bf16 queries, pair grouping, unit table
    float list_refine_ms{0};            // variant 4: exact re-scoring of the kept pairs
    float list_fallback_ms{0};          // variant 4: blocked scan of overflowed queries
    float rerank_ms{0};                 // exact rerank of the candidate pool (use_exact_rerank)
};

class IvfPqIndex {
public:
    IvfPqIndex();
    ~IvfPqIndex();
    IvfPqIndex(IvfPqIndex&&) noexcept;
    IvfPqIndex& operator=(IvfPqIndex&&) noexcept;
    IvfPqIndex(const IvfPqIndex&) = delete;
    IvfPqIndex& operator=(const IvfPqIndex&) = delete;

    auto train(const float* data, std::size_t dim, std::size_t n, const IvfPqTrainParams& params)
        -> std::expected<IvfPqTrainStats, core::error>;
    auto add(const std::uint64_t* ids, const float* data, std::size_t n)
        -> std::expected<void, core::error>;
    // train / add with the inputs in device memory of the index's GPU when on_device.
    auto train_device(const float* data, std::size_t dim, std::size_t n, const IvfPqTrainParams& params,
                      bool on_device) -> std::expected<IvfPqTrainStats, core::error>;
    auto add_device(const std::uint64_t* ids, const float* data, std::size_t n, bool on_device)
        -> std::expected<void, core::error>;
    auto search(const float* query, const IvfPqSearchParams& params) const
        -> std::expected<std::vector<std::pair<std::uint64_t, float>>, core::error>;
    auto search_batch(const float* queries, std::size_t n_queries, const IvfPqSearchParams& params) const
        -> std::expected<std::vector<std::vector<std::pair<std::uint64_t, float>>>, core::error>;

    // Flat-output batch search (the C ABI's layout): out_ids/out_dist [nq x k], padded
    // like vesper_ivfpq_search_batch; out_counts (optional) receives the number of
    // real results per query.  `on_device` = all four pointers are device pointers.
    auto search_batch_flat(const float* queries, std::size_t n_queries,
                           const IvfPqSearchParams& params, std::uint64_t* out_ids,
                           float* out_dist, std::uint32_t* out_counts, bool on_device) const
        -> std::expected<void, core::error>;

    // The coarse stage alone: the nprobe nearest lists of each query (device arrays
    // [nq x min(nprobe, nlist)], the probe order of search).  With
    // search_batch_device_probed, ranks that share a query batch can each probe a slice
    // of it and exchange the lists instead of all probing every query.
    auto probe_device(const float* d_queries, std::size_t n_queries, std::uint32_t nprobe, std::uint32_t* d_probe,
                      float* d_probe_d) const -> std::expected<void, core::error>;
    // Device search with the probe lists given (as probe_device writes them).
    auto search_batch_device_probed(const float* d_queries, std::size_t n_queries, const IvfPqSearchParams& params,
                                    const std::uint32_t* d_probe, const float* d_probe_d, std::uint64_t* d_out_ids,
                                    float* d_out_dist, std::uint32_t* d_out_counts) const
        -> std::expected<void, core::error>;

    // Threshold exchange between the shards of one database (one index per GPU, each
    // holding a part of the base set, all searching the same batch with the same
    // parameters).  While set, every search calls fn once per query chunk, on the host,
    // with d_tau [nq] on the index's device: each query's upper bound of its k-th FAST
    // distance over this shard (+inf where the shard has none), and the index's CUDA
    // stream.  fn must leave the element-wise minimum over all shards in d_tau, ordered
    // on that stream (e.g. an all-reduce MIN issued on it), and return 0; any other
    // return fails the search.  The tensor-core list scan then keeps only the entries
    // that can reach the shared bound, so each shard refines about its share of the
    // union's candidates; the union's top k is unchanged.  Searches that do not run the
    // list scan pass +inf for every query.  fn = nullptr removes it.
    // shards > 1: this index runs its own threshold pass only for the queries q with
    // q mod shards == shard and takes the other queries' bounds from the exchange, so
    // each shard of a W-way database pays 1/W of the pass (shards = 1: every query).
    using ThresholdExchangeFn = int (*)(float* d_tau, std::size_t n_queries, void* stream, void* user);
    void set_threshold_exchange(ThresholdExchangeFn fn, void* user, std::uint32_t shard = 0,
                                std::uint32_t shards = 1);

    // FAST-mode device search that allocates nothing: its temporary buffers come from
    // a fixed 64 MiB device array (noalloc_search.cu) instead of cudaMalloc.
    auto search_batch_device_noalloc(const float* d_queries, std::size_t n_queries,
                                     const IvfPqSearchParams& params, std::uint64_t* d_out_ids,
                                     float* d_out_dist, std::uint32_t* d_out_counts) const
        -> std::expected<void, core::error>;

    // The rest of the reference's index API (include/vesper/index/ivf_pq.hpp:252-386).
    // Vectors are rebuilt exactly as the reference does: centroid + apply_rotation_T(decode).
    // An id held by several entries resolves to the first in list order.
    auto reconstruct_cluster(std::uint32_t cluster_id, std::vector<std::uint64_t>& ids,
                             std::vector<float>& vectors) const -> std::expected<void, core::error>;
    auto reconstruct(std::uint64_t id) const -> std::expected<std::vector<float>, core::error>;
    auto get_vector(std::uint64_t id) const -> std::expected<std::vector<float>, core::error> {
        return reconstruct(id);
    }
    auto get_num_clusters() const -> std::expected<std::uint32_t, core::error>;
    auto get_dimension() const -> std::expected<std::size_t, core::error>;
    auto get_cluster_assignment(std::uint64_t id) const -> std::expected<std::uint32_t, core::error>;
    auto get_cluster_centroid(std::uint32_t cluster_id) const -> std::expected<std::vector<float>, core::error>;
    auto update_cluster_centroid(std::uint32_t cluster_id, const float* centroid)
        -> std::expected<void, core::error>;
    auto reassign_vector(std::uint64_t id, std::uint32_t new_cluster) -> std::expected<void, core::error>;
    // compact_inverted_list with the deleted ids given as a 32-bit id set (the reference
    // takes a roaring bitmap and tests static_cast<uint32_t>(id)); returns the number removed.
    auto compact_inverted_list(std::uint32_t cluster_id, const std::uint32_t* deleted_ids, std::size_t n_deleted)
        -> std::expected<std::size_t, core::error>;
    // Require VESPER_IVFPQ_DEBUG=1 like the reference.  (rank, assigned cluster) and
    // (rank, exact ADC distance); ranks are 1 + the number of strictly smaller values.
    auto debug_explain_centroid_rank(const float* query, std::uint64_t target_id) const
        -> std::expected<std::pair<std::size_t, std::uint32_t>, core::error>;
    auto debug_explain_adc_rank(const float* query, std::uint64_t target_id) const
        -> std::expected<std::pair<std::size_t, float>, core::error>;

    void set_metadata_json(std::string_view json);
    auto get_metadata_json() const -> std::string;

    struct Stats {
        std::size_t n_vectors{0};
        std::size_t n_lists{0};
        std::size_t m{0};
        std::size_t code_size{0};
        std::size_t memory_bytes{0};
        float avg_list_size{0.0f};
        bool timings_enabled{false};
        double t_assign_ms{0.0};
        double t_encode_ms{0.0};
        double t_lists_ms{0.0};
    };
    auto get_stats() const noexcept -> Stats;
    auto is_trained() const noexcept -> bool;
    auto dimension() const noexcept -> std::size_t;
    auto clear() -> void;
    auto reset() -> void;
    auto last_search_timings() const -> SearchTimings;

    // Model access (host copies) for tests and tools.
    auto centroids() const -> std::vector<float>;
    auto codebooks() const -> std::vector<float>;
    auto rotation() const -> std::vector<float>;
    auto list_offsets() const -> std::vector<std::uint64_t>;
    auto list_ids() const -> std::vector<std::uint64_t>;
    auto list_codes() const -> std::vector<std::uint8_t>;
    auto params() const -> IvfPqTrainParams;

    // Install a pre-trained model (centroids [nlist x dim], codebooks [m*ksub x dsub],
    // optional rotation [dim x dim]); clears the lists.
    auto set_model(std::size_t dim, std::uint32_t nlist, std::uint32_t m, std::uint32_t nbits,
                   const float* centroids, const float* codebooks, const float* rotation)
        -> std::expected<void, core::error>;

    // Persistence: v1.0 monolithic layout in <path>/ivfpq.bin (ivf_pq.cpp:4412-4490).
    auto save(const std::string& path) const -> std::expected<void, core::error>;
    static auto load(const std::string& path) -> std::expected<IvfPqIndex, core::error>;

    class Impl;

private:
    std::unique_ptr<Impl> impl_;
};

}  // namespace vesper::index
