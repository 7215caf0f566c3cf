/* B200 extensions to the Vesper IVF-PQ C ABI (libvesper_c.so).
 *
 * The reference's C struct carries only nlist/m/nbits and k/nprobe
 * (include/vesper/c/vesper.h:43-52); everything else in IvfPqTrainParams /
 * IvfPqSearchParams (include/vesper/index/ivf_pq.hpp:59-117) is reachable only from
 * its C++ API.  These entry points expose those fields, plus device-resident search
 * and per-stage timings.  All existing vesper.h symbols stay ABI-identical.
 */
#ifndef VESPER_B200_EXT_H
#define VESPER_B200_EXT_H

#include "vesper.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Full training parameters (IvfPqTrainParams, ivf_pq.hpp:59-106).  Set struct_size to
 * sizeof(vesper_ivfpq_train_params_ex_t); vesper_ivfpq_train_params_ex_init fills the
 * reference defaults. */
typedef struct vesper_ivfpq_train_params_ex_s {
  size_t struct_size;
  uint32_t nlist;
  uint32_t m;
  uint32_t nbits;
  uint32_t max_iter;       /* k-means iterations, default 25 */
  float epsilon;           /* k-means convergence threshold, default 1e-4 */
  int use_opq;             /* default 1 */
  uint32_t opq_iter;       /* default 10 (the alternation runs at most 3) */
  size_t opq_sample_n;     /* default 20000 */
  int opq_init_pca;        /* 1 = PCA (default), 0 = identity */
  uint32_t seed;           /* default 42 */
  int verbose;
} vesper_ivfpq_train_params_ex_t;

VESPER_C_API void vesper_ivfpq_train_params_ex_init(vesper_ivfpq_train_params_ex_t* p);

/* IvfPqIndex::train with every field of IvfPqTrainParams (ivf_pq.hpp:161-163). */
VESPER_C_API vesper_status_t vesper_ivfpq_train_ex(vesper_index_t* index, const float* base_vectors,
                                                   size_t dim, size_t n,
                                                   const vesper_ivfpq_train_params_ex_t* params);

/* vesper_ivfpq_train_ex / vesper_ivfpq_add with the input vectors (and ids) in device
 * memory of the index's GPU: no host staging of the data set. */
VESPER_C_API vesper_status_t vesper_ivfpq_train_ex_device(vesper_index_t* index, const float* d_base_vectors,
                                                          size_t dim, size_t n,
                                                          const vesper_ivfpq_train_params_ex_t* params);
VESPER_C_API vesper_status_t vesper_ivfpq_add_device(vesper_index_t* index, const uint64_t* d_ids,
                                                     const float* d_base_vectors, size_t n);

/* Report of the last train call: whether the OPQ rotation was kept and the two
 * reconstruction errors the keep/drop decision compared (ivf_pq.cpp:2730-2748). */
typedef struct vesper_ivfpq_train_report_s {
  int opq_kept;
  double err_unrot;
  double err_opq;
  uint32_t coarse_iterations;
  float train_time_sec;
} vesper_ivfpq_train_report_t;
VESPER_C_API vesper_status_t vesper_ivfpq_get_train_report(const vesper_index_t* index,
                                                           vesper_ivfpq_train_report_t* out);

/* Search arithmetic: FAST builds the lookup table once per query (distances equal the
 * exact ones to fp32 rounding); EXACT reproduces the reference's per-(query, list)
 * lookup tables and rotations operation for operation (bit-identical results). */
typedef enum vesper_search_mode_e { VESPER_SEARCH_FAST = 0, VESPER_SEARCH_EXACT = 1 } vesper_search_mode_t;

typedef struct vesper_ivfpq_search_params_ex_s {
  size_t struct_size;
  uint32_t k;              /* at most 1024 */
  uint32_t nprobe;         /* clamped to nlist, at most 1024 */
  uint32_t mode;           /* vesper_search_mode_t */
  /* IvfPqSearchParams (include/vesper/index/ivf_pq.hpp:109-117); read only when
   * struct_size covers them (callers built against the shorter struct get 0s). */
  uint32_t cand_k;           /* ADC candidate pool; 0 = k (matters only with the rerank) */
  uint32_t use_exact_rerank; /* 1: re-score the pool's head exactly (ivf_pq.cpp:3995-4091) */
  uint32_t rerank_k;         /* head size; 0 = the whole pool of max(k, cand_k, max(3k, 1000)) */
} vesper_ivfpq_search_params_ex_t;
/* struct_size of callers that predate cand_k / use_exact_rerank / rerank_k. */
#define VESPER_IVFPQ_SEARCH_PARAMS_EX_V1_SIZE (sizeof(size_t) + 3 * sizeof(uint32_t))

/* vesper_ivfpq_search_batch with a search mode; out_counts (may be NULL) receives the
 * number of real results per query (the rest of each row is padding). */
VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_ex(const vesper_index_t* index,
                                                          const float* queries, size_t nq,
                                                          const vesper_ivfpq_search_params_ex_t* params,
                                                          uint64_t* out_ids, float* out_distances,
                                                          uint32_t* out_counts);

/* Same, with queries and outputs in device memory of the index's GPU (no host copies). */
VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device(const vesper_index_t* index,
                                                              const float* d_queries, size_t nq,
                                                              const vesper_ivfpq_search_params_ex_t* params,
                                                              uint64_t* d_out_ids, float* d_out_distances,
                                                              uint32_t* d_out_counts);

/* Allocation-free variant of vesper_ivfpq_search_batch_device (FAST mode only).  This
 * entry point has no counterpart in the reference.  It is for callers that cannot let
 * the library allocate device memory: applications whose own arena or framework
 * allocator owns the GPU's memory, and latency-critical loops where cudaMalloc or
 * cudaFree -- which can synchronize the device -- must not run.  The caller passes the
 * queries and the outputs (device pointers on the index's GPU); all temporary buffers
 * come from one fixed 64 MiB device array compiled into the library, which every GPU
 * that loads the library holds until exit.  The first call on a device looks the
 * array's address up (make it before any stream capture).  Calls share the array and
 * are serialized by a process-wide lock, because calls overlapping on the GPU would
 * race on it.  Queries are processed in chunks that fit; an index whose single query
 * would need more than 64 MiB of scratch (nlist * 4 + m * 2^nbits * 4 + ... bytes) is
 * rejected with VESPER_ERROR_INVALID_PARAM and a message, as are mode EXACT and shapes
 * whose lookup table or top-k buffer exceed the kernels' shared memory; such a call
 * queues no GPU work.  The cached address belongs to the device's primary context:
 * after cudaDeviceReset on that device the entry point must not be called again in the
 * same process. */
VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device_noalloc(const vesper_index_t* index,
                                                                      const float* d_queries, size_t nq,
                                                                      const vesper_ivfpq_search_params_ex_t* params,
                                                                      uint64_t* d_out_ids, float* d_out_distances,
                                                                      uint32_t* d_out_counts);

/* The coarse stage alone: for each query the min(nprobe, nlist) nearest lists in the
 * search's probe order (d_probe uint32 [nq x np]) and their distances (d_probe_d float
 * [nq x np]); device pointers on the index's GPU.  No counterpart in the reference: with
 * vesper_ivfpq_search_batch_device_probed it lets several indexes that share a query
 * batch (one per GPU, each holding a shard of the base set) probe a slice of the batch
 * each and exchange the lists, instead of every GPU probing every query. */
VESPER_C_API vesper_status_t vesper_ivfpq_probe_device(const vesper_index_t* index, const float* d_queries,
                                                       size_t nq, uint32_t nprobe, uint32_t* d_probe,
                                                       float* d_probe_d);

/* vesper_ivfpq_search_batch_device with the probe lists given (as
 * vesper_ivfpq_probe_device writes them, for the same nprobe); results are those of the
 * plain call.  The exact rerank is not available here. */
VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device_probed(
    const vesper_index_t* index, const float* d_queries, size_t nq, const vesper_ivfpq_search_params_ex_t* params,
    const uint32_t* d_probe, const float* d_probe_d, uint64_t* d_out_ids, float* d_out_distances,
    uint32_t* d_out_counts);

/* Threshold exchange between the shards of one database.  No counterpart in the
 * reference (it has one index per process).  Several indexes, one per GPU, each hold a
 * part of the base set and search the same batch with the same parameters; with an
 * exchange set on each, every batch search (plain, device or probed; not the
 * allocation-free one) calls fn once per query chunk, on the calling thread, with d_tau
 * [n_queries] float on the index's device -- each query's upper bound of its k-th FAST
 * distance over this index's shard, +inf where it has none -- and the index's CUDA
 * stream (a cudaStream_t).  fn must leave the element-wise minimum over all shards in
 * d_tau, ordered on that stream (an all-reduce MIN issued on it), and return 0; any
 * other value fails the search with VESPER_ERROR_INVALID_PARAM.  The tensor-core list
 * scan then keeps only entries that can reach the shared bound, so each shard refines
 * about its share of the union's candidates; the union's top k (the per-shard results
 * merged) is unchanged.  Searches that do not run the list scan pass +inf for every
 * query, so the calls of all shards pair up.  fn must not call back into the index.
 * fn = NULL removes the exchange. */
typedef int (*vesper_ivfpq_tau_exchange_fn)(float* d_tau, size_t n_queries, void* cuda_stream, void* user);
/* shard / shards: with shards > 1 this index computes its own bounds only for the
 * queries q (0-based in the call's batch) with q % shards == shard and relies on the
 * exchange for the rest, so each of W shards pays 1/W of the threshold pass; give every
 * shard a different `shard` and the same `shards` (shards = 1: every query; shard must
 * be below shards). */
VESPER_C_API vesper_status_t vesper_ivfpq_set_threshold_exchange(vesper_index_t* index,
                                                                 vesper_ivfpq_tau_exchange_fn fn, void* user,
                                                                 uint32_t shard, uint32_t shards);

/* Merge of per-shard results on the device.  No counterpart in the reference (one
 * index per process).  For a database split across GPUs, each shard's batch search
 * returns per query up to k results sorted by distance (ids [nq x k], distances
 * [nq x k], counts [nq]); after an all-gather, part p's arrays start at d_dist +
 * p * dist_stride, d_ids + p * ids_stride and d_counts + p * counts_stride (strides in
 * elements of each array).  Writes per query the k smallest over all parts -- ties to
 * the lower part, then the earlier slot -- with slots past d_out_counts[q] padded like
 * vesper_ivfpq_search_batch (id 0, the last distance).  d_out_counts may be NULL.
 * 1 <= parts <= 64.  Device pointers; the kernel is queued on cuda_stream (a
 * cudaStream_t, NULL = the legacy default stream) and the call does not wait for it. */
VESPER_C_API vesper_status_t vesper_topk_merge_device(uint32_t parts, size_t nq, uint32_t k, const float* d_dist,
                                                     size_t dist_stride, const uint64_t* d_ids, size_t ids_stride,
                                                     const uint32_t* d_counts, size_t counts_stride,
                                                     uint64_t* d_out_ids, float* d_out_distances,
                                                     uint32_t* d_out_counts, void* cuda_stream);

/* ---------------------------------------------------------------------------------
 * The rest of IvfPqIndex's API (include/vesper/index/ivf_pq.hpp:252-386), which the
 * reference reaches from C++ only.  Vectors are rebuilt exactly as the reference does:
 * centroid + apply_rotation_T(decode(code)); an id held by several entries resolves to
 * the first one in list order.  Errors: VESPER_ERROR_NOT_TRAINED before training,
 * VESPER_ERROR_INVALID_PARAM with the reference's message otherwise ("Vector ID not
 * found", "Cluster ID out of range", ...).
 * ------------------------------------------------------------------------------- */
VESPER_C_API vesper_status_t vesper_ivfpq_reconstruct(const vesper_index_t* index, uint64_t id,
                                                      float* out_vector /* [dim] */);
/* Entries of a cluster in list order: *out_count receives their number; ids and vectors
 * are written when capacity (entries) suffices, else VESPER_ERROR_INVALID_PARAM. */
VESPER_C_API vesper_status_t vesper_ivfpq_reconstruct_cluster(const vesper_index_t* index, uint32_t cluster_id,
                                                              uint64_t* out_ids, float* out_vectors,
                                                              size_t capacity, size_t* out_count);
VESPER_C_API vesper_status_t vesper_ivfpq_get_cluster_assignment(const vesper_index_t* index, uint64_t id,
                                                                 uint32_t* out_cluster);
VESPER_C_API vesper_status_t vesper_ivfpq_get_cluster_centroid(const vesper_index_t* index, uint32_t cluster_id,
                                                               float* out_centroid /* [dim] */);
VESPER_C_API vesper_status_t vesper_ivfpq_update_cluster_centroid(vesper_index_t* index, uint32_t cluster_id,
                                                                  const float* centroid /* [dim] */);
VESPER_C_API vesper_status_t vesper_ivfpq_reassign_vector(vesper_index_t* index, uint64_t id, uint32_t new_cluster);
/* compact_inverted_list: removes the cluster's entries whose id, cut to 32 bits, is in
 * deleted_ids (the reference takes a roaring bitmap of 32-bit ids). */
VESPER_C_API vesper_status_t vesper_ivfpq_compact_inverted_list(vesper_index_t* index, uint32_t cluster_id,
                                                                const uint32_t* deleted_ids, size_t n_deleted,
                                                                size_t* out_removed);
/* debug_explain_centroid_rank / debug_explain_adc_rank (VESPER_IVFPQ_DEBUG=1 required, as
 * in the reference): rank = 1 + the number of centroids (entries) strictly closer. */
VESPER_C_API vesper_status_t vesper_ivfpq_debug_explain_centroid_rank(const vesper_index_t* index,
                                                                      const float* query, uint64_t target_id,
                                                                      uint64_t* out_rank, uint32_t* out_cluster);
VESPER_C_API vesper_status_t vesper_ivfpq_debug_explain_adc_rank(const vesper_index_t* index, const float* query,
                                                                 uint64_t target_id, uint64_t* out_rank,
                                                                 float* out_distance);

/* Device time per stage of the last search call (CUDA events, milliseconds). */
typedef struct vesper_ivfpq_timings_s {
  float coarse_ms;   /* query-centroid distances */
  float select_ms;   /* top-nprobe selection */
  float rotate_ms;   /* OPQ rotation of queries / residuals */
  float scan_ms;     /* lookup tables + inverted-list scan + per-list top-k */
  float merge_ms;    /* per-query merge (EXACT mode) */
  float total_ms;
  uint64_t scanned_entries; /* sum over queries of the probed lists' sizes */
  uint32_t kernel_launches; /* kernels launched by the call */
  uint32_t scan_variant;    /* 1 exact per-(query, list) tables, 2 per-query tables, 3 blocked layout,
                               4 tensor-core list scan (bf16 screen + exact FAST refine) */
  uint32_t coarse_variant;  /* 1 CUDA-core exact distances, 2 tensor-core screen + exact refine, 3 tensor-core filter against a sampled threshold + exact refine */
  float list_kernel_ms;     /* variant 4: device time of the tensor-core screening kernel */
  uint64_t list_candidates; /* variant 4: (query, entry) pairs the screen kept */
  uint32_t list_fallback_queries; /* variant 4: queries scanned by the blocked scan instead */
  float list_threshold_ms;  /* variant 4: nearest-list scan that gives the screen thresholds */
  float list_prep_ms;       /* variant 4: bf16 queries, pair grouping by list, unit table */
  float list_refine_ms;     /* variant 4: exact FAST re-scoring of the kept pairs */
  float list_fallback_ms;   /* variant 4: blocked scan of queries whose candidates overflowed */
  float rerank_ms;          /* exact rerank of the candidate pool (use_exact_rerank) */
} vesper_ivfpq_timings_t;
VESPER_C_API vesper_status_t vesper_ivfpq_get_last_timings(const vesper_index_t* index,
                                                           vesper_ivfpq_timings_t* out);

/* Install a trained model (centroids [nlist x dim], codebooks [m * 2^nbits x dim/m],
 * rotation [dim x dim] or NULL) and empty the lists.  Used to search or add with a
 * model trained elsewhere, e.g. by the reference CPU implementation. */
VESPER_C_API vesper_status_t vesper_ivfpq_set_model(vesper_index_t* index, size_t dim, uint32_t nlist,
                                                    uint32_t m, uint32_t nbits, const float* centroids,
                                                    const float* codebooks, const float* rotation);

/* Copy out the inverted lists: offsets [nlist + 1], ids [n_vectors], codes
 * [n_vectors x m], entries list-contiguous in insertion order.  Any pointer may be NULL. */
VESPER_C_API vesper_status_t vesper_ivfpq_get_lists(const vesper_index_t* index, uint64_t* out_offsets,
                                                    uint64_t* out_ids, uint8_t* out_codes);

/* k-means on the GPU of the calling thread's current device.  The reference reaches
 * k-means from C++ only -- kmeans_cluster (src/index/kmeans.cpp:137-252) and
 * KmeansElkan::cluster (src/index/kmeans_elkan.cpp:293-430) -- so these entry points
 * have no C counterpart there; they take the fields of KmeansParams
 * (include/vesper/index/kmeans.hpp:26-36) that the two functions read.
 * Both algorithms start from the reference's k-means++ (kmeans.cpp:45-89, same
 * std::mt19937 draws) and produce the same assignments and centroids:
 *   ELKAN  convergence test on the inertia of the current assignment, Kahan fp64 mean
 *          x (1/count), a point keeps its centroid on a distance tie; result.inertia is
 *          the inertia the loop stopped at (the reference's return value);
 *   LLOYD  one run of kmeans_cluster (n_redo = 1): lowest index wins a tie, fp64 sum /
 *          count, and after the loop one more mean update and the inertia of the final
 *          assignment, the reference's float running total over every (point,
 *          dimension) term in order.
 * Errors as the reference: k == 0 or n < k -> VESPER_ERROR_INVALID_PARAM with its message. */
typedef enum vesper_kmeans_algorithm_e { VESPER_KMEANS_ELKAN = 0, VESPER_KMEANS_LLOYD = 1 } vesper_kmeans_algorithm_t;

typedef struct vesper_kmeans_params_s {
  size_t struct_size;      /* sizeof(vesper_kmeans_params_t) */
  uint32_t k;
  uint32_t max_iter;       /* default 25 */
  float epsilon;           /* default 1e-4 */
  uint32_t seed;           /* default 42 */
  uint32_t algorithm;      /* vesper_kmeans_algorithm_t, default ELKAN */
} vesper_kmeans_params_t;

typedef struct vesper_kmeans_result_s {
  uint32_t iterations;
  float inertia;
  float time_sec;          /* wall time of the call */
} vesper_kmeans_result_t;

VESPER_C_API void vesper_kmeans_params_init(vesper_kmeans_params_t* p);

/* data [n x dim] host; out_centroids [k x dim] host; out_assignments [n] host or NULL;
 * out_result may be NULL. */
VESPER_C_API vesper_status_t vesper_kmeans_fit(const float* data, size_t n, size_t dim,
                                               const vesper_kmeans_params_t* params, float* out_centroids,
                                               uint32_t* out_assignments, vesper_kmeans_result_t* out_result);

/* Same with data, centroids and assignments in device memory of the current device.
 * The inputs must be complete when the call starts (it does not order itself after
 * work queued on the caller's streams); the outputs are complete when it returns. */
VESPER_C_API vesper_status_t vesper_kmeans_fit_device(const float* d_data, size_t n, size_t dim,
                                                      const vesper_kmeans_params_t* params, float* d_out_centroids,
                                                      uint32_t* d_out_assignments, vesper_kmeans_result_t* out_result);

/* k-means over points sharded across GPUs (one process per GPU).  The building blocks
 * of the fit above, for a driver that owns the collectives (vesper_db_b200.shard
 * .kmeans_fit_sharded runs them over torch.distributed / NCCL).  Points are split into
 * contiguous shards in point order; centroids are replicated.  Per iteration every
 * shard assigns its own points (vesper_kmeans_shard_assign), the per-point distances
 * are gathered for the fp64 inertia in point order, and the mean update runs as a
 * chain in shard order: each shard continues the (sum, Kahan compensation, count)
 * state the previous shard left (vesper_kmeans_shard_accumulate, state [k x dim] f64,
 * [k x dim] f64, [k] u64, zero before the first shard) and the last one turns it into
 * centroids (vesper_kmeans_shard_finish), which are then broadcast.  The chain keeps
 * the reference's sums in point order, so the sharded fit equals the one-GPU fit bit
 * for bit.  k-means++ draws use vesper_kmeanspp_sampler_* on the gathered D^2 vector.
 * All pointers but the sampler's d2 are device memory of the handle's device; every
 * call's outputs are complete when it returns, and its inputs must be complete when
 * it starts. */
typedef struct vesper_kmeans_shard_s vesper_kmeans_shard_t;

/* A handle on the calling thread's current device (own stream and scratch). */
VESPER_C_API vesper_status_t vesper_kmeans_shard_create(vesper_kmeans_shard_t** out);
VESPER_C_API void vesper_kmeans_shard_destroy(vesper_kmeans_shard_t* shard);
/* Nearest centroid of each of the n rows of x (reference lane order; the lowest index
 * wins a tie, or, with keep_on_tie, the current d_assign entry does).  d_min_dist may
 * be NULL. */
VESPER_C_API vesper_status_t vesper_kmeans_shard_assign(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                        size_t dim, const float* d_centroids, uint32_t k,
                                                        int keep_on_tie, uint32_t* d_assign, float* d_min_dist);
/* k-means++ D^2 refresh: d_min_dist[i] = min(d_min_dist[i], l2(x_i, centroid)). */
VESPER_C_API vesper_status_t vesper_kmeans_shard_pp_update(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                           size_t dim, const float* d_centroid, float* d_min_dist);
/* This shard's part of the mean update (algorithm: ELKAN = Kahan, LLOYD = plain sum). */
VESPER_C_API vesper_status_t vesper_kmeans_shard_accumulate(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                            size_t dim, const uint32_t* d_assign, uint32_t k,
                                                            uint32_t algorithm, double* d_sum, double* d_comp,
                                                            uint64_t* d_count);
/* Centroids from the final state; a cluster with count 0 keeps its centroid. */
VESPER_C_API vesper_status_t vesper_kmeans_shard_finish(vesper_kmeans_shard_t* shard, const double* d_sum,
                                                        const uint64_t* d_count, uint32_t k, size_t dim,
                                                        uint32_t algorithm, float* d_centroids);
/* LLOYD's final inertia (kmeans.cpp:230-241), a float running total over every
 * (point, dimension) term (x - c)^2 in point order: *inout_total (host) is continued
 * over this shard's points.  Start from 0 on the first shard and pass the total along
 * in shard order. */
VESPER_C_API vesper_status_t vesper_kmeans_shard_running_inertia(vesper_kmeans_shard_t* shard, const float* d_x,
                                                                 size_t n, size_t dim, const float* d_centroids,
                                                                 const uint32_t* d_assign, float* inout_total);

/* The k-means++ draws of kmeans_plusplus_init (src/index/kmeans.cpp:45-89) for n points:
 * create returns the first row; next takes the D^2 value of every point (host, n
 * floats, point order) and returns the next row. */
typedef struct vesper_kmeanspp_sampler_s vesper_kmeanspp_sampler_t;
VESPER_C_API vesper_status_t vesper_kmeanspp_sampler_create(uint32_t seed, size_t n, vesper_kmeanspp_sampler_t** out,
                                                            size_t* first_index);
VESPER_C_API vesper_status_t vesper_kmeanspp_sampler_next(vesper_kmeanspp_sampler_t* sampler, const float* d2,
                                                          size_t* index);
VESPER_C_API void vesper_kmeanspp_sampler_destroy(vesper_kmeanspp_sampler_t* sampler);

/* ---------------------------------------------------------------------------------
 * Exact flat top-k: find_nearest_centroids_batch_fused
 * (include/vesper/kernels/batch_distances.hpp:338-456), which the reference calls from
 * C++ only.  For each of nq queries the k_eff = min(k, n_base) best base vectors:
 *   VESPER_FLAT_L2  squared L2 (avx2_l2_sq lane order), smallest first;
 *   VESPER_FLAT_IP  inner product (avx2_inner_product lane order), largest first;
 * equal scores go to the smaller index.  Row q of out_indices / out_scores holds k
 * entries; entries k_eff..k-1 (only when k > n_base) are index 0xffffffff with score
 * FLT_MAX (L2) or -FLT_MAX (IP) -- the reference leaves them undefined.
 * Limits: k <= 1024, dim a multiple of 4 and >= 32, n_base < 2^31.
 * ------------------------------------------------------------------------------- */
typedef enum vesper_flat_op_e { VESPER_FLAT_L2 = 0, VESPER_FLAT_IP = 1 } vesper_flat_op_t;

typedef struct vesper_flat_timings_s {
  float total_ms;          /* device time of the call (norms to results) */
  float norms_ms;          /* row norms */
  float sample_ms;         /* pass 1 (screen + exact top-k over a strided sample); the
                              whole search when single_pass */
  float filter_ms;         /* pass 2 tensor-core screen over the whole base */
  float refine_ms;         /* pass 2 exact re-scoring and selection */
  float fallback_ms;       /* queries whose kept-column list overflowed */
  uint64_t candidates;     /* kept columns, all queries (pass 2) */
  uint32_t overflow_queries;
  uint32_t sample_stride;
  uint32_t single_pass;    /* 1: base small enough for one screen + select */
  uint32_t kernel_launches; /* kernels the call launched */
} vesper_flat_timings_t;

/* queries [nq x dim], base [n_base x dim] host; outputs [nq x k] host. */
VESPER_C_API vesper_status_t vesper_flat_topk(vesper_flat_op_t op, const float* queries, size_t nq,
                                              const float* base, size_t n_base, size_t dim, uint32_t k,
                                              uint32_t* out_indices, float* out_scores);

/* Same with all arrays in device memory of the current device (16-byte aligned); the
 * outputs are complete when the call returns. */
VESPER_C_API vesper_status_t vesper_flat_topk_device(vesper_flat_op_t op, const float* d_queries, size_t nq,
                                                     const float* d_base, size_t n_base, size_t dim, uint32_t k,
                                                     uint32_t* d_out_indices, float* d_out_scores);

/* Stage times of this thread's last vesper_flat_topk[_device] call. */
VESPER_C_API vesper_status_t vesper_flat_get_last_timings(vesper_flat_timings_t* out);

/* Number of CUDA devices visible to the library. */
VESPER_C_API int vesper_b200_device_count(void);

/* ---------------------------------------------------------------------------------
 * IndexManager (include/vesper_manager.h): the search mode its IVF-PQ searches use,
 * VESPER_SEARCH_FAST (default) or VESPER_SEARCH_EXACT (the reference's arithmetic). */
typedef struct vesper_manager_t vesper_manager_t;
VESPER_C_API vesper_status_t vesper_mgr_set_search_mode(vesper_manager_t* mgr, uint32_t mode);

#ifdef __cplusplus
}
#endif

#endif /* VESPER_B200_EXT_H */
