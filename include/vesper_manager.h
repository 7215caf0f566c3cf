/*
 * The reference's IndexManager C ABI (include/vesper/c/vesper_manager.h) served by the
 * B200 IVF-PQ engine.  Names, enum values and struct layouts are the reference's, so a
 * program compiled against its header links against libvesper_c.so unchanged.
 *
 * What the manager routes here: the IVF-PQ index (build, add, update, remove via
 * tombstones, search with the reference's cand_k / rerank heuristics and tombstone
 * oversampling, save/load in the reference's directory layout).  HNSW and DiskANN
 * indexes are not part of this engine: building, preferring or loading one is
 * refused or yields no results, as each entry point below states.
 */
#ifndef VESPER_MANAGER_H
#define VESPER_MANAGER_H

#include <stddef.h>
#include <stdint.h>

#include "vesper.h"

#ifdef __cplusplus
extern "C" {
#endif

/* vesper_manager.h:13-23 */
typedef enum vesper_index_type_e {
  VESPER_INDEX_HNSW = 0,
  VESPER_INDEX_IVF_PQ = 1,
  VESPER_INDEX_DISKANN = 2
} vesper_index_type_t;

typedef enum vesper_selection_strategy_e {
  VESPER_SELECT_AUTO = 0,
  VESPER_SELECT_MANUAL = 1,
  VESPER_SELECT_HYBRID = 2
} vesper_selection_strategy_t;

/* vesper_manager.h:26 */
typedef struct vesper_manager_t vesper_manager_t;

/* vesper_manager.h:29-47 */
typedef struct vesper_hnsw_build_params_s {
  uint32_t M;
  uint32_t ef_construction;
  uint32_t seed;
} vesper_hnsw_build_params_t;

typedef struct vesper_vamana_build_params_s {
  uint32_t degree;
  uint32_t L;
  float    alpha;
} vesper_vamana_build_params_t;

typedef struct vesper_manager_build_config_s {
  vesper_index_type_t          type;
  vesper_selection_strategy_t  strategy;
  vesper_ivfpq_train_params_t  ivf;
  vesper_hnsw_build_params_t   hnsw;
  vesper_vamana_build_params_t vamana;
} vesper_manager_build_config_t;

/* vesper_manager.h:49-65 */
typedef struct vesper_query_config_s {
  uint32_t k;
  float    epsilon;
  uint32_t ef_search;
  uint32_t nprobe;                  /* 0 -> 8 */
  uint32_t l_search;
  int      use_exact_rerank;
  uint32_t rerank_k;
  float    rerank_alpha;
  uint32_t rerank_cand_ceiling;
  int      use_query_planner;
  int      has_preferred_index;
  vesper_index_type_t preferred_index;
  int      has_filter;
  const char* filter_json;
} vesper_query_config_t;

/* vesper_manager.h:67-76 */
typedef struct vesper_index_stats_s {
  vesper_index_type_t type;
  size_t  num_vectors;
  size_t  memory_usage_bytes;
  size_t  disk_usage_bytes;
  float   build_time_seconds;
  float   avg_query_time_ms;
  float   measured_recall;
  uint64_t query_count;
} vesper_index_stats_t;

/* vesper_manager.h:79-80 (IndexManager(dim), src/index/index_manager.cpp:142-160) */
VESPER_C_API vesper_status_t vesper_mgr_create(size_t dim, vesper_manager_t** out_mgr);
VESPER_C_API vesper_status_t vesper_mgr_destroy(vesper_manager_t* mgr);

/* vesper_manager.h:82-83 (index_manager.cpp:187-241, 1682-1770).  MANUAL builds cfg->type;
 * AUTO and HYBRID build the IVF-PQ index (the reference may pick HNSW or DiskANN there).
 * IVF-PQ is trained on at most 200 000 evenly spaced rows with the reference's defaults
 * for zero nlist / m / nbits outside MANUAL, then every row is added with id = row.
 * MANUAL with HNSW or DiskANN -> VESPER_ERROR_INVALID_PARAM ("... not available"). */
VESPER_C_API vesper_status_t vesper_mgr_build(vesper_manager_t* mgr,
  const float* base_vectors, size_t n, const vesper_manager_build_config_t* cfg);

/* vesper_manager.h:85-86 (index_manager.cpp:289-341) */
VESPER_C_API vesper_status_t vesper_mgr_add_batch(vesper_manager_t* mgr,
  const uint64_t* ids, const float* vectors, size_t n);

/* vesper_manager.h:89-92 (index_manager.cpp:612-821).  update adds a new entry under the
 * id (the old entry stays, as in the reference); remove marks (uint32_t)id deleted and
 * fails if it already is. */
VESPER_C_API vesper_status_t vesper_mgr_update(vesper_manager_t* mgr, uint64_t id, const float* vector);
VESPER_C_API vesper_status_t vesper_mgr_update_batch(vesper_manager_t* mgr, const uint64_t* ids, const float* vectors, size_t n);
VESPER_C_API vesper_status_t vesper_mgr_remove(vesper_manager_t* mgr, uint64_t id);
VESPER_C_API vesper_status_t vesper_mgr_remove_batch(vesper_manager_t* mgr, const uint64_t* ids, size_t n);

/* vesper_manager.h:95-100 (index_manager.cpp:344-602).  out_ids / out_dists hold k per
 * query, padded past the real results with id 0 and the last real distance (0 if none).
 * A whole batch runs as one GPU search.  has_filter with a non-NULL filter_json ->
 * VESPER_ERROR_INVALID_PARAM (metadata filters are not part of this engine). */
VESPER_C_API vesper_status_t vesper_mgr_search(const vesper_manager_t* mgr,
  const float* query, const vesper_query_config_t* qc,
  uint64_t* out_ids, float* out_dists);
VESPER_C_API vesper_status_t vesper_mgr_search_batch(const vesper_manager_t* mgr,
  const float* queries, size_t nq, const vesper_query_config_t* qc,
  uint64_t* out_ids, float* out_dists);

/* vesper_manager.h:104-105 (index_manager.cpp:1100-1346): <dir>/index_manager.manifest,
 * <dir>/ivf_pq/ivfpq.bin, <dir>/tombstones.bin, byte-compatible with the reference. */
VESPER_C_API vesper_status_t vesper_mgr_save(const vesper_manager_t* mgr, const char* dir_path);
VESPER_C_API vesper_status_t vesper_mgr_load(vesper_manager_t* mgr, const char* dir_path);

/* vesper_manager.h:108-109 (index_manager.cpp:1348-1373): the reference's estimates. */
VESPER_C_API vesper_status_t vesper_mgr_memory_usage(const vesper_manager_t* mgr, size_t* out_bytes);
VESPER_C_API vesper_status_t vesper_mgr_disk_usage(const vesper_manager_t* mgr, size_t* out_bytes);

/* vesper_manager.h:112-113 (index_manager.cpp:1375-1388, 1444-1600): a budget below the
 * IVF-PQ estimate evicts the index, as the reference's enforcement does. */
VESPER_C_API vesper_status_t vesper_mgr_set_memory_budget_mb(vesper_manager_t* mgr, uint32_t mb);
VESPER_C_API vesper_status_t vesper_mgr_get_memory_budget_mb(const vesper_manager_t* mgr, uint32_t* out_mb);

/* vesper_manager.h:116-117 */
VESPER_C_API vesper_status_t vesper_mgr_get_stats(const vesper_manager_t* mgr,
  vesper_index_stats_t* out_stats, size_t* inout_capacity, size_t* out_count);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VESPER_MANAGER_H */
