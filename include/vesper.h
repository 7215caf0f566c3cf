/* Vesper IVF-PQ C ABI, B200 implementation (libvesper_c.so).
 *
 * Drop-in for the reference's include/vesper/c/vesper.h: the same types, the same
 * symbols, the same status codes and the same output conventions, so a caller linked
 * against the reference's libvesper_c.so relinks against this library unchanged.
 * Each declaration cites the reference declaration it replaces.
 *
 * Semantics kept from the reference implementation (src/c/vesper_c_api.cpp):
 *   - NULL arguments return VESPER_ERROR_INVALID_PARAM without touching the last error.
 *   - Errors reported by train / add / search return VESPER_ERROR_INVALID_PARAM with a
 *     message; save / load errors return VESPER_ERROR_IO; internal failures (CUDA
 *     errors) VESPER_ERROR_INTERNAL.  The last error is thread-local.
 *   - Results are squared L2 distances, ascending; when fewer than k results exist the
 *     ids are padded with 0 and the distances with the last valid distance (or 0).
 *   - vesper_ivfpq_train uses the reference defaults for every field the C struct does
 *     not carry (use_opq = 1 with PCA init, max_iter 25, epsilon 1e-4, seed 42).
 *
 * The index lives on the CUDA device that is current when vesper_ivfpq_create is
 * called; host buffers are copied to and from it inside each call.
 */
#ifndef VESPER_B200_VESPER_H
#define VESPER_B200_VESPER_H

#ifdef __cplusplus
extern "C" {
#endif

#define VESPER_C_API __attribute__((visibility("default")))

#include <stddef.h>
#include <stdint.h>

/* vesper.h:22 */
typedef struct vesper_index_t vesper_index_t;

/* vesper.h:24-31 */
typedef enum vesper_status_e {
  VESPER_OK = 0,
  VESPER_ERROR_UNKNOWN = 1,
  VESPER_ERROR_INVALID_PARAM = 2,
  VESPER_ERROR_NOT_TRAINED = 3,
  VESPER_ERROR_IO = 4,
  VESPER_ERROR_INTERNAL = 5
} vesper_status_t;

/* vesper.h:34 */
VESPER_C_API const char* vesper_get_last_error(void);
/* vesper.h:37 */
VESPER_C_API const char* vesper_version(void);

/* vesper.h:43-47 */
typedef struct vesper_ivfpq_train_params_s {
  uint32_t nlist;
  uint32_t m;
  uint32_t nbits;
} vesper_ivfpq_train_params_t;

/* vesper.h:49-52 */
typedef struct vesper_ivfpq_search_params_s {
  uint32_t k;
  uint32_t nprobe;
} vesper_ivfpq_search_params_t;

/* vesper.h:55-61 */
typedef struct vesper_ivfpq_stats_s {
  size_t n_vectors;
  size_t n_lists;
  size_t m;
  size_t memory_bytes;
  float  avg_list_size;
} vesper_ivfpq_stats_t;

/* vesper.h:64-65 */
VESPER_C_API vesper_status_t vesper_ivfpq_create(vesper_index_t** out_index);
VESPER_C_API vesper_status_t vesper_ivfpq_destroy(vesper_index_t* index);

/* vesper.h:68-73 */
VESPER_C_API vesper_status_t vesper_ivfpq_train(vesper_index_t* index, const float* base_vectors,
                                                size_t dim, size_t n,
                                                const vesper_ivfpq_train_params_t* params);

/* vesper.h:76-80 */
VESPER_C_API vesper_status_t vesper_ivfpq_add(vesper_index_t* index, const uint64_t* ids,
                                              const float* base_vectors, size_t n);

/* vesper.h:83-88 */
VESPER_C_API vesper_status_t vesper_ivfpq_search(const vesper_index_t* index, const float* query,
                                                 const vesper_ivfpq_search_params_t* params,
                                                 uint64_t* out_ids, float* out_distances);

/* vesper.h:91-97 */
VESPER_C_API vesper_status_t vesper_ivfpq_search_batch(const vesper_index_t* index,
                                                       const float* queries, size_t nq,
                                                       const vesper_ivfpq_search_params_t* params,
                                                       uint64_t* out_ids, float* out_distances);

/* vesper.h:100-102 */
VESPER_C_API vesper_status_t vesper_ivfpq_is_trained(const vesper_index_t* index, int* out_is_trained);
VESPER_C_API vesper_status_t vesper_ivfpq_get_dimension(const vesper_index_t* index, size_t* out_dim);
VESPER_C_API vesper_status_t vesper_ivfpq_get_stats(const vesper_index_t* index,
                                                    vesper_ivfpq_stats_t* out_stats);

/* vesper.h:105-108 */
VESPER_C_API vesper_status_t vesper_ivfpq_set_metadata_json(vesper_index_t* index, const char* json_str);
VESPER_C_API vesper_status_t vesper_ivfpq_get_metadata_json(const vesper_index_t* index,
                                                            char* out_buffer, size_t buffer_size,
                                                            size_t* out_required_size);

/* vesper.h:111-117: <file_path> is a directory; the index is <file_path>/ivfpq.bin (v1.0). */
VESPER_C_API vesper_status_t vesper_ivfpq_save(const vesper_index_t* index, const char* file_path);
VESPER_C_API vesper_status_t vesper_ivfpq_load(vesper_index_t* index, const char* file_path);

#ifdef __cplusplus
}
#endif

#endif /* VESPER_B200_VESPER_H */
