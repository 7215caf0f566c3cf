// Oracle: a CPU restatement of the reference IVF-PQ / k-means arithmetic.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU-baseline
// leg of bench.py may load liboracle.so, and only as the checker.  The product path
// (vesper_db_b200/) never links or calls it.
//
// Parity is pinned: tests/test_oracle_pin.py checks every function here bit-for-bit
// against the reference sources compiled in place (oracle/_ref/libvesper_ref_nc.so,
// built with -ffp-contract=off) and against the reference's golden fixtures
// (algorithms/fixtures/pq/pq_lut_small.json, distance_kernels/l2_ip_small.json)
// committed as tests/golden/*.json.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float orc_l2_sq(const float* a, const float* b, size_t n);
float orc_inner_product(const float* a, const float* b, size_t n);

void orc_assign(const float* x, size_t n, const float* c, uint32_t k, size_t dim, uint32_t* out,
                float* out_dist);
void orc_coarse_probe(const float* q, size_t nq, const float* c, uint32_t nlist, size_t dim,
                      uint32_t nprobe, uint32_t* out_lists, float* out_d);
void orc_rotate(const float* in, const float* R, size_t n, size_t dim, float* out);
void orc_rotate_T(const float* in, const float* R, size_t n, size_t dim, float* out);
void orc_pq_encode(const float* x, size_t n, const float* cb, uint32_t m, uint32_t ksub,
                   size_t dsub, uint8_t* codes);
void orc_pq_decode(const uint8_t* codes, size_t n, const float* cb, uint32_t m, uint32_t ksub,
                   size_t dsub, float* out);
void orc_pq_lut(const float* r, const float* cb, uint32_t m, uint32_t ksub, size_t dsub,
                float* lut);
float orc_adc(const float* lut, const uint8_t* code, uint32_t m, uint32_t ksub);

void orc_ivfpq_add(const float* x, size_t n, const float* c, uint32_t nlist, size_t dim,
                   const float* R, const float* cb, uint32_t m, uint32_t ksub,
                   uint32_t* out_assign, uint8_t* out_codes);

uint32_t orc_ivfpq_search(const float* q, const float* c, uint32_t nlist, size_t dim,
                          const float* R, const float* cb, uint32_t m, uint32_t ksub,
                          const uint64_t* list_offsets, const uint64_t* ids,
                          const uint8_t* codes, uint32_t k, uint32_t nprobe, uint64_t* out_ids,
                          float* out_d);
void orc_ivfpq_search_batch(const float* q, size_t nq, const float* c, uint32_t nlist,
                            size_t dim, const float* R, const float* cb, uint32_t m,
                            uint32_t ksub, const uint64_t* list_offsets, const uint64_t* ids,
                            const uint8_t* codes, uint32_t k, uint32_t nprobe, uint64_t* out_ids,
                            float* out_d, uint32_t* out_counts);

void orc_ivfpq_search_batch_ex(const float* q, size_t nq, const float* c, uint32_t nlist,
                               size_t dim, const float* R, const float* cb, uint32_t m,
                               uint32_t ksub, const uint64_t* list_offsets, const uint64_t* ids,
                               const uint8_t* codes, uint32_t k, uint32_t nprobe, uint32_t cand_k,
                               int rerank, uint32_t rerank_k, uint64_t* out_ids, float* out_d,
                               uint32_t* out_counts);

void orc_flat_topk(int op, const float* q, size_t nq, const float* base, uint32_t nb,
                   size_t dim, uint32_t k, uint32_t* out_idx, float* out_score);

void orc_kmeanspp_init(const float* x, size_t n, size_t dim, uint32_t k, uint32_t seed,
                       float* out_c, uint32_t* out_idx);
float orc_lloyd_assign(const float* x, size_t n, const float* c, uint32_t k, size_t dim,
                       uint32_t* out);
void orc_lloyd_update(const float* x, size_t n, size_t dim, const uint32_t* assign, uint32_t k,
                      float* c_inout);
void orc_elkan_update_centroid(const float* x, size_t dim, const uint32_t* assign, size_t n,
                               uint32_t k, float* c_inout);
int orc_kmeans_elkan(const float* x, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                     float eps, uint32_t seed, float* out_c, uint32_t* out_assign,
                     uint32_t* out_iters, float* out_inertia);
int orc_kmeans_lloyd(const float* x, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                     float eps, uint32_t seed, float* out_c, uint32_t* out_assign,
                     uint32_t* out_iters, float* out_inertia);
int orc_pq_train(const float* x, size_t n, size_t dim, uint32_t m, uint32_t nbits, float* out_cb);

#ifdef __cplusplus
}
#endif
