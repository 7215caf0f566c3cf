// Test-infrastructure bridge: a flat extern "C" surface over the reference's own
// C++ IVF-PQ, FastScanPq, k-means and fused top-k code, so the Python tests and the
// CPU-baseline leg of bench.py can call the reference implementation through ctypes.
//
// Linked only into oracle/_ref/libvesper_ref*.so together with the reference
// translation units compiled in place.  Nothing in the product links this file.
//
// Every function forwards to the reference API it names; the only logic here is
// argument marshalling (flat arrays <-> std::vector) and error capture.

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "vesper/index/ivf_pq.hpp"
#include "vesper/index/kmeans.hpp"
#include "vesper/index/kmeans_elkan.hpp"
#include "vesper/index/pq_fastscan.hpp"
#include "vesper/kernels/batch_distances.hpp"
#include "vesper/kernels/dispatch.hpp"

using namespace vesper;
using namespace vesper::index;

namespace {
thread_local std::string g_err;
void set_err(const std::string& s) { g_err = s; }
}  // namespace

extern "C" {

const char* rb_last_error(void) { return g_err.c_str(); }

// ---------------------------------------------------------------- distances
// kernels/dispatch.hpp:16-29 select_backend_auto() -> l2_sq / inner_product
float rb_l2_sq(const float* a, const float* b, size_t n) {
    const auto& ops = kernels::select_backend_auto();
    return ops.l2_sq(std::span(a, n), std::span(b, n));
}
float rb_inner_product(const float* a, const float* b, size_t n) {
    const auto& ops = kernels::select_backend_auto();
    return ops.inner_product(std::span(a, n), std::span(b, n));
}

// ---------------------------------------------------------------- IVF-PQ index
struct RbIndex { IvfPqIndex idx; };

void* rb_ivfpq_create(void) { return new RbIndex(); }
void rb_ivfpq_destroy(void* h) { delete static_cast<RbIndex*>(h); }

// IvfPqIndex::train (ivf_pq.hpp:161) with the parameters the C ABI hides.
// brute_assign=1 selects CoarseAssigner::Brute with use_centroid_ann=false,
// i.e. the brute-force add() branch (src/index/ivf_pq.cpp:3252-3265).
int rb_ivfpq_train(void* h, const float* data, size_t dim, size_t n, uint32_t nlist,
                   uint32_t m, uint32_t nbits, int use_opq, int brute_assign,
                   uint32_t max_iter, float epsilon, uint32_t seed, size_t opq_sample_n,
                   uint32_t opq_iter) {
    IvfPqTrainParams p;
    p.nlist = nlist; p.m = m; p.nbits = nbits;
    p.use_opq = use_opq != 0;
    p.max_iter = max_iter; p.epsilon = epsilon; p.seed = seed;
    p.opq_sample_n = opq_sample_n; p.opq_iter = opq_iter;
    if (brute_assign) { p.coarse_assigner = CoarseAssigner::Brute; p.use_centroid_ann = false; }
    try {
        auto r = static_cast<RbIndex*>(h)->idx.train(data, dim, n, p);
        if (!r) { set_err(r.error().message); return 2; }
        return 0;
    } catch (const std::exception& e) { set_err(e.what()); return 5; }
}

int rb_ivfpq_add(void* h, const uint64_t* ids, const float* data, size_t n) {
    try {
        auto r = static_cast<RbIndex*>(h)->idx.add(ids, data, n);
        if (!r) { set_err(r.error().message); return 2; }
        return 0;
    } catch (const std::exception& e) { set_err(e.what()); return 5; }
}

// IvfPqIndex::search_batch (ivf_pq.hpp:213).  Raw results (no padding):
// out_counts[q] = number of results returned for query q (<= k).
int rb_ivfpq_search_batch(void* h, const float* queries, size_t nq, uint32_t k,
                          uint32_t nprobe, uint64_t* out_ids, float* out_d,
                          uint32_t* out_counts) {
    IvfPqSearchParams sp; sp.k = k; sp.nprobe = nprobe;
    try {
        auto r = static_cast<RbIndex*>(h)->idx.search_batch(queries, nq, sp);
        if (!r) { set_err(r.error().message); return 2; }
        for (size_t q = 0; q < nq; ++q) {
            const auto& v = (*r)[q];
            const size_t take = v.size() < k ? v.size() : k;
            out_counts[q] = static_cast<uint32_t>(take);
            for (size_t i = 0; i < take; ++i) {
                out_ids[q * k + i] = v[i].first;
                out_d[q * k + i] = v[i].second;
            }
        }
        return 0;
    } catch (const std::exception& e) { set_err(e.what()); return 5; }
}

// The same with the search parameters the C ABI hides (ivf_pq.hpp:109-117): candidate
// pool cand_k and the opt-in exact rerank of the pool's head (use_exact_rerank,
// rerank_k).  At most k results per query are copied out.
int rb_ivfpq_search_batch_ex(void* h, const float* queries, size_t nq, uint32_t k,
                             uint32_t nprobe, uint32_t cand_k, int use_exact_rerank,
                             uint32_t rerank_k, uint64_t* out_ids, float* out_d,
                             uint32_t* out_counts) {
    IvfPqSearchParams sp; sp.k = k; sp.nprobe = nprobe; sp.cand_k = cand_k;
    sp.use_exact_rerank = use_exact_rerank != 0; sp.rerank_k = rerank_k;
    try {
        auto r = static_cast<RbIndex*>(h)->idx.search_batch(queries, nq, sp);
        if (!r) { set_err(r.error().message); return 2; }
        for (size_t q = 0; q < nq; ++q) {
            const auto& v = (*r)[q];
            const size_t take = v.size() < k ? v.size() : k;
            out_counts[q] = static_cast<uint32_t>(take);
            for (size_t i = 0; i < take; ++i) {
                out_ids[q * k + i] = v[i].first;
                out_d[q * k + i] = v[i].second;
            }
        }
        return 0;
    } catch (const std::exception& e) { set_err(e.what()); return 5; }
}

// The rest of IvfPqIndex's API (ivf_pq.hpp:252-386).  Each returns 0 or the reference's
// error code number (core::error_code) and writes its outputs.
static int code_of(const core::error& e) { set_err(e.message); return static_cast<int>(e.code); }

int rb_ivfpq_reconstruct(void* h, uint64_t id, float* out) {
    auto r = static_cast<RbIndex*>(h)->idx.reconstruct(id);
    if (!r) return code_of(r.error());
    std::memcpy(out, r->data(), r->size() * sizeof(float));
    return 0;
}
// out_ids / out_vec must hold the cluster's entries; *n receives their count.
int rb_ivfpq_reconstruct_cluster(void* h, uint32_t cluster, uint64_t* out_ids, float* out_vec, size_t cap,
                                 size_t* n) {
    std::vector<uint64_t> ids;
    std::vector<float> vec;
    auto r = static_cast<RbIndex*>(h)->idx.reconstruct_cluster(cluster, ids, vec);
    if (!r) return code_of(r.error());
    *n = ids.size();
    if (ids.size() > cap) return -1;
    std::memcpy(out_ids, ids.data(), ids.size() * 8);
    std::memcpy(out_vec, vec.data(), vec.size() * 4);
    return 0;
}
int rb_ivfpq_get_cluster_assignment(void* h, uint64_t id, uint32_t* out) {
    auto r = static_cast<RbIndex*>(h)->idx.get_cluster_assignment(id);
    if (!r) return code_of(r.error());
    *out = *r;
    return 0;
}
int rb_ivfpq_update_cluster_centroid(void* h, uint32_t cluster, const float* c) {
    auto r = static_cast<RbIndex*>(h)->idx.update_cluster_centroid(cluster, c);
    if (!r) return code_of(r.error());
    return 0;
}
int rb_ivfpq_reassign_vector(void* h, uint64_t id, uint32_t cluster) {
    auto r = static_cast<RbIndex*>(h)->idx.reassign_vector(id, cluster);
    if (!r) return code_of(r.error());
    return 0;
}
int rb_ivfpq_debug_centroid_rank(void* h, const float* q, uint64_t id, uint64_t* rank, uint32_t* cluster) {
    auto r = static_cast<RbIndex*>(h)->idx.debug_explain_centroid_rank(q, id);
    if (!r) return code_of(r.error());
    *rank = r->first;
    *cluster = r->second;
    return 0;
}
int rb_ivfpq_debug_adc_rank(void* h, const float* q, uint64_t id, uint64_t* rank, float* dist) {
    auto r = static_cast<RbIndex*>(h)->idx.debug_explain_adc_rank(q, id);
    if (!r) return code_of(r.error());
    *rank = r->first;
    *dist = r->second;
    return 0;
}

int rb_ivfpq_save(void* h, const char* dir) {
    auto r = static_cast<RbIndex*>(h)->idx.save(std::string(dir));
    if (!r) { set_err(r.error().message); return 4; }
    return 0;
}

void rb_ivfpq_set_metadata_json(void* h, const char* js) { static_cast<RbIndex*>(h)->idx.set_metadata_json(js); }
// Copies up to cap-1 bytes (NUL-terminated) and returns the full length.
size_t rb_ivfpq_get_metadata_json(void* h, char* out, size_t cap) {
    const std::string s = static_cast<RbIndex*>(h)->idx.get_metadata_json();
    if (out && cap) {
        const size_t n = std::min(cap - 1, s.size());
        std::memcpy(out, s.data(), n);
        out[n] = 0;
    }
    return s.size();
}

int rb_ivfpq_load(void* h, const char* dir) {
    auto r = IvfPqIndex::load(std::string(dir));
    if (!r) { set_err(r.error().message); return 4; }
    static_cast<RbIndex*>(h)->idx = std::move(*r);
    return 0;
}

// ---------------------------------------------------------------- k-means
// kmeans_plusplus_init (src/index/kmeans.cpp:45-89)
void rb_kmeanspp_init(const float* data, size_t n, size_t dim, uint32_t k, uint32_t seed,
                      float* out_centroids) {
    auto c = kmeans_plusplus_init(data, n, dim, k, seed);
    for (uint32_t i = 0; i < k; ++i) std::memcpy(out_centroids + i * dim, c[i].data(), dim * 4);
}

// KmeansElkan::cluster (src/index/kmeans_elkan.cpp:293-430), k-means++ init.
int rb_kmeans_elkan(const float* data, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                    float epsilon, uint32_t seed, float* out_centroids, uint32_t* out_assign,
                    uint32_t* out_iters, float* out_inertia) {
    KmeansElkan elkan;
    KmeansElkan::Config cfg{.k = k, .max_iter = max_iter, .epsilon = epsilon, .seed = seed};
    auto r = elkan.cluster(data, n, dim, cfg);
    if (!r) { set_err(r.error().message); return 2; }
    for (uint32_t i = 0; i < k; ++i) std::memcpy(out_centroids + i * dim, r->centroids[i].data(), dim * 4);
    if (out_assign) std::memcpy(out_assign, r->assignments.data(), n * 4);
    if (out_iters) *out_iters = r->iterations;
    if (out_inertia) *out_inertia = r->inertia;
    return 0;
}

// kmeans_cluster (Lloyd, src/index/kmeans.cpp:137-252)
int rb_kmeans_lloyd(const float* data, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                    float epsilon, uint32_t seed, float* out_centroids, uint32_t* out_assign,
                    uint32_t* out_iters, float* out_inertia) {
    KmeansParams p; p.k = k; p.max_iter = max_iter; p.epsilon = epsilon; p.seed = seed;
    auto r = kmeans_cluster(data, n, dim, p);
    if (!r) { set_err(r.error().message); return 2; }
    for (uint32_t i = 0; i < k; ++i) std::memcpy(out_centroids + i * dim, r->centroids[i].data(), dim * 4);
    if (out_assign) std::memcpy(out_assign, r->assignments.data(), n * 4);
    if (out_iters) *out_iters = r->iterations;
    if (out_inertia) *out_inertia = r->inertia;
    return 0;
}

static std::vector<std::vector<float>> to_vv(const float* c, uint32_t k, size_t dim) {
    std::vector<std::vector<float>> v(k);
    for (uint32_t i = 0; i < k; ++i) v[i].assign(c + i * dim, c + (i + 1) * dim);
    return v;
}

// kmeans_assign (src/index/kmeans.cpp:91-105)
float rb_kmeans_assign(const float* data, size_t n, const float* centroids, uint32_t k,
                       size_t dim, uint32_t* out_assign) {
    auto c = to_vv(centroids, k, dim);
    return kmeans_assign(data, n, c, std::span<std::uint32_t>(out_assign, n));
}

// kmeans_update_centroids (src/index/kmeans.cpp:107-135)
void rb_kmeans_update(const float* data, size_t n, size_t dim, const uint32_t* assign,
                      uint32_t k, float* centroids_inout) {
    auto c = to_vv(centroids_inout, k, dim);
    kmeans_update_centroids(data, n, dim, std::span<const std::uint32_t>(assign, n), k, c);
    for (uint32_t i = 0; i < k; ++i) std::memcpy(centroids_inout + i * dim, c[i].data(), dim * 4);
}

// ---------------------------------------------------------------- FastScanPq
void* rb_pq_create(uint32_t m, uint32_t nbits) {
    FastScanPqConfig cfg{.m = m, .nbits = nbits, .block_size = 32, .use_avx512 = false};
    return new FastScanPq(cfg);
}
void rb_pq_destroy(void* h) { delete static_cast<FastScanPq*>(h); }
int rb_pq_train(void* h, const float* data, size_t n, size_t dim) {
    auto r = static_cast<FastScanPq*>(h)->train(data, n, dim);
    if (!r) { set_err(r.error().message); return 2; }
    return 0;
}
void rb_pq_import(void* h, size_t dsub, const float* cb, size_t count) {
    static_cast<FastScanPq*>(h)->import_pretrained(dsub, std::span<const float>(cb, count));
}
void rb_pq_export(void* h, float* out) {
    std::vector<float> v; static_cast<FastScanPq*>(h)->export_codebooks(v);
    std::memcpy(out, v.data(), v.size() * 4);
}
void rb_pq_encode(void* h, const float* data, size_t n, uint8_t* codes) {
    static_cast<FastScanPq*>(h)->encode(data, n, codes);
}
// compute_lookup_tables (src/index/pq_fastscan.cpp:145-172), de-strided to [m x ksub]
void rb_pq_lut(void* h, const float* q, float* out) {
    auto* pq = static_cast<FastScanPq*>(h);
    auto luts = pq->compute_lookup_tables(q);
    const uint32_t m = pq->config().m, ksub = pq->ksub();
    for (uint32_t s = 0; s < m; ++s) std::memcpy(out + s * ksub, luts[s], ksub * 4);
}
// compute_distances_avx2 over blocks built from row-major codes (pq_fastscan.cpp:201-234)
void rb_pq_adc(void* h, const float* q, const uint8_t* codes, size_t n, float* out) {
    auto* pq = static_cast<FastScanPq*>(h);
    const uint32_t m = pq->config().m;
    std::vector<PqCodeBlock> blocks;
    PqCodeBlock blk(m, 32);
    for (size_t i = 0; i < n; ++i) {
        if (!blk.add_code(codes + i * m)) { blocks.push_back(blk); blk.clear(); blk.add_code(codes + i * m); }
    }
    if (blk.size() > 0) blocks.push_back(blk);
    std::vector<float> d(blocks.size() * 32, 0.0f);
    pq->compute_distances_avx2(q, blocks, d.data());
    std::memcpy(out, d.data(), n * 4);
}

// ---------------------------------------------------------------- flat top-k
// find_nearest_centroids_batch_fused (kernels/batch_distances.hpp:338-456)
// op: 0 = L2, 1 = InnerProduct
void rb_flat_topk(int op, const float* queries, size_t nq, const float* base, uint32_t nb,
                  size_t dim, uint32_t k, uint32_t* out_idx, float* out_score) {
    AlignedCentroidBuffer buf(nb, dim);
    for (uint32_t i = 0; i < nb; ++i) std::memcpy(buf[i], base + (size_t)i * dim, dim * 4);
    kernels::find_nearest_centroids_batch_fused(
        op == 0 ? kernels::DistanceOp::L2 : kernels::DistanceOp::InnerProduct, queries, nq, buf,
        k, out_idx, out_score);
}

// The same search over a base held in the reference's AlignedCentroidBuffer across
// calls (the copy into it is not part of a timed search).
void* rb_flat_buffer_create(const float* base, uint32_t nb, size_t dim) {
    auto* buf = new AlignedCentroidBuffer(nb, dim);
    for (uint32_t i = 0; i < nb; ++i) std::memcpy((*buf)[i], base + (size_t)i * dim, dim * 4);
    return buf;
}
void rb_flat_buffer_destroy(void* h) { delete static_cast<AlignedCentroidBuffer*>(h); }
void rb_flat_topk_buffer(int op, const float* queries, size_t nq, void* h, uint32_t k, uint32_t* out_idx,
                         float* out_score) {
    kernels::find_nearest_centroids_batch_fused(
        op == 0 ? kernels::DistanceOp::L2 : kernels::DistanceOp::InnerProduct, queries, nq,
        *static_cast<AlignedCentroidBuffer*>(h), k, out_idx, out_score);
}

}  // extern "C"
