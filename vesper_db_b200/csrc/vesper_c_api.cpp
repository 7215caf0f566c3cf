// C ABI of the B200 IVF-PQ engine: the reference's vesper_ivfpq_* surface
// (include/vesper/c/vesper.h, src/c/vesper_c_api.cpp) over vesper::index::IvfPqIndex,
// plus the extensions declared in include/vesper_b200.h.
//
// Status mapping follows the reference: NULL arguments -> INVALID_PARAM without
// touching the last error; an error returned by train/add/search -> INVALID_PARAM
// with its message; save/load -> IO; std::exception -> INTERNAL; anything else ->
// UNKNOWN.  The last error is a thread-local string.
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "../../include/vesper_b200.h"
#include "c_error.hpp"
#include "ivf_pq_gpu.hpp"
#include "kernels_tc.cuh"
#include "kmeans_gpu.hpp"

using vesper::index::IvfPqIndex;
using vesper::index::IvfPqSearchParams;
using vesper::index::IvfPqTrainParams;
using vesper::index::IvfPqTrainStats;
using vesper::index::SearchMode;

struct vesper_index_t {
    std::unique_ptr<IvfPqIndex> ivfpq;
    IvfPqTrainStats last_train;
};

namespace {
thread_local std::string g_last_error;
}  // namespace

namespace vesper_c {
void set_error(const std::string& s) { g_last_error = s; }
void clear_error() { g_last_error.clear(); }
}  // namespace vesper_c

using vesper_c::clear_error;
using vesper_c::set_error;

namespace {

template <class F>
vesper_status_t guarded(const char* what, F&& f) {
    try {
        return f();
    } catch (const std::bad_alloc&) {
        set_error("allocation failure");
        return VESPER_ERROR_INTERNAL;
    } catch (const std::exception& e) {
        set_error(e.what());
        return VESPER_ERROR_INTERNAL;
    } catch (...) {
        set_error(std::string("unknown error in ") + what);
        return VESPER_ERROR_UNKNOWN;
    }
}

// Pad rows beyond counts[q] the way the reference does (vesper_c_api.cpp:243-253).
// The engine already pads; this keeps the contract explicit for search().
}  // namespace

extern "C" {

VESPER_C_API const char* vesper_get_last_error(void) { return g_last_error.c_str(); }
VESPER_C_API const char* vesper_version(void) { return "dev"; }

VESPER_C_API vesper_status_t vesper_ivfpq_is_trained(const vesper_index_t* index, int* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("is_trained", [&] { *out = index->ivfpq->is_trained() ? 1 : 0; return VESPER_OK; });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_dimension(const vesper_index_t* index, size_t* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_dimension", [&] { *out = index->ivfpq->dimension(); return VESPER_OK; });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_stats(const vesper_index_t* index, vesper_ivfpq_stats_t* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_stats", [&] {
        const auto s = index->ivfpq->get_stats();
        out->n_vectors = s.n_vectors;
        out->n_lists = s.n_lists;
        out->m = s.m;
        out->memory_bytes = s.memory_bytes;
        out->avg_list_size = s.avg_list_size;
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_set_metadata_json(vesper_index_t* index, const char* json) {
    if (!index || !index->ivfpq || !json) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("set_metadata_json", [&] { index->ivfpq->set_metadata_json(json); return VESPER_OK; });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_metadata_json(const vesper_index_t* index, char* out_buffer,
                                                            size_t buffer_size, size_t* out_required) {
    if (!index || !index->ivfpq) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_metadata_json", [&] {
        const std::string s = index->ivfpq->get_metadata_json();
        const size_t required = s.size() + 1;
        if (out_required) *out_required = required;
        if (!out_buffer || buffer_size == 0) return VESPER_OK;
        if (buffer_size < required) {
            set_error("buffer too small for metadata json");
            return VESPER_ERROR_INVALID_PARAM;
        }
        std::memcpy(out_buffer, s.c_str(), required);
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_create(vesper_index_t** out_index) {
    if (!out_index) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("create", [&] {
        auto h = std::make_unique<vesper_index_t>();
        h->ivfpq = std::make_unique<IvfPqIndex>();
        *out_index = h.release();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_destroy(vesper_index_t* index) {
    clear_error();
    return guarded("destroy", [&] { delete index; return VESPER_OK; });
}

static vesper_status_t do_train(vesper_index_t* index, const float* base, size_t dim, size_t n,
                                const IvfPqTrainParams& tp, bool on_device = false) {
    return guarded("train", [&] {
        auto r = index->ivfpq->train_device(base, dim, n, tp, on_device);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        index->last_train = *r;
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_train(vesper_index_t* index, const float* base, size_t dim,
                                                size_t n, const vesper_ivfpq_train_params_t* params) {
    if (!index || !index->ivfpq || !base || !params || dim == 0 || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    IvfPqTrainParams tp;
    tp.nlist = params->nlist;
    tp.m = params->m;
    tp.nbits = params->nbits;
    tp.timings_enabled = false;
    return do_train(index, base, dim, n, tp);
}

VESPER_C_API void vesper_ivfpq_train_params_ex_init(vesper_ivfpq_train_params_ex_t* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->struct_size = sizeof(*p);
    p->nlist = 256;
    p->m = 8;
    p->nbits = 8;
    p->max_iter = 25;
    p->epsilon = 1e-4f;
    p->use_opq = 1;
    p->opq_iter = 10;
    p->opq_sample_n = 20000;
    p->opq_init_pca = 1;
    p->seed = 42;
}

static IvfPqTrainParams to_params(const vesper_ivfpq_train_params_ex_t* p) {
    IvfPqTrainParams tp;
    tp.nlist = p->nlist;
    tp.m = p->m;
    tp.nbits = p->nbits;
    tp.max_iter = p->max_iter;
    tp.epsilon = p->epsilon;
    tp.use_opq = p->use_opq != 0;
    tp.opq_iter = p->opq_iter;
    tp.opq_sample_n = p->opq_sample_n;
    tp.opq_init = p->opq_init_pca ? vesper::index::OpqInit::PCA : vesper::index::OpqInit::Identity;
    tp.seed = p->seed;
    tp.verbose = p->verbose != 0;
    return tp;
}

VESPER_C_API vesper_status_t vesper_ivfpq_train_ex(vesper_index_t* index, const float* base, size_t dim,
                                                   size_t n, const vesper_ivfpq_train_params_ex_t* p) {
    if (!index || !index->ivfpq || !base || !p || dim == 0 || n == 0) return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < sizeof(vesper_ivfpq_train_params_ex_t)) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_train(index, base, dim, n, to_params(p), false);
}

VESPER_C_API vesper_status_t vesper_ivfpq_train_ex_device(vesper_index_t* index, const float* d_base, size_t dim,
                                                          size_t n, const vesper_ivfpq_train_params_ex_t* p) {
    if (!index || !index->ivfpq || !d_base || !p || dim == 0 || n == 0) return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < sizeof(vesper_ivfpq_train_params_ex_t)) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_train(index, d_base, dim, n, to_params(p), true);
}

VESPER_C_API vesper_status_t vesper_ivfpq_add_device(vesper_index_t* index, const uint64_t* d_ids,
                                                     const float* d_base, size_t n) {
    if (!index || !index->ivfpq || !d_ids || !d_base || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("add", [&] {
        auto r = index->ivfpq->add_device(d_ids, d_base, n, true);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_train_report(const vesper_index_t* index,
                                                           vesper_ivfpq_train_report_t* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    out->opq_kept = index->last_train.opq_kept ? 1 : 0;
    out->err_unrot = index->last_train.err_unrot;
    out->err_opq = index->last_train.err_opq;
    out->coarse_iterations = index->last_train.coarse_iterations;
    out->train_time_sec = index->last_train.train_time_sec;
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_ivfpq_add(vesper_index_t* index, const uint64_t* ids, const float* base,
                                              size_t n) {
    if (!index || !index->ivfpq || !ids || !base || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("add", [&] {
        auto r = index->ivfpq->add(ids, base, n);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

// The fields of vesper_ivfpq_search_params_ex_t the caller's struct_size covers.
static IvfPqSearchParams ex_params(const vesper_ivfpq_search_params_ex_t* p) {
    IvfPqSearchParams sp;
    sp.k = p->k;
    sp.nprobe = p->nprobe;
    sp.mode = p->mode == VESPER_SEARCH_EXACT ? SearchMode::Exact : SearchMode::Fast;
    if (p->struct_size >= sizeof(vesper_ivfpq_search_params_ex_t)) {
        sp.cand_k = p->cand_k;
        sp.use_exact_rerank = p->use_exact_rerank != 0;
        sp.rerank_k = p->rerank_k;
    }
    return sp;
}

static vesper_status_t do_search(const vesper_index_t* index, const float* q, size_t nq, uint32_t k,
                                 uint32_t nprobe, uint32_t mode, uint64_t* ids, float* d, uint32_t* counts,
                                 bool on_device, const vesper_ivfpq_search_params_ex_t* ex = nullptr) {
    IvfPqSearchParams sp;
    if (ex) sp = ex_params(ex);
    sp.k = k;
    sp.nprobe = nprobe;
    sp.mode = mode == VESPER_SEARCH_EXACT ? SearchMode::Exact : SearchMode::Fast;
    return guarded("search", [&] {
        auto r = index->ivfpq->search_batch_flat(q, nq, sp, ids, d, counts, on_device);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_search(const vesper_index_t* index, const float* query,
                                                 const vesper_ivfpq_search_params_t* params, uint64_t* out_ids,
                                                 float* out_d) {
    if (!index || !index->ivfpq || !query || !params || !out_ids || !out_d) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_search(index, query, 1, params->k, params->nprobe, VESPER_SEARCH_FAST, out_ids, out_d, nullptr,
                     false);
}

VESPER_C_API vesper_status_t vesper_ivfpq_search_batch(const vesper_index_t* index, const float* queries,
                                                       size_t nq, const vesper_ivfpq_search_params_t* params,
                                                       uint64_t* out_ids, float* out_d) {
    if (!index || !index->ivfpq || !queries || !params || !out_ids || !out_d || nq == 0)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_search(index, queries, nq, params->k, params->nprobe, VESPER_SEARCH_FAST, out_ids, out_d, nullptr,
                     false);
}

VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_ex(const vesper_index_t* index, const float* queries,
                                                          size_t nq, const vesper_ivfpq_search_params_ex_t* p,
                                                          uint64_t* out_ids, float* out_d, uint32_t* out_counts) {
    if (!index || !index->ivfpq || !queries || !p || !out_ids || !out_d || nq == 0)
        return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < VESPER_IVFPQ_SEARCH_PARAMS_EX_V1_SIZE) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_search(index, queries, nq, p->k, p->nprobe, p->mode, out_ids, out_d, out_counts, false, p);
}

VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device(const vesper_index_t* index, const float* d_q,
                                                              size_t nq, const vesper_ivfpq_search_params_ex_t* p,
                                                              uint64_t* d_ids, float* d_d, uint32_t* d_counts) {
    if (!index || !index->ivfpq || !d_q || !p || !d_ids || !d_d || nq == 0) return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < VESPER_IVFPQ_SEARCH_PARAMS_EX_V1_SIZE) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return do_search(index, d_q, nq, p->k, p->nprobe, p->mode, d_ids, d_d, d_counts, true, p);
}

VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device_noalloc(
    const vesper_index_t* index, const float* d_q, size_t nq, const vesper_ivfpq_search_params_ex_t* p,
    uint64_t* d_ids, float* d_d, uint32_t* d_counts) {
    if (!index || !index->ivfpq || !d_q || !p || !d_ids || !d_d || nq == 0) return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < VESPER_IVFPQ_SEARCH_PARAMS_EX_V1_SIZE) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    const IvfPqSearchParams sp = ex_params(p);
    if (sp.use_exact_rerank) {
        set_error("the allocation-free search does not support the exact rerank");
        return VESPER_ERROR_INVALID_PARAM;
    }
    return guarded("search_noalloc", [&] {
        auto r = index->ivfpq->search_batch_device_noalloc(d_q, nq, sp, d_ids, d_d, d_counts);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_probe_device(const vesper_index_t* index, const float* d_q, size_t nq,
                                                       uint32_t nprobe, uint32_t* d_probe, float* d_probe_d) {
    if (!index || !index->ivfpq || !d_q || !d_probe || !d_probe_d || nq == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("probe", [&] {
        auto r = index->ivfpq->probe_device(d_q, nq, nprobe, d_probe, d_probe_d);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_search_batch_device_probed(
    const vesper_index_t* index, const float* d_q, size_t nq, const vesper_ivfpq_search_params_ex_t* p,
    const uint32_t* d_probe, const float* d_probe_d, uint64_t* d_ids, float* d_d, uint32_t* d_counts) {
    if (!index || !index->ivfpq || !d_q || !p || !d_probe || !d_probe_d || !d_ids || !d_d || nq == 0)
        return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < VESPER_IVFPQ_SEARCH_PARAMS_EX_V1_SIZE) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    const IvfPqSearchParams sp = ex_params(p);
    return guarded("search_probed", [&] {
        auto r = index->ivfpq->search_batch_device_probed(d_q, nq, sp, d_probe, d_probe_d, d_ids, d_d, d_counts);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_set_threshold_exchange(vesper_index_t* index,
                                                                 vesper_ivfpq_tau_exchange_fn fn, void* user,
                                                                 uint32_t shard, uint32_t shards) {
    if (!index || !index->ivfpq || shards == 0 || shard >= shards) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("set_threshold_exchange", [&] {
        index->ivfpq->set_threshold_exchange(fn, user, shard, shards);
        return VESPER_OK;
    });
}

}  // extern "C"

namespace {
// Status of an index-API result: not trained -> NOT_TRAINED, other errors -> INVALID_PARAM
// with the message.
template <class R>
vesper_status_t api_status(const R& r) {
    if (r) return VESPER_OK;
    set_error(r.error().message);
    using vesper::core::error_code;
    return r.error().code == error_code::not_initialized || r.error().message == "Index not trained"
               ? VESPER_ERROR_NOT_TRAINED
               : (r.error().code == error_code::internal ? VESPER_ERROR_INTERNAL : VESPER_ERROR_INVALID_PARAM);
}
}  // namespace

extern "C" {

VESPER_C_API vesper_status_t vesper_ivfpq_reconstruct(const vesper_index_t* index, uint64_t id, float* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("reconstruct", [&] {
        auto r = index->ivfpq->reconstruct(id);
        if (r) std::memcpy(out, r->data(), r->size() * sizeof(float));
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_reconstruct_cluster(const vesper_index_t* index, uint32_t cluster_id,
                                                              uint64_t* out_ids, float* out_vectors, size_t capacity,
                                                              size_t* out_count) {
    if (!index || !index->ivfpq || !out_count) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("reconstruct_cluster", [&] {
        std::vector<uint64_t> ids;
        std::vector<float> vec;
        auto r = index->ivfpq->reconstruct_cluster(cluster_id, ids, vec);
        if (!r) return api_status(r);
        *out_count = ids.size();
        if (ids.size() > capacity || (!ids.empty() && (!out_ids || !out_vectors))) {
            set_error("reconstruct_cluster: output capacity too small");
            return VESPER_ERROR_INVALID_PARAM;
        }
        if (!ids.empty()) {
            std::memcpy(out_ids, ids.data(), ids.size() * sizeof(uint64_t));
            std::memcpy(out_vectors, vec.data(), vec.size() * sizeof(float));
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_cluster_assignment(const vesper_index_t* index, uint64_t id,
                                                                 uint32_t* out_cluster) {
    if (!index || !index->ivfpq || !out_cluster) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_cluster_assignment", [&] {
        auto r = index->ivfpq->get_cluster_assignment(id);
        if (r) *out_cluster = *r;
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_cluster_centroid(const vesper_index_t* index, uint32_t cluster_id,
                                                               float* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_cluster_centroid", [&] {
        auto r = index->ivfpq->get_cluster_centroid(cluster_id);
        if (r) std::memcpy(out, r->data(), r->size() * sizeof(float));
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_update_cluster_centroid(vesper_index_t* index, uint32_t cluster_id,
                                                                  const float* centroid) {
    if (!index || !index->ivfpq) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("update_cluster_centroid",
                   [&] { return api_status(index->ivfpq->update_cluster_centroid(cluster_id, centroid)); });
}

VESPER_C_API vesper_status_t vesper_ivfpq_reassign_vector(vesper_index_t* index, uint64_t id, uint32_t new_cluster) {
    if (!index || !index->ivfpq) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("reassign_vector", [&] { return api_status(index->ivfpq->reassign_vector(id, new_cluster)); });
}

VESPER_C_API vesper_status_t vesper_ivfpq_compact_inverted_list(vesper_index_t* index, uint32_t cluster_id,
                                                                const uint32_t* deleted_ids, size_t n_deleted,
                                                                size_t* out_removed) {
    if (!index || !index->ivfpq || (n_deleted && !deleted_ids)) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("compact_inverted_list", [&] {
        auto r = index->ivfpq->compact_inverted_list(cluster_id, deleted_ids, n_deleted);
        if (r && out_removed) *out_removed = *r;
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_debug_explain_centroid_rank(const vesper_index_t* index, const float* query,
                                                                      uint64_t target_id, uint64_t* out_rank,
                                                                      uint32_t* out_cluster) {
    if (!index || !index->ivfpq || !query || !out_rank || !out_cluster) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("debug_explain_centroid_rank", [&] {
        auto r = index->ivfpq->debug_explain_centroid_rank(query, target_id);
        if (r) { *out_rank = r->first; *out_cluster = r->second; }
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_debug_explain_adc_rank(const vesper_index_t* index, const float* query,
                                                                 uint64_t target_id, uint64_t* out_rank,
                                                                 float* out_distance) {
    if (!index || !index->ivfpq || !query || !out_rank || !out_distance) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("debug_explain_adc_rank", [&] {
        auto r = index->ivfpq->debug_explain_adc_rank(query, target_id);
        if (r) { *out_rank = r->first; *out_distance = r->second; }
        return api_status(r);
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_last_timings(const vesper_index_t* index, vesper_ivfpq_timings_t* out) {
    if (!index || !index->ivfpq || !out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    const auto t = index->ivfpq->last_search_timings();
    out->coarse_ms = t.coarse_ms;
    out->select_ms = t.select_ms;
    out->rotate_ms = t.rotate_ms;
    out->scan_ms = t.scan_ms;
    out->merge_ms = t.merge_ms;
    out->total_ms = t.total_ms;
    out->scanned_entries = t.scanned_entries;
    out->kernel_launches = t.kernel_launches;
    out->scan_variant = t.scan_variant;
    out->coarse_variant = t.coarse_variant;
    out->list_kernel_ms = t.list_kernel_ms;
    out->list_candidates = t.list_candidates;
    out->list_fallback_queries = t.list_fallback_queries;
    out->list_threshold_ms = t.list_threshold_ms;
    out->list_prep_ms = t.list_prep_ms;
    out->list_refine_ms = t.list_refine_ms;
    out->list_fallback_ms = t.list_fallback_ms;
    out->rerank_ms = t.rerank_ms;
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_ivfpq_set_model(vesper_index_t* index, size_t dim, uint32_t nlist, uint32_t m,
                                                    uint32_t nbits, const float* centroids, const float* codebooks,
                                                    const float* rotation) {
    if (!index || !index->ivfpq || !centroids || !codebooks) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("set_model", [&] {
        auto r = index->ivfpq->set_model(dim, nlist, m, nbits, centroids, codebooks, rotation);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_INVALID_PARAM;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_get_lists(const vesper_index_t* index, uint64_t* out_offsets,
                                                    uint64_t* out_ids, uint8_t* out_codes) {
    if (!index || !index->ivfpq) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("get_lists", [&] {
        if (out_offsets) {
            const auto o = index->ivfpq->list_offsets();
            std::memcpy(out_offsets, o.data(), o.size() * sizeof(uint64_t));
        }
        if (out_ids) {
            const auto v = index->ivfpq->list_ids();
            std::memcpy(out_ids, v.data(), v.size() * sizeof(uint64_t));
        }
        if (out_codes) {
            const auto v = index->ivfpq->list_codes();
            std::memcpy(out_codes, v.data(), v.size());
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_save(const vesper_index_t* index, const char* file_path) {
    if (!index || !index->ivfpq || !file_path) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("save", [&] {
        auto r = index->ivfpq->save(file_path);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_IO;
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_ivfpq_load(vesper_index_t* index, const char* file_path) {
    if (!index || !file_path) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("load", [&] {
        auto r = IvfPqIndex::load(file_path);
        if (!r) {
            set_error(r.error().message);
            return VESPER_ERROR_IO;
        }
        index->ivfpq = std::make_unique<IvfPqIndex>(std::move(*r));
        return VESPER_OK;
    });
}

VESPER_C_API void vesper_kmeans_params_init(vesper_kmeans_params_t* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->struct_size = sizeof(*p);
    p->k = 256;
    p->max_iter = 25;
    p->epsilon = 1e-4f;
    p->seed = 42;
    p->algorithm = VESPER_KMEANS_ELKAN;
}

}  // extern "C"

namespace {
// Shared body of vesper_kmeans_fit / _fit_device: on_device says where data and the
// outputs live.  Checks follow kmeans_cluster (src/index/kmeans.cpp:141-151).
vesper_status_t kmeans_fit(const float* data, size_t n, size_t dim, const vesper_kmeans_params_t* p,
                           float* out_c, uint32_t* out_a, vesper_kmeans_result_t* out_r, bool on_device) {
    if (!data || !p || !out_c || dim == 0 || n == 0) return VESPER_ERROR_INVALID_PARAM;
    if (p->struct_size < sizeof(vesper_kmeans_params_t) || p->algorithm > VESPER_KMEANS_LLOYD)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    if (n < p->k) {
        set_error("Not enough data points for k clusters");
        return VESPER_ERROR_INVALID_PARAM;
    }
    if (p->k == 0) {
        set_error("k must be > 0");
        return VESPER_ERROR_INVALID_PARAM;
    }
    if (dim > (size_t)INT32_MAX) return VESPER_ERROR_INVALID_PARAM;
    return guarded("kmeans", [&] {
        const auto t0 = std::chrono::steady_clock::now();
        cudaStream_t st = nullptr;
        vgpu::check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
        struct StreamOwner {
            cudaStream_t s;
            ~StreamOwner() { cudaStreamSynchronize(s); cudaStreamDestroy(s); }
        } owner{st};
        vgpu::DeviceBuffer<float> x_own, c_own;
        vgpu::DeviceBuffer<uint32_t> a_own;
        const float* x = data;
        float* c = out_c;
        uint32_t* a = out_a;
        if (!on_device) {
            x_own.resize(n * dim);
            vgpu::check(cudaMemcpyAsync(x_own.data(), data, n * dim * sizeof(float), cudaMemcpyHostToDevice, st),
                        "h2d");
            x = x_own.data();
            c_own.resize((size_t)p->k * dim);
            c = c_own.data();
        }
        if (!on_device || !out_a) {
            a_own.resize(n);
            a = a_own.data();
        }
        vgpu::KmeansEngine eng(st);
        const auto r = eng.fit(x, n, (int)dim, p->k, p->max_iter, p->epsilon, p->seed,
                               p->algorithm == VESPER_KMEANS_ELKAN, c, a);
        if (!on_device) {
            vgpu::check(cudaMemcpyAsync(out_c, c, (size_t)p->k * dim * sizeof(float), cudaMemcpyDeviceToHost, st),
                        "d2h");
            if (out_a)
                vgpu::check(cudaMemcpyAsync(out_a, a, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
        }
        vgpu::check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        if (out_r) {
            out_r->iterations = r.iterations;
            out_r->inertia = r.inertia;
            out_r->time_sec = std::chrono::duration<float>(std::chrono::steady_clock::now() - t0).count();
        }
        return VESPER_OK;
    });
}
}  // namespace

extern "C" {

VESPER_C_API vesper_status_t vesper_kmeans_fit(const float* data, size_t n, size_t dim,
                                               const vesper_kmeans_params_t* params, float* out_centroids,
                                               uint32_t* out_assignments, vesper_kmeans_result_t* out_result) {
    return kmeans_fit(data, n, dim, params, out_centroids, out_assignments, out_result, false);
}

VESPER_C_API vesper_status_t vesper_kmeans_fit_device(const float* d_data, size_t n, size_t dim,
                                                      const vesper_kmeans_params_t* params, float* d_out_centroids,
                                                      uint32_t* d_out_assignments, vesper_kmeans_result_t* out_result) {
    return kmeans_fit(d_data, n, dim, params, d_out_centroids, d_out_assignments, out_result, true);
}

}  // extern "C"

struct vesper_kmeans_shard_s {
    cudaStream_t st = nullptr;
    std::unique_ptr<vgpu::KmeansEngine> eng;
    ~vesper_kmeans_shard_s() {
        eng.reset();
        if (st) { cudaStreamSynchronize(st); cudaStreamDestroy(st); }
    }
};

struct vesper_kmeanspp_sampler_s {
    vgpu::KmeansPPSampler s;
};

extern "C" {

VESPER_C_API vesper_status_t vesper_kmeans_shard_create(vesper_kmeans_shard_t** out) {
    if (!out) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    *out = nullptr;
    return guarded("kmeans_shard_create", [&] {
        auto h = std::make_unique<vesper_kmeans_shard_s>();
        vgpu::check(cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking), "cudaStreamCreate");
        h->eng = std::make_unique<vgpu::KmeansEngine>(h->st);
        *out = h.release();
        return VESPER_OK;
    });
}

VESPER_C_API void vesper_kmeans_shard_destroy(vesper_kmeans_shard_t* shard) { delete shard; }

VESPER_C_API vesper_status_t vesper_kmeans_shard_assign(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                        size_t dim, const float* d_centroids, uint32_t k,
                                                        int keep_on_tie, uint32_t* d_assign, float* d_min_dist) {
    if (!shard || (n && (!d_x || !d_assign)) || !d_centroids || k == 0 || dim == 0 || dim > (size_t)INT32_MAX)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeans_shard_assign", [&] {
        if (n) shard->eng->assign(d_x, n, (int)dim, d_centroids, k, d_assign, d_min_dist, keep_on_tie != 0);
        shard->eng->sync();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeans_shard_pp_update(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                           size_t dim, const float* d_centroid, float* d_min_dist) {
    if (!shard || (n && (!d_x || !d_min_dist)) || !d_centroid || dim == 0 || dim > (size_t)INT32_MAX)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeans_shard_pp_update", [&] {
        shard->eng->pp_update(d_x, n, (int)dim, d_centroid, d_min_dist);
        shard->eng->sync();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeans_shard_accumulate(vesper_kmeans_shard_t* shard, const float* d_x, size_t n,
                                                            size_t dim, const uint32_t* d_assign, uint32_t k,
                                                            uint32_t algorithm, double* d_sum, double* d_comp,
                                                            uint64_t* d_count) {
    if (!shard || (n && (!d_x || !d_assign)) || !d_sum || !d_comp || !d_count || k == 0 || dim == 0 ||
        dim > (size_t)INT32_MAX || algorithm > VESPER_KMEANS_LLOYD)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeans_shard_accumulate", [&] {
        shard->eng->accumulate(d_x, n, (int)dim, d_assign, k, algorithm == VESPER_KMEANS_ELKAN, d_sum, d_comp,
                               reinterpret_cast<unsigned long long*>(d_count));
        shard->eng->sync();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeans_shard_finish(vesper_kmeans_shard_t* shard, const double* d_sum,
                                                        const uint64_t* d_count, uint32_t k, size_t dim,
                                                        uint32_t algorithm, float* d_centroids) {
    if (!shard || !d_sum || !d_count || !d_centroids || k == 0 || dim == 0 || dim > (size_t)INT32_MAX ||
        algorithm > VESPER_KMEANS_LLOYD)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeans_shard_finish", [&] {
        shard->eng->finish_means(d_sum, reinterpret_cast<const unsigned long long*>(d_count), k, (int)dim,
                                 algorithm == VESPER_KMEANS_ELKAN, d_centroids);
        shard->eng->sync();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeans_shard_running_inertia(vesper_kmeans_shard_t* shard, const float* d_x,
                                                                 size_t n, size_t dim, const float* d_centroids,
                                                                 const uint32_t* d_assign, float* inout_total) {
    if (!shard || (n && (!d_x || !d_assign)) || !d_centroids || !inout_total || dim == 0 || dim > (size_t)INT32_MAX)
        return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeans_shard_running_inertia", [&] {
        if (n) shard->eng->running_inertia(d_x, n, (int)dim, d_centroids, d_assign, inout_total);
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeanspp_sampler_create(uint32_t seed, size_t n, vesper_kmeanspp_sampler_t** out,
                                                            size_t* first_index) {
    if (!out || !first_index || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    *out = nullptr;
    return guarded("kmeanspp_sampler_create", [&] {
        *out = new vesper_kmeanspp_sampler_s{vgpu::KmeansPPSampler(seed, n)};
        *first_index = (*out)->s.first();
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_kmeanspp_sampler_next(vesper_kmeanspp_sampler_t* sampler, const float* d2,
                                                          size_t* index) {
    if (!sampler || !d2 || !index) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded("kmeanspp_sampler_next", [&] {
        *index = sampler->s.next(d2);
        return VESPER_OK;
    });
}

VESPER_C_API void vesper_kmeanspp_sampler_destroy(vesper_kmeanspp_sampler_t* sampler) { delete sampler; }

}  // extern "C"

namespace {
// Per-thread flat top-k context on the current device: stream + reusable scratch.
struct FlatCtx {
    int device = -1;
    cudaStream_t st = nullptr;
    std::unique_ptr<vgpu::FlatWork> w;
    ~FlatCtx() {
        w.reset();
        if (st) cudaStreamDestroy(st);
    }
};
thread_local FlatCtx g_flat;

FlatCtx& flat_ctx() {
    int dev = 0;
    vgpu::check(cudaGetDevice(&dev), "cudaGetDevice");
    if (g_flat.device != dev) {
        g_flat.w.reset();
        if (g_flat.st) cudaStreamDestroy(g_flat.st);
        g_flat.st = nullptr;
        g_flat.device = dev;
        vgpu::check(cudaStreamCreateWithFlags(&g_flat.st, cudaStreamNonBlocking), "cudaStreamCreate");
        g_flat.w = std::make_unique<vgpu::FlatWork>();
    }
    return g_flat;
}

// Shared body of vesper_flat_topk / _device; the checks mirror the reference's early
// return (n_base, nq or k == 0 -> nothing written).
vesper_status_t flat_topk(vesper_flat_op_t op, const float* q, size_t nq, const float* base, size_t nb, size_t dim,
                          uint32_t k, uint32_t* out_i, float* out_s, bool on_device) {
    if (op != VESPER_FLAT_L2 && op != VESPER_FLAT_IP) return VESPER_ERROR_INVALID_PARAM;
    if (nq == 0 || nb == 0 || k == 0) return VESPER_OK;
    if (!q || !base || !out_i || !out_s || dim == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    if (k > 1024 || dim % 4 != 0 || dim < 32 || dim > (size_t)INT32_MAX || nb > (size_t)INT32_MAX ||
        nq > (size_t)INT32_MAX) {
        set_error("flat_topk: unsupported shape (k <= 1024, dim % 4 == 0, dim >= 32, n_base < 2^31)");
        return VESPER_ERROR_INVALID_PARAM;
    }
    return guarded("flat_topk", [&] {
        FlatCtx& ctx = flat_ctx();
        cudaStream_t st = ctx.st;
        vgpu::DeviceBuffer<float> q_own, b_own, s_own;
        vgpu::DeviceBuffer<uint32_t> i_own;
        const float* dq = q;
        const float* db = base;
        uint32_t* di = out_i;
        float* ds = out_s;
        if (!on_device) {
            q_own.resize(nq * dim);
            b_own.resize(nb * dim);
            i_own.resize(nq * k);
            s_own.resize(nq * k);
            vgpu::check(cudaMemcpyAsync(q_own.data(), q, nq * dim * sizeof(float), cudaMemcpyHostToDevice, st), "h2d");
            dq = q_own.data();
            di = i_own.data();
            ds = s_own.data();
            // the base's copy overlaps the threshold pass and the filter
            vgpu::launch_flat_topk_host(op == VESPER_FLAT_IP, dq, (long long)nq, base, b_own.data(), (long long)nb,
                                        (int)dim, (int)k, di, ds, *ctx.w, st);
        } else {
            vgpu::launch_flat_topk(op == VESPER_FLAT_IP, dq, (long long)nq, db, (long long)nb, (int)dim, (int)k, di,
                                   ds, *ctx.w, st);
        }
        if (!on_device) {
            vgpu::check(cudaMemcpyAsync(out_i, di, nq * k * sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
            vgpu::check(cudaMemcpyAsync(out_s, ds, nq * k * sizeof(float), cudaMemcpyDeviceToHost, st), "d2h");
        }
        vgpu::check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        return VESPER_OK;
    });
}
}  // namespace

extern "C" {

VESPER_C_API vesper_status_t vesper_flat_topk(vesper_flat_op_t op, const float* queries, size_t nq,
                                              const float* base, size_t n_base, size_t dim, uint32_t k,
                                              uint32_t* out_indices, float* out_scores) {
    return flat_topk(op, queries, nq, base, n_base, dim, k, out_indices, out_scores, false);
}

VESPER_C_API vesper_status_t vesper_flat_topk_device(vesper_flat_op_t op, const float* d_queries, size_t nq,
                                                     const float* d_base, size_t n_base, size_t dim, uint32_t k,
                                                     uint32_t* d_out_indices, float* d_out_scores) {
    return flat_topk(op, d_queries, nq, d_base, n_base, dim, k, d_out_indices, d_out_scores, true);
}

VESPER_C_API vesper_status_t vesper_flat_get_last_timings(vesper_flat_timings_t* out) {
    if (!out) return VESPER_ERROR_INVALID_PARAM;
    std::memset(out, 0, sizeof(*out));
    if (!g_flat.w) return VESPER_OK;
    const vgpu::FlatStats& s = g_flat.w->last;
    out->total_ms = s.total_ms;
    out->norms_ms = s.norms_ms;
    out->sample_ms = s.sample_ms;
    out->filter_ms = s.filter_ms;
    out->refine_ms = s.refine_ms;
    out->fallback_ms = s.fallback_ms;
    out->candidates = s.candidates;
    out->overflow_queries = s.overflow_queries;
    out->sample_stride = (uint32_t)s.sample_stride;
    out->single_pass = (uint32_t)s.single_pass;
    out->kernel_launches = s.launches;
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_topk_merge_device(uint32_t parts, size_t nq, uint32_t k, const float* d_dist,
                                                     size_t dist_stride, const uint64_t* d_ids, size_t ids_stride,
                                                     const uint32_t* d_counts, size_t counts_stride,
                                                     uint64_t* d_out_ids, float* d_out_distances,
                                                     uint32_t* d_out_counts, void* cuda_stream) {
    if (!d_dist || !d_ids || !d_counts || !d_out_ids || !d_out_distances || parts == 0 || parts > 64 || k == 0)
        return VESPER_ERROR_INVALID_PARAM;
    if (parts > 1 && (dist_stride < nq * k || ids_stride < nq * k || counts_stride < nq))
        return VESPER_ERROR_INVALID_PARAM;
    if (nq == 0) return VESPER_OK;
    clear_error();
    return guarded("topk_merge", [&] {
        vgpu::launch_topk_merge((int)parts, (long long)nq, (int)k, d_dist, (long long)dist_stride, d_ids,
                                (long long)ids_stride, d_counts, (long long)counts_stride, d_out_ids, d_out_distances,
                                d_out_counts, static_cast<cudaStream_t>(cuda_stream));
        return VESPER_OK;
    });
}

VESPER_C_API int vesper_b200_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

}  // extern "C"
