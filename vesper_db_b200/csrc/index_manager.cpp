// The reference's IndexManager (src/index/index_manager.cpp) for its IVF-PQ index, on
// the GPU engine, and the vesper_mgr_* C ABI over it (src/c/vesper_manager_c_api.cpp).
//
// Kept from the reference, entry point by entry point: how a build picks and trains the
// IVF-PQ index (defaults for zero parameters outside MANUAL, at most 200 000 evenly
// spaced training rows, ids = row numbers), the search parameter mapping (nprobe 0 -> 8,
// the cand_k heuristic alpha * k * log2(1 + nprobe) capped by the ceiling, the
// VESPER_USE_EXACT_RERANK / VESPER_RERANK_* overrides), tombstones on (uint32_t)id with
// the oversampled re-search (factor 1 + 1.25 * deleted / 100000, at most two nested
// re-searches), update = add another entry under the id, the memory estimates and budget
// eviction, and the on-disk layout (manifest, ivf_pq/, tombstones.bin as a CRoaring
// portable bitmap).  A batch is one GPU search; only the queries left short after the
// tombstone filter are searched again.
//
// The reference's result filter reads the id out of item.second, which for the
// manager's (id, distance) pairs is the distance (tombstone_manager.hpp:150-170), so it
// drops results whose truncated distance is a deleted id and keeps deleted ids.  This
// engine does the same by default, so that a drop-in returns the reference's results;
// VESPER_MGR_TOMBSTONE_FILTER=id filters by id instead, which is what remove() asks for.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <expected>
#include <filesystem>
#include <fstream>
#include <memory>
#include <mutex>
#include <set>
#include <shared_mutex>
#include <string>
#include <vector>

#include "../../include/vesper_b200.h"
#include "../../include/vesper_manager.h"
#include "c_error.hpp"
#include "ivf_pq_gpu.hpp"

using vesper::index::IvfPqIndex;
using vesper::index::IvfPqSearchParams;
using vesper::index::IvfPqTrainParams;
using vesper::index::SearchMode;
using vesper_c::clear_error;
using vesper_c::set_error;

namespace {

// IndexType / SelectionStrategy values (include/vesper/index/index_manager.hpp:34-45).
enum class IndexType : int32_t { HNSW = 0, IVF_PQ = 1, DiskANN = 2 };
enum class Strategy : int32_t { Auto = 0, Manual = 1, Hybrid = 2 };

// The IndexBuildConfig fields the manifest stores (index_manager.hpp:47-76).
struct BuildConfig {
    IndexType type{IndexType::HNSW};
    Strategy strategy{Strategy::Auto};
    uint64_t memory_budget_mb{1024};
    uint64_t cache_size_mb{256};
    uint32_t hnsw_M{16}, hnsw_ef{200}, hnsw_seed{42};
    IvfPqTrainParams ivf;
    uint32_t vamana_degree{64};
    float vamana_alpha{1.2f};
    uint32_t vamana_L{128};
};

struct Error {
    vesper_status_t status;
    std::string message;
};

// ------------------------------------------------------------------ roaring bitmap IO
// The portable serialization of CRoaring (the published RoaringFormatSpec): containers
// keyed by the high 16 bits, each an array (<= 4096 values, sorted u16), a 1024-word
// bitset, or a run list.  Written without runs (cookie 12346); read in every form.
constexpr uint32_t kCookieNoRun = 12346, kCookieRun = 12347;

void roaring_write(const std::set<uint32_t>& v, std::vector<char>& out) {
    std::vector<std::pair<uint16_t, std::vector<uint16_t>>> cont;
    for (uint32_t x : v) {
        const uint16_t key = (uint16_t)(x >> 16);
        if (cont.empty() || cont.back().first != key) cont.push_back({key, {}});
        cont.back().second.push_back((uint16_t)(x & 0xffff));
    }
    auto put = [&](const void* p, size_t n) {
        out.insert(out.end(), static_cast<const char*>(p), static_cast<const char*>(p) + n);
    };
    const uint32_t size = (uint32_t)cont.size();
    put(&kCookieNoRun, 4);
    put(&size, 4);
    for (auto& [key, vals] : cont) {
        const uint16_t card1 = (uint16_t)(vals.size() - 1);
        put(&key, 2);
        put(&card1, 2);
    }
    uint32_t off = 8 + 8 * size;
    for (auto& [key, vals] : cont) {
        put(&off, 4);
        off += vals.size() <= 4096 ? (uint32_t)vals.size() * 2 : 8192;
    }
    for (auto& [key, vals] : cont) {
        if (vals.size() <= 4096) {
            put(vals.data(), vals.size() * 2);
        } else {
            uint64_t words[1024] = {};
            for (uint16_t x : vals) words[x >> 6] |= 1ull << (x & 63);
            put(words, sizeof(words));
        }
    }
}

bool roaring_read(const char* p, size_t n, std::set<uint32_t>& v) {
    size_t o = 0;
    auto get = [&](void* dst, size_t k) {
        if (o + k > n) return false;
        std::memcpy(dst, p + o, k);
        o += k;
        return true;
    };
    uint32_t cookie = 0;
    if (!get(&cookie, 4)) return false;
    uint32_t size = 0;
    std::vector<uint8_t> run_flags;
    bool has_offsets = true;
    if (cookie == kCookieNoRun) {
        if (!get(&size, 4)) return false;
    } else if ((cookie & 0xffff) == kCookieRun) {
        size = (cookie >> 16) + 1;
        run_flags.resize((size + 7) / 8);
        if (!get(run_flags.data(), run_flags.size())) return false;
        has_offsets = size >= 4;
    } else {
        return false;
    }
    if (size > 65536) return false;
    std::vector<uint16_t> keys(size), card(size);
    for (uint32_t i = 0; i < size; ++i) {
        uint16_t c1 = 0;
        if (!get(&keys[i], 2) || !get(&c1, 2)) return false;
        card[i] = c1;
    }
    if (has_offsets) {
        if (o + 4ull * size > n) return false;
        o += 4ull * size;
    }
    for (uint32_t i = 0; i < size; ++i) {
        const uint32_t hi = (uint32_t)keys[i] << 16;
        const uint32_t c = (uint32_t)card[i] + 1;
        if (!run_flags.empty() && (run_flags[i / 8] >> (i % 8) & 1)) {
            uint16_t nruns = 0;
            if (!get(&nruns, 2)) return false;
            for (uint16_t r = 0; r < nruns; ++r) {
                uint16_t start = 0, len = 0;
                if (!get(&start, 2) || !get(&len, 2)) return false;
                for (uint32_t x = start; x <= (uint32_t)start + len; ++x) v.insert(hi | x);
            }
        } else if (c <= 4096) {
            for (uint32_t j = 0; j < c; ++j) {
                uint16_t x = 0;
                if (!get(&x, 2)) return false;
                v.insert(hi | x);
            }
        } else {
            uint64_t words[1024];
            if (!get(words, sizeof(words))) return false;
            for (uint32_t w = 0; w < 1024; ++w)
                for (uint64_t b = words[w]; b; b &= b - 1) v.insert(hi | (w << 6 | (uint32_t)__builtin_ctzll(b)));
        }
    }
    return true;
}

bool env_true(const char* name) {
    // parse_bool_ci (index_manager.cpp:98-108): "1" / "true" (any case) -> true
    const char* v = std::getenv(name);
    if (!v || !*v) return false;
    std::string s(v);
    std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return (char)std::tolower(c); });
    return s == "1" || s == "true";
}

}  // namespace

// ---------------------------------------------------------------------- the manager
struct vesper_manager_t {
    explicit vesper_manager_t(size_t dim) : dimension(dim) {}

    size_t dimension;
    uint64_t memory_budget_mb = 1024;
    uint64_t total_vectors = 0;
    bool needs_optimization = false;
    BuildConfig config;
    std::unique_ptr<IvfPqIndex> ivf;
    std::set<uint32_t> deleted;          // tombstones, as the reference's bitmap of (uint32_t)id
    uint64_t total_deleted = 0;          // TombstoneStats::total_deleted (never decreases)
    SearchMode mode = SearchMode::Fast;
    mutable std::atomic<uint64_t> query_count{0};
    mutable std::mutex stats_mu;
    mutable double query_ms = 0.0;    // guarded by stats_mu
    float build_seconds = 0.0f;
    mutable std::shared_mutex mu;

    uint64_t ivf_memory() const {
        // estimate_ivf_pq_memory (index_manager.cpp:1789-1793)
        return ivf ? total_vectors * 32 + 256 * (uint64_t)dimension * sizeof(float) : 0;
    }

    std::expected<void, Error> build(const float* x, size_t n, const BuildConfig& cfg);
    std::expected<void, Error> add_batch(const uint64_t* ids, const float* x, size_t n);
    std::expected<void, Error> mark_deleted(uint64_t id);
    std::expected<std::vector<std::vector<std::pair<uint64_t, float>>>, Error> search_rows(
        const float* q, const std::vector<size_t>& rows, uint32_t k, const vesper_query_config_t& qc, int depth) const;
    std::expected<void, Error> save(const std::string& dir) const;
    std::expected<void, Error> load(const std::string& dir);
    std::expected<void, Error> set_budget(uint64_t mb);
};

std::expected<void, Error> vesper_manager_t::build(const float* x, size_t n, const BuildConfig& cfg_in) {
    config = cfg_in;
    total_vectors = n;
    // Which indexes (index_manager.cpp:206-232): this engine holds IVF-PQ only.
    if (cfg_in.strategy == Strategy::Manual && cfg_in.type != IndexType::IVF_PQ)
        return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM,
                                     std::string(cfg_in.type == IndexType::HNSW ? "HNSW" : "DiskANN") +
                                         " index is not available in this engine (IVF-PQ only)"});
    if (cfg_in.strategy == Strategy::Hybrid && !(n >= 10000 && n <= 10000000))
        return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM,
                                     "hybrid selection builds IVF-PQ only for 10 000 <= n <= 10 000 000"});
    const auto t0 = std::chrono::steady_clock::now();
    // build_index(IVF_PQ) (index_manager.cpp:1682-1770)
    IvfPqTrainParams p = cfg_in.ivf;
    if (cfg_in.strategy != Strategy::Manual) {
        if (p.nlist == 0) p.nlist = n >= 1000000 ? 4096 : (n >= 100000 ? 2048 : 512);
        if (p.m == 0) p.m = dimension % 16 == 0 ? 16 : (dimension % 8 == 0 ? 8 : 4);
        if (p.nbits == 0) p.nbits = 8;
    }
    config.ivf = p;
    const size_t train_n = std::min<size_t>(n, 200000);
    std::vector<float> sub;
    const float* tx = x;
    if (train_n < n) {
        sub.resize(train_n * dimension);
        const double step = (double)n / (double)train_n;
        for (size_t t = 0; t < train_n; ++t) {
            size_t i = (size_t)((double)t * step);
            if (i >= n) i = n - 1;
            std::memcpy(sub.data() + t * dimension, x + i * dimension, dimension * sizeof(float));
        }
        tx = sub.data();
    }
    if (cfg_in.strategy != Strategy::Manual) p.max_iter = std::min<uint32_t>(p.max_iter, 20);
    auto idx = std::make_unique<IvfPqIndex>();
    auto tr = idx->train(tx, dimension, train_n, p);
    if (!tr) return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM, tr.error().message});
    std::vector<uint64_t> ids(n);
    for (size_t i = 0; i < n; ++i) ids[i] = i;
    auto ar = idx->add(ids.data(), x, n);
    if (!ar) return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM, ar.error().message});
    ivf = std::move(idx);
    build_seconds = std::chrono::duration<float>(std::chrono::steady_clock::now() - t0).count();
    return {};
}

std::expected<void, Error> vesper_manager_t::add_batch(const uint64_t* ids, const float* x, size_t n) {
    if (ivf) {
        auto r = ivf->add(ids, x, n);
        if (!r) return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM, r.error().message});
    }
    total_vectors += n;
    return {};
}

std::expected<void, Error> vesper_manager_t::mark_deleted(uint64_t id) {
    // TombstoneManager::mark_deleted (src/tombstone/tombstone_manager.cpp:27-60)
    if (!deleted.insert((uint32_t)id).second)
        return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM, "Vector already marked as deleted"});
    ++total_deleted;
    return {};
}

// IndexManager::search (index_manager.cpp:344-585) for the given query rows at k: one
// GPU search of all of them, the tombstone filter, then the oversampled re-search of the
// rows left short.
std::expected<std::vector<std::vector<std::pair<uint64_t, float>>>, Error> vesper_manager_t::search_rows(
    const float* q, const std::vector<size_t>& rows, uint32_t k, const vesper_query_config_t& qc, int depth) const {
    std::vector<std::vector<std::pair<uint64_t, float>>> res(rows.size());
    const bool prefer_other = qc.has_preferred_index && qc.preferred_index != VESPER_INDEX_IVF_PQ;
    if (ivf && !prefer_other && !rows.empty()) {
        // rerank controls and their environment overrides (index_manager.cpp:110-134, 393-436)
        bool use_exact = qc.use_exact_rerank != 0;
        uint32_t rerank_k = qc.rerank_k;
        float alpha = qc.rerank_alpha;
        uint32_t ceil_val = qc.rerank_cand_ceiling;
        if (const char* v = std::getenv("VESPER_USE_EXACT_RERANK"); v && *v) use_exact = env_true("VESPER_USE_EXACT_RERANK");
        if (const char* v = std::getenv("VESPER_RERANK_K"); v && *v) {
            try { rerank_k = (uint32_t)std::stoull(v); } catch (...) {}
        }
        if (const char* v = std::getenv("VESPER_RERANK_ALPHA"); v && *v) {
            try { alpha = std::stof(v); } catch (...) {}
        }
        if (const char* v = std::getenv("VESPER_RERANK_CEIL"); v && *v) {
            try { ceil_val = (uint32_t)std::stoull(v); } catch (...) {}
        }
        if (!(alpha > 0.0f) || !std::isfinite(alpha)) alpha = 2.0f;
        IvfPqSearchParams sp;
        sp.k = k;
        sp.nprobe = qc.nprobe > 0 ? qc.nprobe : 8;
        sp.mode = mode;
        uint32_t cand_k = 0;
        if (use_exact) {
            if (rerank_k > 0) {
                cand_k = rerank_k;
            } else {
                const double base = (double)k, probe = (double)sp.nprobe;
                const double h = std::max(base, (double)alpha * base * std::log2(1.0 + probe));
                cand_k = (uint32_t)std::ceil(h);
                if (ceil_val > 0) cand_k = std::min<uint32_t>(cand_k, ceil_val);
            }
        }
        sp.cand_k = cand_k;
        sp.use_exact_rerank = use_exact;
        sp.rerank_k = rerank_k > 0 ? rerank_k : cand_k;
        const size_t nq = rows.size(), d = dimension;
        std::vector<float> qs(nq * d);
        for (size_t i = 0; i < nq; ++i) std::memcpy(qs.data() + i * d, q + rows[i] * d, d * sizeof(float));
        std::vector<uint64_t> ids(nq * (size_t)k);
        std::vector<float> dist(nq * (size_t)k);
        std::vector<uint32_t> cnt(nq);
        auto r = ivf->search_batch_flat(qs.data(), nq, sp, ids.data(), dist.data(), cnt.data(), false);
        if (!r) return std::unexpected(Error{VESPER_ERROR_INVALID_PARAM, r.error().message});
        for (size_t i = 0; i < nq; ++i)
            for (uint32_t j = 0; j < cnt[i]; ++j) res[i].emplace_back(ids[i * k + j], dist[i * k + j]);
    }
    // tombstones (index_manager.cpp:552-576, tombstone_manager.hpp:150-170)
    const bool by_distance = [] {
        const char* v = std::getenv("VESPER_MGR_TOMBSTONE_FILTER");
        return !(v && std::string(v) == "id");
    }();
    std::vector<size_t> short_rows, short_pos;
    for (size_t i = 0; i < res.size(); ++i) {
        if (!deleted.empty()) {
            auto& r = res[i];
            r.erase(std::remove_if(r.begin(), r.end(),
                                   [&](const std::pair<uint64_t, float>& e) {
                                       const uint32_t key = by_distance ? (uint32_t)e.second : (uint32_t)e.first;
                                       return deleted.count(key) != 0;
                                   }),
                    r.end());
        }
        if (res[i].size() < k) {
            short_rows.push_back(rows[i]);
            short_pos.push_back(i);
        }
    }
    // get_oversampling_factor (tombstone_manager.cpp:345-351)
    const float factor = (float)(1.0 + ((double)total_deleted / 100000.0) * 1.25);
    if (!short_rows.empty() && factor > 1.0f && depth < 2) {
        const uint32_t k2 = (uint32_t)((float)k * factor * 1.5f);
        auto again = search_rows(q, short_rows, k2, qc, depth + 1);
        if (again)
            for (size_t j = 0; j < short_rows.size(); ++j)
                if ((*again)[j].size() >= k) res[short_pos[j]] = std::move((*again)[j]);
    }
    for (auto& r : res)
        if (r.size() > k) r.resize(k);
    return res;
}

std::expected<void, Error> vesper_manager_t::set_budget(uint64_t mb) {
    // set_memory_budget + enforce_memory_budget (index_manager.cpp:1375-1388, 1444-1600):
    // over budget, the IVF-PQ index is evicted.
    memory_budget_mb = mb;
    const uint64_t cur = ivf_memory() / (1024 * 1024);
    if (cur <= mb) return {};
    ivf.reset();
    needs_optimization = true;
    return {};
}

std::expected<void, Error> vesper_manager_t::save(const std::string& dir) const {
    namespace fs = std::filesystem;
    std::error_code ec;
    fs::create_directories(dir, ec);
    if (ec) return std::unexpected(Error{VESPER_ERROR_IO, "Failed to create directory: " + ec.message()});
    {
        // manifest (index_manager.cpp:1114-1161): fields in their in-memory widths
        std::ofstream f(dir + "/index_manager.manifest", std::ios::binary);
        if (!f) return std::unexpected(Error{VESPER_ERROR_IO, "Failed to create manifest file"});
        auto put = [&](const auto& v) { f.write(reinterpret_cast<const char*>(&v), sizeof(v)); };
        put(uint32_t{1});
        put((uint64_t)dimension);
        put(total_vectors);
        put(memory_budget_mb);
        put(needs_optimization);
        put(config.strategy);
        put(config.type);
        put(config.memory_budget_mb);
        put(config.cache_size_mb);
        put(config.hnsw_M);
        put(config.hnsw_ef);
        put(config.hnsw_seed);
        put(config.ivf.nlist);
        put(config.ivf.m);
        put(config.ivf.nbits);
        put(config.vamana_degree);
        put(config.vamana_alpha);
        put(config.vamana_L);
        put(false);
        put((bool)ivf);
        put(false);
        if (!f) return std::unexpected(Error{VESPER_ERROR_IO, "Failed writing manifest"});
    }
    if (ivf) {
        auto r = ivf->save(dir + "/ivf_pq");
        if (!r) return std::unexpected(Error{VESPER_ERROR_IO, r.error().message});
    }
    // TombstoneManager::save (tombstone_manager.cpp:196-236): version, size, bitmap
    std::vector<char> bm;
    roaring_write(deleted, bm);
    std::ofstream t(dir + "/tombstones.bin", std::ios::binary);
    if (!t) return std::unexpected(Error{VESPER_ERROR_IO, "Failed to open file for writing"});
    const uint32_t version = 1;
    const uint64_t sz = bm.size();
    t.write(reinterpret_cast<const char*>(&version), 4);
    t.write(reinterpret_cast<const char*>(&sz), 8);
    t.write(bm.data(), (std::streamsize)bm.size());
    if (!t) return std::unexpected(Error{VESPER_ERROR_IO, "Failed writing tombstones"});
    return {};
}

std::expected<void, Error> vesper_manager_t::load(const std::string& dir) {
    namespace fs = std::filesystem;
    // IndexManager::load (index_manager.cpp:1193-1346)
    if (!fs::exists(dir)) return std::unexpected(Error{VESPER_ERROR_IO, "Index directory not found: " + dir});
    const std::string mpath = dir + "/index_manager.manifest";
    std::ifstream f(mpath, std::ios::binary);
    if (!f) return std::unexpected(Error{VESPER_ERROR_IO, "Manifest file not found: " + mpath});
    auto get = [&](auto& v) { f.read(reinterpret_cast<char*>(&v), sizeof(v)); };
    uint32_t version = 0;
    get(version);
    if (version != 1)
        return std::unexpected(Error{VESPER_ERROR_IO, "Unsupported manifest version: " + std::to_string(version)});
    uint64_t dim = 0, total = 0, budget = 0;
    bool needs_opt = false;
    BuildConfig c;
    get(dim);
    get(total);
    get(budget);
    get(needs_opt);
    get(c.strategy);
    get(c.type);
    get(c.memory_budget_mb);
    get(c.cache_size_mb);
    get(c.hnsw_M);
    get(c.hnsw_ef);
    get(c.hnsw_seed);
    get(c.ivf.nlist);
    get(c.ivf.m);
    get(c.ivf.nbits);
    get(c.vamana_degree);
    get(c.vamana_alpha);
    get(c.vamana_L);
    bool has_hnsw = false, has_ivf = false, has_disk = false;
    get(has_hnsw);
    get(has_ivf);
    get(has_disk);
    if (!f.good()) return std::unexpected(Error{VESPER_ERROR_IO, "Failed to read manifest file"});
    if (has_hnsw || has_disk)
        return std::unexpected(Error{VESPER_ERROR_IO, std::string("Manifest lists a") +
                                                          (has_hnsw ? "n HNSW" : " DiskGraph") +
                                                          " index, which this engine (IVF-PQ only) cannot load"});
    std::unique_ptr<IvfPqIndex> idx;
    if (has_ivf) {
        auto r = IvfPqIndex::load(dir + "/ivf_pq");
        if (!r) return std::unexpected(Error{VESPER_ERROR_IO, "Failed to load IVF-PQ index: " + r.error().message});
        idx = std::make_unique<IvfPqIndex>(std::move(*r));
    }
    std::set<uint32_t> del;
    if (fs::exists(dir + "/tombstones.bin")) {
        std::ifstream t(dir + "/tombstones.bin", std::ios::binary);
        uint32_t tv = 0;
        uint64_t sz = 0;
        t.read(reinterpret_cast<char*>(&tv), 4);
        if (!t || tv != 1)
            return std::unexpected(Error{VESPER_ERROR_IO, "Failed to load tombstone data: Unsupported tombstone file version"});
        t.read(reinterpret_cast<char*>(&sz), 8);
        std::vector<char> buf(t ? sz : 0);
        if (!t || !t.read(buf.data(), (std::streamsize)sz) || !roaring_read(buf.data(), buf.size(), del))
            return std::unexpected(Error{VESPER_ERROR_IO, "Failed to load tombstone data: bad bitmap"});
    }
    dimension = dim;
    total_vectors = total;
    memory_budget_mb = budget;
    needs_optimization = needs_opt;
    config = c;
    ivf = std::move(idx);
    deleted = std::move(del);
    total_deleted = 0;  // a loaded TombstoneManager starts its statistics at zero
    return {};
}

// ---------------------------------------------------------------------- C ABI
namespace {

template <class F>
vesper_status_t guarded_mgr(const char* what, F&& f) {
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

vesper_status_t report(const Error& e) {
    set_error(e.message);
    return e.status;
}

// to_query_config (src/c/vesper_manager_c_api.cpp:179-210), the filter part.
bool check_filter(const vesper_query_config_t* qc) {
    if (!qc->has_filter) return true;
    if (!qc->filter_json) {
        set_error("has_filter=1 but filter_json is NULL");
        return false;
    }
    set_error("metadata filters are not available in this engine (IVF-PQ only)");
    return false;
}

vesper_status_t mgr_search(const vesper_manager_t* mgr, const float* queries, size_t nq,
                           const vesper_query_config_t* qc, uint64_t* out_ids, float* out_dists) {
    if (!check_filter(qc)) return VESPER_ERROR_INVALID_PARAM;
    const auto t0 = std::chrono::steady_clock::now();
    std::shared_lock lock(mgr->mu);
    if (!mgr->ivf) {
        set_error("No suitable index available");
        return VESPER_ERROR_INVALID_PARAM;
    }
    std::vector<size_t> rows(nq);
    for (size_t i = 0; i < nq; ++i) rows[i] = i;
    auto r = mgr->search_rows(queries, rows, qc->k, *qc, 0);
    if (!r) return report(r.error());
    // padding (vesper_manager_c_api.cpp:227-234)
    const size_t k = qc->k;
    for (size_t qi = 0; qi < nq; ++qi) {
        const auto& row = (*r)[qi];
        const size_t take = std::min(row.size(), k);
        for (size_t i = 0; i < take; ++i) {
            out_ids[qi * k + i] = row[i].first;
            out_dists[qi * k + i] = row[i].second;
        }
        for (size_t i = take; i < k; ++i) {
            out_ids[qi * k + i] = 0;
            out_dists[qi * k + i] = take > 0 ? row[take - 1].second : 0.0f;
        }
    }
    mgr->query_count += nq;
    std::lock_guard<std::mutex> sl(mgr->stats_mu);
    mgr->query_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    return VESPER_OK;
}

}  // namespace

extern "C" {

VESPER_C_API vesper_status_t vesper_mgr_create(size_t dim, vesper_manager_t** out_mgr) {
    if (!out_mgr || dim == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_create", [&] {
        *out_mgr = new vesper_manager_t(dim);
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_mgr_destroy(vesper_manager_t* mgr) {
    clear_error();
    return guarded_mgr("vesper_mgr_destroy", [&] {
        delete mgr;
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_mgr_build(vesper_manager_t* mgr, const float* base_vectors, size_t n,
                                              const vesper_manager_build_config_t* cfg) {
    if (!mgr || !base_vectors || n == 0 || !cfg) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_build", [&] {
        BuildConfig c;
        c.type = cfg->type == VESPER_INDEX_HNSW ? IndexType::HNSW
                 : cfg->type == VESPER_INDEX_DISKANN ? IndexType::DiskANN : IndexType::IVF_PQ;
        c.strategy = cfg->strategy == VESPER_SELECT_AUTO ? Strategy::Auto
                     : cfg->strategy == VESPER_SELECT_HYBRID ? Strategy::Hybrid : Strategy::Manual;
        c.ivf.nlist = cfg->ivf.nlist;
        c.ivf.m = cfg->ivf.m;
        c.ivf.nbits = cfg->ivf.nbits;
        c.hnsw_M = cfg->hnsw.M;
        c.hnsw_ef = cfg->hnsw.ef_construction;
        c.hnsw_seed = cfg->hnsw.seed;
        c.vamana_degree = cfg->vamana.degree;
        c.vamana_L = cfg->vamana.L;
        c.vamana_alpha = cfg->vamana.alpha;
        std::unique_lock lock(mgr->mu);
        auto r = mgr->build(base_vectors, n, c);
        return r ? VESPER_OK : report(r.error());
    });
}

VESPER_C_API vesper_status_t vesper_mgr_add_batch(vesper_manager_t* mgr, const uint64_t* ids, const float* vectors,
                                                  size_t n) {
    if (!mgr || !ids || !vectors || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_add_batch", [&] {
        std::unique_lock lock(mgr->mu);
        auto r = mgr->add_batch(ids, vectors, n);
        return r ? VESPER_OK : report(r.error());
    });
}

// update / update_batch (index_manager.cpp:612-784): the id is tombstoned, a new entry is
// added under it, and the tombstone is lifted again, so the old entry stays searchable.
VESPER_C_API vesper_status_t vesper_mgr_update_batch(vesper_manager_t* mgr, const uint64_t* ids,
                                                     const float* vectors, size_t n) {
    if (!mgr || !ids || !vectors || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_update_batch", [&] {
        std::unique_lock lock(mgr->mu);
        std::vector<uint32_t> marked;
        for (size_t i = 0; i < n; ++i) {
            auto r = mgr->mark_deleted(ids[i]);
            if (!r) {
                for (uint32_t t : marked) mgr->deleted.erase(t);
                return report(r.error());
            }
            marked.push_back((uint32_t)ids[i]);
        }
        vesper_status_t st = VESPER_OK;
        if (mgr->ivf) {
            auto r = mgr->ivf->add(ids, vectors, n);
            if (!r) {
                set_error(r.error().message);
                st = VESPER_ERROR_INVALID_PARAM;
            }
        }
        for (uint32_t t : marked) mgr->deleted.erase(t);
        return st;
    });
}

VESPER_C_API vesper_status_t vesper_mgr_update(vesper_manager_t* mgr, uint64_t id, const float* vector) {
    if (!mgr || !vector) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    {
        std::shared_lock lock(mgr->mu);
        if (!mgr->ivf) {
            set_error("Vector ID not found in any index");
            return VESPER_ERROR_INVALID_PARAM;
        }
    }
    return vesper_mgr_update_batch(mgr, &id, vector, 1);
}

VESPER_C_API vesper_status_t vesper_mgr_remove(vesper_manager_t* mgr, uint64_t id) {
    if (!mgr) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_remove", [&] {
        std::unique_lock lock(mgr->mu);
        auto r = mgr->mark_deleted(id);
        return r ? VESPER_OK : report(r.error());
    });
}

VESPER_C_API vesper_status_t vesper_mgr_remove_batch(vesper_manager_t* mgr, const uint64_t* ids, size_t n) {
    if (!mgr || !ids || n == 0) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_remove_batch", [&] {
        std::unique_lock lock(mgr->mu);
        for (size_t i = 0; i < n; ++i) {
            auto r = mgr->mark_deleted(ids[i]);
            if (!r) return report(r.error());
        }
        return VESPER_OK;
    });
}

VESPER_C_API vesper_status_t vesper_mgr_search(const vesper_manager_t* mgr, const float* query,
                                               const vesper_query_config_t* qc, uint64_t* out_ids, float* out_dists) {
    if (!mgr || !query || !qc || !out_ids || !out_dists) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_search", [&] { return mgr_search(mgr, query, 1, qc, out_ids, out_dists); });
}

VESPER_C_API vesper_status_t vesper_mgr_search_batch(const vesper_manager_t* mgr, const float* queries, size_t nq,
                                                     const vesper_query_config_t* qc, uint64_t* out_ids,
                                                     float* out_dists) {
    if (!mgr || !queries || nq == 0 || !qc || !out_ids || !out_dists) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_search_batch",
                       [&] { return mgr_search(mgr, queries, nq, qc, out_ids, out_dists); });
}

VESPER_C_API vesper_status_t vesper_mgr_save(const vesper_manager_t* mgr, const char* dir_path) {
    if (!mgr || !dir_path) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_save", [&] {
        std::shared_lock lock(mgr->mu);
        auto r = mgr->save(dir_path);
        return r ? VESPER_OK : report(r.error());
    });
}

VESPER_C_API vesper_status_t vesper_mgr_load(vesper_manager_t* mgr, const char* dir_path) {
    if (!mgr || !dir_path) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_load", [&] {
        std::unique_lock lock(mgr->mu);
        auto r = mgr->load(dir_path);
        return r ? VESPER_OK : report(r.error());
    });
}

VESPER_C_API vesper_status_t vesper_mgr_memory_usage(const vesper_manager_t* mgr, size_t* out_bytes) {
    if (!mgr || !out_bytes) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    std::shared_lock lock(mgr->mu);
    *out_bytes = mgr->ivf_memory();
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_mgr_disk_usage(const vesper_manager_t* mgr, size_t* out_bytes) {
    if (!mgr || !out_bytes) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    *out_bytes = 0;  // disk_usage counts DiskGraph indexes only (index_manager.cpp:1365-1373)
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_mgr_set_memory_budget_mb(vesper_manager_t* mgr, uint32_t mb) {
    if (!mgr) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    return guarded_mgr("vesper_mgr_set_memory_budget_mb", [&] {
        std::unique_lock lock(mgr->mu);
        auto r = mgr->set_budget(mb);
        return r ? VESPER_OK : report(r.error());
    });
}

VESPER_C_API vesper_status_t vesper_mgr_get_memory_budget_mb(const vesper_manager_t* mgr, uint32_t* out_mb) {
    if (!mgr || !out_mb) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    std::shared_lock lock(mgr->mu);
    *out_mb = (uint32_t)mgr->memory_budget_mb;
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_mgr_get_stats(const vesper_manager_t* mgr, vesper_index_stats_t* out_stats,
                                                  size_t* inout_capacity, size_t* out_count) {
    if (!mgr || !out_count) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    std::shared_lock lock(mgr->mu);
    *out_count = mgr->ivf ? 1 : 0;
    if (!out_stats) return VESPER_OK;
    if (!inout_capacity) {
        set_error("inout_capacity must be provided when out_stats is non-NULL");
        return VESPER_ERROR_INVALID_PARAM;
    }
    if (mgr->ivf && *inout_capacity >= 1) {
        vesper_index_stats_t& s = out_stats[0];
        s.type = VESPER_INDEX_IVF_PQ;
        s.num_vectors = mgr->total_vectors;
        s.memory_usage_bytes = mgr->ivf_memory();
        s.disk_usage_bytes = 0;
        s.build_time_seconds = mgr->build_seconds;
        const uint64_t qn = mgr->query_count.load();
        {
            std::lock_guard<std::mutex> sl(mgr->stats_mu);
            s.avg_query_time_ms = (float)(mgr->query_ms / (double)std::max<uint64_t>(1, qn));
        }
        s.measured_recall = 0.0f;
        s.query_count = qn;
    }
    return VESPER_OK;
}

VESPER_C_API vesper_status_t vesper_mgr_set_search_mode(vesper_manager_t* mgr, uint32_t mode) {
    if (!mgr || mode > VESPER_SEARCH_EXACT) return VESPER_ERROR_INVALID_PARAM;
    clear_error();
    std::unique_lock lock(mgr->mu);
    mgr->mode = mode == VESPER_SEARCH_EXACT ? SearchMode::Exact : SearchMode::Fast;
    return VESPER_OK;
}

}  // extern "C"
