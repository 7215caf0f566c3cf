// Oracle: CPU restatement of the reference IVF-PQ / PQ / k-means arithmetic.
//
// TEST INFRASTRUCTURE ONLY -- the checker, never the thing measured or shipped.
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
//
// Every function restates the reference routine it cites (paths relative to the
// Vesper source tree) with the same operation order, so results are bit-identical to
// the reference compiled with -ffp-contract=off:
//   * l2 / inner product: 8 FMA lane accumulators over floor(n/8)*8 elements, the
//     hsum ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)), then a rounded-multiply/add scalar tail.
//   * arg-min scans use a strict `<` from FLT_MAX, so the lowest index wins ties.
//   * sequential fp32 ADC sums in sub-quantizer order; sequential fp32 rotation dots.
// Built with -ffp-contract=off so the compiler cannot fuse any multiply/add that the
// reference leaves separate; the lane FMAs are explicit std::fma calls.
#include "vesper_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <queue>
#include <random>
#include <utility>
#include <vector>

namespace {

// avx2_l2_sq (include/vesper/kernels/backends/avx2.hpp:76-108) and hsum_ps (:37-46).
inline float l2_lanes(const float* a, const float* b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const size_t simd_end = n & ~size_t(7);
    size_t i = 0;
    for (; i < simd_end; i += 8) {
        for (int l = 0; l < 8; ++l) {
            const float d = a[i + l] - b[i + l];
            acc[l] = std::fma(d, d, acc[l]);
        }
    }
    const float s0 = acc[4] + acc[0], s1 = acc[5] + acc[1];
    const float s2 = acc[6] + acc[2], s3 = acc[7] + acc[3];
    float result = (s0 + s1) + (s2 + s3);
    for (; i < n; ++i) {
        const float d = a[i] - b[i];
        const float sq = d * d;
        result = result + sq;
    }
    return result;
}

// avx2_inner_product (include/vesper/kernels/backends/avx2.hpp:124-154).
inline float ip_lanes(const float* a, const float* b, size_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const size_t simd_end = n & ~size_t(7);
    size_t i = 0;
    for (; i < simd_end; i += 8)
        for (int l = 0; l < 8; ++l) acc[l] = std::fma(a[i + l], b[i + l], acc[l]);
    const float s0 = acc[4] + acc[0], s1 = acc[5] + acc[1];
    const float s2 = acc[6] + acc[2], s3 = acc[7] + acc[3];
    float result = (s0 + s1) + (s2 + s3);
    for (; i < n; ++i) {
        const float p = a[i] * b[i];
        result = result + p;
    }
    return result;
}

// TopKBuffer (src/index/ivf_pq.cpp:163-198): the heapless top-k for pool_k <= 64.
struct TopKBuffer {
    explicit TopKBuffer(size_t K) : K_(K), dists(K, std::numeric_limits<float>::infinity()), ids(K, 0) {}
    void consider(float dist, uint64_t id) {
        if (count_ < K_) {
            dists[count_] = dist; ids[count_] = id;
            if (count_ == 0 || dist > worst_val_) { worst_val_ = dist; worst_idx_ = count_; }
            ++count_;
            return;
        }
        if (dist >= worst_val_) return;
        dists[worst_idx_] = dist; ids[worst_idx_] = id;
        worst_idx_ = 0; worst_val_ = dists[0];
        for (size_t i = 1; i < K_; ++i)
            if (dists[i] > worst_val_) { worst_val_ = dists[i]; worst_idx_ = i; }
    }
    std::vector<std::pair<uint64_t, float>> sorted() const {
        std::vector<std::pair<uint64_t, float>> out;
        for (size_t i = 0; i < count_; ++i) out.emplace_back(ids[i], dists[i]);
        std::sort(out.begin(), out.end(), [](const auto& a, const auto& b) { return a.second < b.second; });
        return out;
    }
    size_t K_, count_ = 0;
    std::vector<float> dists;
    std::vector<uint64_t> ids;
    size_t worst_idx_ = 0;
    float worst_val_ = std::numeric_limits<float>::infinity();
};

// find_nearest_centroids (src/index/ivf_pq.cpp:3442-3474): partial_sort of
// pair<float, uint32> -> ordered by (distance, list index).
void coarse_probe_one(const float* q, const float* c, uint32_t nlist, size_t dim, uint32_t nprobe,
                      std::vector<std::pair<float, uint32_t>>& out) {
    nprobe = std::min(nprobe, nlist);
    std::vector<std::pair<float, uint32_t>> d;
    d.reserve(nlist);
    for (uint32_t i = 0; i < nlist; ++i) d.emplace_back(l2_lanes(q, c + size_t(i) * dim, dim), i);
    std::partial_sort(d.begin(), d.begin() + nprobe, d.end());
    out.assign(d.begin(), d.begin() + nprobe);
}

// apply_rotation (src/index/ivf_pq.cpp:2947-2968): out[j] = sum_k in[k] * R[k*d + j],
// accumulated sequentially in k with a rounded product then a rounded add.
void rotate_one(const float* in, const float* R, size_t dim, float* out) {
    for (size_t j = 0; j < dim; ++j) {
        float sum = 0.0f;
        for (size_t k = 0; k < dim; ++k) {
            const float p = in[k] * R[k * dim + j];
            sum = sum + p;
        }
        out[j] = sum;
    }
}

// find_nearest_code (src/index/pq_fastscan.cpp:78-99).
inline uint8_t nearest_code(const float* v, const float* cb_sub, uint32_t ksub, size_t dsub) {
    float best = std::numeric_limits<float>::max();
    uint8_t code = 0;
    for (uint32_t j = 0; j < ksub; ++j) {
        const float d = l2_lanes(v, cb_sub + size_t(j) * dsub, dsub);
        if (d < best) { best = d; code = static_cast<uint8_t>(j); }
    }
    return code;
}

// compute_lookup_tables (src/index/pq_fastscan.cpp:145-172).
void lut_one(const float* r, const float* cb, uint32_t m, uint32_t ksub, size_t dsub, float* lut) {
    for (uint32_t s = 0; s < m; ++s)
        for (uint32_t j = 0; j < ksub; ++j)
            lut[size_t(s) * ksub + j] = l2_lanes(r + s * dsub, cb + (size_t(s) * ksub + j) * dsub, dsub);
}

// accumulate_distances_avx2 (include/vesper/index/pq_fastscan.hpp:284-317): a running
// sum that starts at 0.0f and adds one LUT entry per sub-quantizer, in order.
inline float adc_one(const float* lut, const uint8_t* code, uint32_t m, uint32_t ksub) {
    float d = 0.0f;
    for (uint32_t s = 0; s < m; ++s) d = d + lut[size_t(s) * ksub + code[s]];
    return d;
}

// Exact rerank of the head of a search result (src/index/ivf_pq.cpp:3995-4091): each
// candidate's entry is the first one in list order holding its id; the vector is
// rebuilt as centroid + apply_rotation_T(decode(code)) (rounded adds), its squared
// distance to q summed sequentially with rounded products and adds; the head is
// re-sorted by that distance (std::sort in the reference: order among exact ties is
// unspecified; stable here) and the result trimmed to k.
void rerank_one(const float* q, const float* c, size_t dim, const float* R, const float* cb,
                uint32_t m, uint32_t ksub, uint32_t nlist, const uint64_t* offs, const uint64_t* ids,
                const uint8_t* codes, size_t head, std::vector<std::pair<uint64_t, float>>& res) {
    const size_t dsub = dim / m;
    std::vector<float> rc(dim), ro(dim);
    for (size_t i = 0; i < head; ++i) {
        const uint64_t id = res[i].first;
        uint64_t e = offs[nlist];
        for (uint64_t j = 0; j < offs[nlist]; ++j)
            if (ids[j] == id) { e = j; break; }
        if (e == offs[nlist]) continue;
        const uint32_t l = static_cast<uint32_t>(std::upper_bound(offs, offs + nlist + 1, e) - offs - 1);
        for (uint32_t s = 0; s < m; ++s) {
            const float* cw = cb + (size_t(s) * ksub + codes[e * m + s]) * dsub;
            std::copy(cw, cw + dsub, rc.begin() + size_t(s) * dsub);
        }
        const float* res_v = rc.data();
        if (R) {
            // apply_rotation_T (src/index/ivf_pq.cpp:5369-5390)
            for (size_t j = 0; j < dim; ++j) {
                float sum = 0.0f;
                for (size_t t = 0; t < dim; ++t) {
                    const float p = rc[t] * R[j * dim + t];
                    sum = sum + p;
                }
                ro[j] = sum;
            }
            res_v = ro.data();
        }
        const float* cl = c + size_t(l) * dim;
        float dist = 0.0f;
        for (size_t d = 0; d < dim; ++d) {
            const float rec = cl[d] + res_v[d];
            const float diff = q[d] - rec;
            const float p = diff * diff;
            dist = dist + p;
        }
        res[i].second = dist;
    }
    std::stable_sort(res.begin(), res.begin() + head,
                     [](const auto& a, const auto& b) { return a.second < b.second; });
}

uint32_t search_one(const float* q, const float* c, uint32_t nlist, size_t dim, const float* R,
                    const float* cb, uint32_t m, uint32_t ksub, const uint64_t* offs,
                    const uint64_t* ids, const uint8_t* codes, uint32_t k, uint32_t nprobe,
                    uint32_t cand_k, bool rerank, uint32_t rerank_k, uint64_t* out_ids, float* out_d) {
    // Impl::search (src/index/ivf_pq.cpp:3491-4094).  Candidate pool (:3544-3552):
    // pool_k = max(k, cand_k or k), with rerank also >= rerank_k or max(3k, 1000);
    // TopKBuffer for pool_k <= 64, else a max-heap of (dist, id).
    std::vector<std::pair<float, uint32_t>> probe;
    coarse_probe_one(q, c, nlist, dim, nprobe, probe);
    const size_t dsub = dim / m;
    size_t pool_k = std::max<uint32_t>(k, cand_k > 0 ? cand_k : k);
    if (rerank) pool_k = std::max<size_t>(pool_k, rerank_k > 0 ? rerank_k : std::max<uint32_t>(k * 3, 1000));
    const bool heapless = pool_k <= 64;
    TopKBuffer topk(pool_k);
    std::priority_queue<std::pair<float, uint64_t>> heap;
    std::vector<float> r(dim), rr(dim), lut(size_t(m) * ksub);
    for (const auto& pr : probe) {
        const uint32_t l = pr.second;
        const float* cl = c + size_t(l) * dim;
        for (size_t d = 0; d < dim; ++d) r[d] = q[d] - cl[d];
        const float* rq = r.data();
        if (R) { rotate_one(r.data(), R, dim, rr.data()); rq = rr.data(); }
        lut_one(rq, cb, m, ksub, dsub, lut.data());
        for (uint64_t e = offs[l]; e < offs[l + 1]; ++e) {
            const float dist = adc_one(lut.data(), codes + e * m, m, ksub);
            if (heapless) {
                topk.consider(dist, ids[e]);
            } else if (heap.size() < pool_k) {
                heap.emplace(dist, ids[e]);
            } else if (dist < heap.top().first) {
                heap.pop();
                heap.emplace(dist, ids[e]);
            }
        }
    }
    std::vector<std::pair<uint64_t, float>> res;
    if (heapless) {
        res = topk.sorted();
    } else {
        while (!heap.empty()) { res.emplace_back(heap.top().second, heap.top().first); heap.pop(); }
        std::reverse(res.begin(), res.end());
    }
    if (rerank && !res.empty()) {
        const size_t head = std::min<size_t>(rerank_k > 0 ? rerank_k : pool_k, res.size());
        rerank_one(q, c, dim, R, cb, m, ksub, nlist, offs, ids, codes, head, res);
    }
    const uint32_t take = static_cast<uint32_t>(std::min<size_t>(res.size(), k));
    for (uint32_t i = 0; i < take; ++i) { out_ids[i] = res[i].first; out_d[i] = res[i].second; }
    return take;
}

// update_centroid (src/index/kmeans_elkan.cpp:31-56): Kahan-compensated fp64 sum of
// the cluster's points in point order, times (1/count), rounded to fp32.  An empty
// cluster keeps its previous centroid.
void elkan_update_one(const float* x, size_t dim, const std::vector<size_t>& idx, float* cen) {
    if (idx.empty()) return;
    std::vector<double> sum(dim, 0.0), comp(dim, 0.0);
    for (size_t i : idx) {
        const float* p = x + i * dim;
        for (size_t d = 0; d < dim; ++d) {
            const double y = p[d] - comp[d];
            const double t = sum[d] + y;
            comp[d] = (t - sum[d]) - y;
            sum[d] = t;
        }
    }
    const double scale = 1.0 / static_cast<double>(idx.size());
    for (size_t d = 0; d < dim; ++d) cen[d] = static_cast<float>(sum[d] * scale);
}

void kmeanspp(const float* x, size_t n, size_t dim, uint32_t k, uint32_t seed, float* out_c,
              uint32_t* out_idx) {
    // kmeans_plusplus_init (src/index/kmeans.cpp:45-89): std::mt19937(seed); first pick
    // uniform_int_distribution<size_t>(0, n-1); then D^2 sampling on a sequential fp64
    // cumulative sum with uniform_real_distribution<double>(0, total) and lower_bound.
    std::mt19937 gen(seed);
    std::uniform_int_distribution<size_t> first(0, n - 1);
    size_t idx = first(gen);
    std::memcpy(out_c, x + idx * dim, dim * 4);
    if (out_idx) out_idx[0] = static_cast<uint32_t>(idx);
    std::vector<float> mind(n, std::numeric_limits<float>::max());
    std::vector<double> cum(n);
    for (uint32_t c = 1; c < k; ++c) {
        const float* last = out_c + size_t(c - 1) * dim;
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)n; ++i) {
            const float d = l2_lanes(x + size_t(i) * dim, last, dim);
            mind[i] = std::min(mind[i], d);
        }
        cum[0] = mind[0];
        for (size_t i = 1; i < n; ++i) cum[i] = cum[i - 1] + mind[i];
        std::uniform_real_distribution<double> sd(0.0, cum.back());
        const double target = sd(gen);
        idx = static_cast<size_t>(std::lower_bound(cum.begin(), cum.end(), target) - cum.begin());
        std::memcpy(out_c + size_t(c) * dim, x + idx * dim, dim * 4);
        if (out_idx) out_idx[c] = static_cast<uint32_t>(idx);
    }
}

}  // namespace

extern "C" {

float orc_l2_sq(const float* a, const float* b, size_t n) { return l2_lanes(a, b, n); }
float orc_inner_product(const float* a, const float* b, size_t n) { return ip_lanes(a, b, n); }

// Brute coarse assignment (src/index/ivf_pq.cpp:3252-3265 and the residual passes
// :477-494, :2414-2432): strict `<` from FLT_MAX, lowest index wins ties.
void orc_assign(const float* x, size_t n, const float* c, uint32_t k, size_t dim, uint32_t* out,
                float* out_dist) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        float best = std::numeric_limits<float>::max();
        uint32_t bi = 0;
        for (uint32_t j = 0; j < k; ++j) {
            const float d = l2_lanes(x + size_t(i) * dim, c + size_t(j) * dim, dim);
            if (d < best) { best = d; bi = j; }
        }
        out[i] = bi;
        if (out_dist) out_dist[i] = best;
    }
}

void orc_coarse_probe(const float* q, size_t nq, const float* c, uint32_t nlist, size_t dim,
                      uint32_t nprobe, uint32_t* out_lists, float* out_d) {
    const uint32_t np = std::min(nprobe, nlist);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)nq; ++i) {
        std::vector<std::pair<float, uint32_t>> p;
        coarse_probe_one(q + size_t(i) * dim, c, nlist, dim, nprobe, p);
        for (uint32_t j = 0; j < np; ++j) {
            out_lists[size_t(i) * np + j] = p[j].second;
            out_d[size_t(i) * np + j] = p[j].first;
        }
    }
}

void orc_rotate(const float* in, const float* R, size_t n, size_t dim, float* out) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) rotate_one(in + size_t(i) * dim, R, dim, out + size_t(i) * dim);
}

// apply_rotation_T (src/index/ivf_pq.cpp:5369-5390): out[k] = sum_j in[j] * R[k*d + j].
void orc_rotate_T(const float* in, const float* R, size_t n, size_t dim, float* out) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        const float* v = in + size_t(i) * dim;
        for (size_t k = 0; k < dim; ++k) {
            float sum = 0.0f;
            for (size_t j = 0; j < dim; ++j) {
                const float p = v[j] * R[k * dim + j];
                sum = sum + p;
            }
            out[size_t(i) * dim + k] = sum;
        }
    }
}

// FastScanPq::encode (src/index/pq_fastscan.cpp:101-116).
void orc_pq_encode(const float* x, size_t n, const float* cb, uint32_t m, uint32_t ksub,
                   size_t dsub, uint8_t* codes) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (uint32_t s = 0; s < m; ++s)
            codes[size_t(i) * m + s] = nearest_code(x + size_t(i) * m * dsub + s * dsub,
                                                    cb + size_t(s) * ksub * dsub, ksub, dsub);
}

// FastScanPq::decode (src/index/pq_fastscan.cpp:290-305).
void orc_pq_decode(const uint8_t* codes, size_t n, const float* cb, uint32_t m, uint32_t ksub,
                   size_t dsub, float* out) {
    for (size_t i = 0; i < n; ++i)
        for (uint32_t s = 0; s < m; ++s)
            std::memcpy(out + (i * m + s) * dsub, cb + (size_t(s) * ksub + codes[i * m + s]) * dsub, dsub * 4);
}

void orc_pq_lut(const float* r, const float* cb, uint32_t m, uint32_t ksub, size_t dsub, float* lut) {
    lut_one(r, cb, m, ksub, dsub, lut);
}

float orc_adc(const float* lut, const uint8_t* code, uint32_t m, uint32_t ksub) {
    return adc_one(lut, code, m, ksub);
}

// Impl::add (src/index/ivf_pq.cpp:2970-3440), brute branch: assign -> residual
// x - c[a] -> apply_rotation if a rotation is kept -> FastScanPq::encode.
void orc_ivfpq_add(const float* x, size_t n, const float* c, uint32_t nlist, size_t dim,
                   const float* R, const float* cb, uint32_t m, uint32_t ksub,
                   uint32_t* out_assign, uint8_t* out_codes) {
    orc_assign(x, n, c, nlist, dim, out_assign, nullptr);
    const size_t dsub = dim / m;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        std::vector<float> r(dim), rr(dim);
        const float* cl = c + size_t(out_assign[i]) * dim;
        for (size_t d = 0; d < dim; ++d) r[d] = x[size_t(i) * dim + d] - cl[d];
        const float* e = r.data();
        if (R) { rotate_one(r.data(), R, dim, rr.data()); e = rr.data(); }
        for (uint32_t s = 0; s < m; ++s)
            out_codes[size_t(i) * m + s] = nearest_code(e + s * dsub, cb + size_t(s) * ksub * dsub, ksub, dsub);
    }
}

uint32_t orc_ivfpq_search(const float* q, const float* c, uint32_t nlist, size_t dim,
                          const float* R, const float* cb, uint32_t m, uint32_t ksub,
                          const uint64_t* list_offsets, const uint64_t* ids,
                          const uint8_t* codes, uint32_t k, uint32_t nprobe, uint64_t* out_ids,
                          float* out_d) {
    return search_one(q, c, nlist, dim, R, cb, m, ksub, list_offsets, ids, codes, k, nprobe, 0, false,
                      0, out_ids, out_d);
}

// Impl::search_batch (src/index/ivf_pq.cpp:4096-4113): independent per-query searches.
void orc_ivfpq_search_batch(const float* q, size_t nq, const float* c, uint32_t nlist,
                            size_t dim, const float* R, const float* cb, uint32_t m,
                            uint32_t ksub, const uint64_t* list_offsets, const uint64_t* ids,
                            const uint8_t* codes, uint32_t k, uint32_t nprobe, uint64_t* out_ids,
                            float* out_d, uint32_t* out_counts) {
    orc_ivfpq_search_batch_ex(q, nq, c, nlist, dim, R, cb, m, ksub, list_offsets, ids, codes, k, nprobe, 0, 0,
                              0, out_ids, out_d, out_counts);
}

// With the candidate pool and the exact rerank (IvfPqSearchParams::cand_k,
// use_exact_rerank, rerank_k; include/vesper/index/ivf_pq.hpp:109-117).
void orc_ivfpq_search_batch_ex(const float* q, size_t nq, const float* c, uint32_t nlist,
                               size_t dim, const float* R, const float* cb, uint32_t m,
                               uint32_t ksub, const uint64_t* list_offsets, const uint64_t* ids,
                               const uint8_t* codes, uint32_t k, uint32_t nprobe, uint32_t cand_k,
                               int rerank, uint32_t rerank_k, uint64_t* out_ids, float* out_d,
                               uint32_t* out_counts) {
#pragma omp parallel for schedule(dynamic, 4)
    for (long long i = 0; i < (long long)nq; ++i)
        out_counts[i] = search_one(q + size_t(i) * dim, c, nlist, dim, R, cb, m, ksub, list_offsets,
                                   ids, codes, k, nprobe, cand_k, rerank != 0, rerank_k,
                                   out_ids + size_t(i) * k, out_d + size_t(i) * k);
}

// find_nearest_centroids_batch_fused (include/vesper/kernels/batch_distances.hpp:338-456):
// exact top-k with the total order (score, index); op 0 = L2 ascending, 1 = inner
// product descending; ties go to the smaller index.
void orc_flat_topk(int op, const float* q, size_t nq, const float* base, uint32_t nb,
                   size_t dim, uint32_t k, uint32_t* out_idx, float* out_score) {
    const uint32_t ke = std::min(k, nb);
    if (nb == 0 || nq == 0 || k == 0) return;
#pragma omp parallel for schedule(dynamic, 4)
    for (long long qi = 0; qi < (long long)nq; ++qi) {
        struct P { float s; uint32_t i; };
        auto dist_cmp = [](const P& a, const P& b) { return a.s != b.s ? a.s < b.s : a.i < b.i; };
        auto sim_cmp = [](const P& a, const P& b) { return a.s != b.s ? a.s > b.s : a.i < b.i; };
        std::vector<P> heap;
        heap.reserve(ke + 1);
        const float* qq = q + size_t(qi) * dim;
        for (uint32_t c = 0; c < nb; ++c) {
            const float s = op == 0 ? l2_lanes(qq, base + size_t(c) * dim, dim)
                                    : ip_lanes(qq, base + size_t(c) * dim, dim);
            if (op == 0) {
                if (heap.size() < ke) { heap.push_back({s, c}); std::push_heap(heap.begin(), heap.end(), dist_cmp); }
                else if (s < heap.front().s || (s == heap.front().s && c < heap.front().i)) {
                    std::pop_heap(heap.begin(), heap.end(), dist_cmp); heap.back() = {s, c};
                    std::push_heap(heap.begin(), heap.end(), dist_cmp);
                }
            } else {
                if (heap.size() < ke) { heap.push_back({s, c}); std::push_heap(heap.begin(), heap.end(), sim_cmp); }
                else if (s > heap.front().s || (s == heap.front().s && c < heap.front().i)) {
                    std::pop_heap(heap.begin(), heap.end(), sim_cmp); heap.back() = {s, c};
                    std::push_heap(heap.begin(), heap.end(), sim_cmp);
                }
            }
        }
        if (op == 0) std::sort_heap(heap.begin(), heap.end(), dist_cmp);
        else std::sort_heap(heap.begin(), heap.end(), sim_cmp);
        for (uint32_t i = 0; i < ke; ++i) { out_idx[size_t(qi) * k + i] = heap[i].i; out_score[size_t(qi) * k + i] = heap[i].s; }
    }
}

void orc_kmeanspp_init(const float* x, size_t n, size_t dim, uint32_t k, uint32_t seed,
                       float* out_c, uint32_t* out_idx) {
    kmeanspp(x, n, dim, k, seed, out_c, out_idx);
}

// kmeans_assign (src/index/kmeans.cpp:91-105); the fp64 inertia is summed in point order.
float orc_lloyd_assign(const float* x, size_t n, const float* c, uint32_t k, size_t dim,
                       uint32_t* out) {
    std::vector<float> d(n);
    orc_assign(x, n, c, k, dim, out, d.data());
    double t = 0.0;
    for (size_t i = 0; i < n; ++i) t += d[i];
    return static_cast<float>(t);
}

// kmeans_update_centroids (src/index/kmeans.cpp:107-135): fp64 sums in point order,
// divided by the count; an empty cluster keeps its previous centroid.
void orc_lloyd_update(const float* x, size_t n, size_t dim, const uint32_t* assign, uint32_t k,
                      float* c) {
    std::vector<double> sums(size_t(k) * dim, 0.0);
    std::vector<uint32_t> cnt(k, 0);
    for (size_t i = 0; i < n; ++i) {
        const uint32_t a = assign[i];
        cnt[a]++;
        for (size_t d = 0; d < dim; ++d) sums[size_t(a) * dim + d] += x[i * dim + d];
    }
    for (uint32_t a = 0; a < k; ++a)
        if (cnt[a] > 0)
            for (size_t d = 0; d < dim; ++d)
                c[size_t(a) * dim + d] = static_cast<float>(sums[size_t(a) * dim + d] / cnt[a]);
}

// kmeans_cluster (src/index/kmeans.cpp:137-252) with n_redo = 1: k-means++, Lloyd
// iterations (assign, convergence test on the fp32-cast fp64 inertia, update), one more
// update after the loop, and the returned inertia recomputed as the reference's final
// single fp32 running sum over every (point, dimension) term (:230-241).
int orc_kmeans_lloyd(const float* x, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                     float eps, uint32_t seed, float* out_c, uint32_t* out_assign,
                     uint32_t* out_iters, float* out_inertia) {
    if (n < k) return 2;
    if (k == 0) return 3;
    kmeanspp(x, n, dim, k, seed, out_c, nullptr);
    std::vector<uint32_t> asg(n);
    float prev = std::numeric_limits<float>::max();
    uint32_t it = 0;
    for (; it < max_iter; ++it) {
        const float inertia = orc_lloyd_assign(x, n, out_c, k, dim, asg.data());
        const float change = std::fabs(prev - inertia) / (prev + 1e-10f);
        if (change < eps) break;
        prev = inertia;
        orc_lloyd_update(x, n, dim, asg.data(), k, out_c);
    }
    orc_lloyd_update(x, n, dim, asg.data(), k, out_c);
    float total = 0.0f;
    for (size_t i = 0; i < n; ++i)
        for (size_t d = 0; d < dim; ++d) {
            const float diff = x[i * dim + d] - out_c[size_t(asg[i]) * dim + d];
            total += diff * diff;
        }
    if (out_assign) std::copy(asg.begin(), asg.end(), out_assign);
    if (out_iters) *out_iters = it;
    if (out_inertia) *out_inertia = total;
    return 0;
}

// Elkan M-step for every cluster: indices gathered in point order
// (src/index/kmeans_elkan.cpp:354-356), then update_centroid.
void orc_elkan_update_centroid(const float* x, size_t dim, const uint32_t* assign, size_t n,
                               uint32_t k, float* c) {
    std::vector<std::vector<size_t>> idx(k);
    for (size_t i = 0; i < n; ++i) idx[assign[i]].push_back(i);
    for (uint32_t a = 0; a < k; ++a) elkan_update_one(x, dim, idx[a], c + size_t(a) * dim);
}

// KmeansElkan::cluster (src/index/kmeans_elkan.cpp:293-430) with k-means++ init.
// The fp64 inertia sum runs in point order (the reference's OpenMP reduction order is
// unspecified, so the last bit of the inertia -- and hence, rarely, the convergence
// test -- can differ between runs of the reference itself).
int orc_kmeans_elkan(const float* x, size_t n, size_t dim, uint32_t k, uint32_t max_iter,
                     float eps, uint32_t seed, float* out_c, uint32_t* out_assign,
                     uint32_t* out_iters, float* out_inertia) {
    if (n < k) return 2;
    std::vector<float> C(size_t(k) * dim);
    kmeanspp(x, n, dim, k, seed, C.data(), nullptr);
    const auto cen = [&](uint32_t j) { return C.data() + size_t(j) * dim; };
    std::vector<float> upper(n), lower(n * size_t(k));
    std::vector<uint32_t> asg(n);
    std::vector<char> tight(n);
    // initialize_bounds (:66-98)
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        float best = std::numeric_limits<float>::max();
        uint32_t bc = 0;
        for (uint32_t j = 0; j < k; ++j) {
            const float d = l2_lanes(x + size_t(i) * dim, cen(j), dim);
            lower[size_t(i) * k + j] = d;
            if (d < best) { best = d; bc = j; }
        }
        upper[i] = best; asg[i] = bc; tight[i] = 1;
    }
    std::vector<float> cc(size_t(k) * k), sq(k);
    // update_centroid_distances (:100-133)
    auto centroid_dists = [&]() {
        for (uint32_t i = 0; i < k; ++i) cc[size_t(i) * k + i] = 0.0f;
#pragma omp parallel for schedule(dynamic, 8)
        for (long long i = 0; i < (long long)k; ++i)
            for (uint32_t j = (uint32_t)i + 1; j < k; ++j) {
                const float d = l2_lanes(cen((uint32_t)i), cen(j), dim);
                cc[size_t(i) * k + j] = d; cc[size_t(j) * k + i] = d;
            }
        for (uint32_t i = 0; i < k; ++i) {
            float mn = std::numeric_limits<float>::max();
            for (uint32_t j = 0; j < k; ++j)
                if (i != j && cc[size_t(i) * k + j] < mn) mn = cc[size_t(i) * k + j];
            sq[i] = 0.25f * mn;
        }
    };
    centroid_dists();
    float prev = std::numeric_limits<float>::max();
    uint32_t it = 0;
    std::vector<double> part(n);
    for (; it < max_iter; ++it) {
        // assign_with_bounds (:183-262)
#pragma omp parallel for schedule(static)
        for (long long ii = 0; ii < (long long)n; ++ii) {
            const size_t i = size_t(ii);
            const float* p = x + i * dim;
            float* lo = lower.data() + i * k;
            if (upper[i] <= sq[asg[i]]) {
                if (!tight[i]) { const float d = l2_lanes(p, cen(asg[i]), dim); lo[asg[i]] = d; upper[i] = d; tight[i] = 1; }
                part[i] = upper[i];
                continue;
            }
            if (!tight[i]) {
                const float d = l2_lanes(p, cen(asg[i]), dim); lo[asg[i]] = d; upper[i] = d; tight[i] = 1;
                if (upper[i] <= sq[asg[i]]) { part[i] = upper[i]; continue; }
            }
            for (uint32_t j = 0; j < k; ++j) {
                if (j == asg[i]) continue;
                if (upper[i] <= lo[j]) continue;
                if (upper[i] <= 0.25f * cc[size_t(asg[i]) * k + j]) continue;
                const float d = l2_lanes(p, cen(j), dim);
                lo[j] = d;
                if (d < upper[i]) { asg[i] = j; upper[i] = d; tight[i] = 1; }
            }
            part[i] = upper[i];
        }
        double tot = 0.0;
        for (size_t i = 0; i < n; ++i) tot += part[i];
        const float inertia = static_cast<float>(tot);
        const float change = std::fabs(prev - inertia) / (prev + 1e-10f);
        if (change < eps) break;
        prev = inertia;
        // M-step (:346-368)
        std::vector<float> old(C);
        orc_elkan_update_centroid(x, dim, asg.data(), n, k, C.data());
        std::vector<float> shift(k), delta(k);
        for (uint32_t j = 0; j < k; ++j) shift[j] = l2_lanes(old.data() + size_t(j) * dim, cen(j), dim);
        // update_bounds (:264-291)
        for (uint32_t j = 0; j < k; ++j) delta[j] = std::sqrt(std::max(0.0f, shift[j]));
#pragma omp parallel for schedule(static)
        for (long long ii = 0; ii < (long long)n; ++ii) {
            const size_t i = size_t(ii);
            float u = std::sqrt(std::max(0.0f, upper[i]));
            u += delta[asg[i]];
            upper[i] = u * u;
            tight[i] = 0;
            float* lo = lower.data() + i * k;
            for (uint32_t j = 0; j < k; ++j) {
                float l = std::sqrt(std::max(0.0f, lo[j]));
                l = std::max(0.0f, l - delta[j]);
                lo[j] = l * l;
            }
        }
        centroid_dists();
    }
    std::memcpy(out_c, C.data(), C.size() * 4);
    if (out_assign) std::memcpy(out_assign, asg.data(), n * 4);
    if (out_iters) *out_iters = it;
    if (out_inertia) *out_inertia = prev;
    return 0;
}

// FastScanPq::train / train_subquantizer (src/index/pq_fastscan.cpp:15-76): one Elkan
// k-means per sub-space (k = 2^nbits, max_iter 25, eps 1e-4, seed 42 + s).  A failed
// sub-k-means (n < ksub) leaves that codebook at zero, as the reference does.
int orc_pq_train(const float* x, size_t n, size_t dim, uint32_t m, uint32_t nbits, float* out_cb) {
    if (dim % m != 0) return 2;
    const size_t dsub = dim / m;
    const uint32_t ksub = 1u << nbits;
    std::memset(out_cb, 0, size_t(m) * ksub * dsub * 4);
    for (uint32_t s = 0; s < m; ++s) {
        std::vector<float> sub(n * dsub);
        for (size_t i = 0; i < n; ++i) std::memcpy(sub.data() + i * dsub, x + i * dim + s * dsub, dsub * 4);
        std::vector<float> cbs(size_t(ksub) * dsub);
        if (orc_kmeans_elkan(sub.data(), n, dsub, ksub, 25, 1e-4f, 42 + s, cbs.data(), nullptr, nullptr, nullptr) == 0)
            std::memcpy(out_cb + size_t(s) * ksub * dsub, cbs.data(), cbs.size() * 4);
    }
    return 0;
}

}  // extern "C"
