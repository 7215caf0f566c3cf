// Launch wrappers for the B200 IVF-PQ kernels (definitions in ivfpq_kernels.cu and
// kmeans_kernels.cu).  All pointers are device pointers; all launches go to `st`.
#pragma once

#include "common.cuh"

namespace vgpu {

constexpr int kMaxK = 1024;        // largest k / nprobe the selection kernels accept
constexpr int kScanChunk = 2048;   // list entries scored per selection round

// Per query, the k smallest of `parts` sorted per-shard top-k lists (shard_merge.cu):
// part p's distances at dist + p dist_stride + q k, ids at ids + p ids_stride + q k,
// counts at counts + p counts_stride + q; ties to the lower part, then the earlier
// slot; slots past out_n padded with id 0 and the last distance.  parts <= 64.
void launch_topk_merge(int parts, long long nq, int k, const float* dist, long long dist_stride, const uint64_t* ids,
                       long long ids_stride, const uint32_t* counts, long long counts_stride, uint64_t* out_ids,
                       float* out_d, uint32_t* out_n, cudaStream_t st);

// D[i][j] = ||x_i - c_j||^2 in reference lane order, for i < nx, j < nc; D row stride ldd.
void launch_l2_dist(const float* x, long long nx, const float* c, int nc, int dim, float* D,
                    long long ldd, cudaStream_t st);

// Per row of D (n_rows x ncols, stride ldd): the k smallest (value, column) pairs in
// ascending order -> out_idx[row*k + t], out_val[row*k + t].
void launch_row_topk(const float* D, long long n_rows, int ncols, long long ldd, int k,
                     uint32_t* out_idx, float* out_val, cudaStream_t st);

// Per row: arg-min with a strict `<` scan from FLT_MAX (lowest column wins ties);
// when `keep` is given, a row keeps keep[row] if that column ties the minimum
// (Elkan's assignment rule).  Writes the index and the minimum.
void launch_row_argmin(const float* D, long long n_rows, int ncols, long long ldd,
                       const uint32_t* keep, uint32_t* out_idx, float* out_val, cudaStream_t st);

// out[r][j] = sum_k (x[xrow(r)][k] - c[crow(r)][k]) * R[k][j], sequential in k with a
// rounded product and a rounded add (apply_rotation order).  xrow(r) = xidx ? xidx[r] : r,
// crow(r) = cidx ? cidx[r] : -1 (no subtraction when cidx is null).  R may be null
// (plain residual copy).
void launch_residual_rotate(const float* x, const uint32_t* xidx, const float* c,
                            const uint32_t* cidx, long long rows, int dim, const float* R,
                            float* out, cudaStream_t st);

// codes[i][s] = arg-min_j l2(x_i[s*dsub:(s+1)*dsub], cb[s][j]) (strict <, lowest j).
void launch_pq_encode(const float* x, long long n, int m, int ksub, int dsub, const float* cb,
                      uint8_t* codes, cudaStream_t st);

// Exact per-(query, probe) LUT + scan + local top-k.  pair p = (q, t) with list
// probe[q*nprobe + t]; residuals either given per pair (rres: rotated residual rows,
// one per pair) or formed as query - centroid.  Output per pair: up to k candidates
// sorted by (distance, list position) in cand_d / cand_pos, count in cand_n.
void launch_scan_exact(const float* queries, long long nq, int dim, const float* centroids,
                       const float* rres, const uint32_t* probe, int nprobe, const float* cb, int m,
                       int ksub, int dsub, const uint64_t* list_offsets, const uint8_t* codes,
                       int k, float* cand_d, uint32_t* cand_pos, uint32_t* cand_n,
                       cudaStream_t st);

// Per query: merge nprobe sorted candidate runs into the final top-k by
// (distance, probe rank, list position); map to ids; pad short results the way the
// reference C ABI does (ids 0, distance = last valid or 0).
void launch_merge(const float* cand_d, const uint32_t* cand_pos, const uint32_t* cand_n,
                  long long nq, int nprobe, int k, const uint32_t* probe,
                  const uint64_t* list_offsets, const uint64_t* ids, uint64_t* out_ids,
                  float* out_d, uint32_t* out_n, cudaStream_t st);

// Fast search path (distances within fp32 rounding of the exact ones):
// dist(q, x) = ||Rq - Rc_l||^2 + u(x) + sum_s T_q[s][code_s(x)], with
// T_q[s][j] = -2 <(Rq)_s, y_sj> (one table per query) and u(x) the per-vector term
// stored at add time.
// Fast path in two stages: T[q] = per-query tables [m x ksub] for a batch, then a scan
// with a running top-k filtered by the current k-th (distance, scan position) key.
void launch_lut_fast(const float* rq, long long nq, int dim, const float* cb, int m, int ksub, int dsub,
                     float* T, cudaStream_t st);
// Whether launch_lut_fast / launch_scan_fast2 accept these shapes (their shared-memory
// and k limits); each launch throws CudaError when its check fails.
bool lut_fast_fits(int ksub, int dsub);
bool scan_fast2_fits(int m, int ksub, int k, int nprobe);
void launch_scan_fast2(const float* T, const float* rq, long long nq, int dim, const uint32_t* probe,
                       const float* probe_d, const float* rc, int nprobe, int m, int ksub,
                       const uint64_t* list_offsets, const uint8_t* codes, const float* vterm,
                       const uint64_t* ids, int k, uint64_t* out_ids, float* out_d, uint32_t* out_n,
                       cudaStream_t st);

// Blocked scan layout (see ivfpq_kernels.cu): lists cut into 128-entry blocks whose
// code bytes are pre-rotated so a warp's lookups never share a bank.
bool scan_blocked_supported(int m, int ksub);
void launch_build_blocks(const uint8_t* codes, const float* vterm, const uint64_t* offs, const uint64_t* blk_off,
                         int m, int nlist, uint8_t* bcodes, float* bvterm, cudaStream_t st);
void launch_lut_blocked(const float* rq, long long nq, int dim, const float* cb, int m, int dsub, float* T,
                        cudaStream_t st);
// Base term of each (query, probe) pair for the FAST scans: ||Rq - R c_l||^2 when rc
// (rotated centroids) is given, else probe_d.
void launch_probe_base(const float* rq, long long nq, int dim, const uint32_t* probe, const float* probe_d,
                       const float* rc, int nprobe, float* pbase, cudaStream_t st);
// Scratch of the split blocked scan (grown on demand).
struct SplitWork {
    DeviceBuffer<uint32_t> parts, part_off, nblocks;
    DeviceBuffer<uint4> items;
    DeviceBuffer<unsigned long long> part_keys;
    DeviceBuffer<unsigned char> scan_tmp;
    uint32_t* host_total = nullptr;   // pinned
    void reserve(long long nq);
    SplitWork() = default;
    SplitWork(const SplitWork&) = delete;
    SplitWork& operator=(const SplitWork&) = delete;
    ~SplitWork();
};
// launch_scan_blocked with each query's blocks split over several CTAs (parts of 64
// blocks, at most 8192 / k parts) and merged: the same results, without a single CTA
// scanning a very long probe set.  Synchronizes the stream once (number of parts).
// max_blocks: only the first max_blocks 128-entry blocks of each query's probe set.
void launch_scan_blocked_split(const float* T, long long nq, const float* pbase, const uint32_t* probe, int nprobe,
                               int nscan, int m, const uint64_t* offs, const uint64_t* blk_off,
                               const uint8_t* bcodes, const float* bvterm, const uint64_t* ids, int k,
                               uint64_t* out_ids, float* out_d, uint32_t* out_n, const uint32_t* only_over,
                               uint32_t over_cap, SplitWork& w, cudaStream_t st, uint32_t max_blocks = 0xffffffffu);
// Blocked FAST scan of the first nscan of each query's nprobe probes.  With only_over,
// a query is processed only when only_over[q] > over_cap (the others are left as is).
void launch_scan_blocked(const float* T, long long nq, const float* pbase, const uint32_t* probe, int nprobe,
                         int nscan, int m, const uint64_t* offs, const uint64_t* blk_off, const uint8_t* bcodes,
                         const float* bvterm, const uint64_t* ids, int k, uint64_t* out_ids, float* out_d,
                         uint32_t* out_n, const uint32_t* only_over, uint32_t over_cap, cudaStream_t st);

// u(x) = sum_s ( ||y_s,c_s||^2 + 2 <(R c_l)_s, y_s,c_s> ) for every CSR entry, with
// rc = rotated centroids [nlist x dim]; accumulated in fp64, rounded once.
void launch_vector_terms(const float* rc, int nlist, int dim, const float* cb, int m, int ksub,
                         int dsub, const uint64_t* list_offsets, const uint8_t* codes,
                         long long n_entries, float* vterm, cudaStream_t st);

// Plain fp32 GEMM-like product out = x * R (no ordering guarantee; used only for the
// fast path's Rq and Rc, which are inside the fast path's tolerance).
void launch_rotate_fast(const float* x, long long rows, int dim, const float* R, float* out,
                        cudaStream_t st);

// *out += sum over the n probe entries of the probed list's size.
void launch_probe_sizes(const uint32_t* probe, long long n, const uint64_t* list_offsets,
                        unsigned long long* out, cudaStream_t st);

// CSR rebuild helpers for add(): move old entries to their new offsets, scatter new
// entries to precomputed destinations.
void launch_csr_move(const uint8_t* old_codes, const uint64_t* old_ids, const uint64_t* old_off,
                     const uint64_t* new_off, int nlist, int m, uint8_t* codes, uint64_t* ids,
                     cudaStream_t st);
void launch_csr_scatter(const uint8_t* new_codes, const uint64_t* new_ids, const uint64_t* dest,
                        long long n, int m, uint8_t* codes, uint64_t* ids, cudaStream_t st);

// ----------------------------------------------------------------------- k-means
// k-means++ D^2 update: mind[i] = min(mind[i], l2(x_i, c)).
// k-means++ draws on the device: refresh D^2 with centroid c and write per-block fp64
// sums (kpp_blocks(n) of them), then pick the row whose running D^2 prefix first
// reaches u[ci] * total and copy it into centroids row ci (kmeans_kernels.cu).
long long kpp_blocks(long long n);
void launch_kpp_update_sum(const float* x, long long n, int dim, const float* c, float* mind, double* block_sum,
                           cudaStream_t st);
void launch_kpp_pick(const float* x, long long n, int dim, const float* mind, const double* block_sum,
                     const double* u, int ci, float* centroids, cudaStream_t st);
void launch_kpp_update(const float* x, long long n, int dim, const float* c, float* mind,
                       cudaStream_t st);
// Segmented M-step.  order: point indices grouped by cluster (ascending within a
// cluster), seg: [k+1] offsets.  kahan=1 -> Kahan fp64 sum times (1/count)
// (KmeansElkan update_centroid); kahan=0 -> fp64 sum / count (Lloyd).  Empty clusters
// keep their centroid.
void launch_segment_mean(const float* x, int dim, const uint32_t* order, const uint32_t* seg,
                         int k, int kahan, float* centroids, cudaStream_t st);
// The M-step split over point shards held by different GPUs: each shard continues the
// per-(cluster, dimension) running sums (sum, and the Kahan compensation when kahan=1)
// over its own points in order, starting from the state the previous shard left, and
// adds its cluster sizes to count; finish turns the state into centroids exactly as
// launch_segment_mean does.  Running the shards in point order reproduces
// launch_segment_mean over the whole set bit for bit.
void launch_segment_accumulate(const float* x, int dim, const uint32_t* order, const uint32_t* seg, int k,
                               int kahan, double* sum, double* comp, unsigned long long* count, cudaStream_t st);
void launch_finish_means(const double* sum, const unsigned long long* count, int k, int dim, int kahan,
                         float* centroids, cudaStream_t st);
// *total = *total + sum over points i in order, dims d in order, of (x_id - c_{a_i}d)^2,
// one rounded float add per term (kmeans_cluster's final inertia).
void launch_ordered_sq_sum(const float* x, const float* c, const uint32_t* assign, long long n, int dim,
                           float* total, cudaStream_t st);

// ----------------------------------------------------------------------- exact rerank (rerank.cu)
void launch_iota(uint32_t* out, long long n, cudaStream_t st);
// sorted_ids / sorted_entry: the ids of the n entries in ascending order with their
// entry index, equal ids in entry order (id -> first entry holding it).
void launch_id_map_build(const uint64_t* ids, long long n, uint64_t* sorted_ids, uint32_t* sorted_entry,
                         DeviceBuffer<uint32_t>& iota, DeviceBuffer<unsigned char>& tmp, cudaStream_t st);
struct RerankArgs {
    const float* q;                  // [nq x dim] queries
    const uint64_t* pool_ids;        // [nq x P] ADC pool, ascending ADC distance
    const float* pool_d;             // [nq x P]
    const uint32_t* pool_n;          // [nq] pool sizes
    long long nq;
    int P, head_cap, k;              // head = min(pool_n, head_cap) candidates are reranked
    const uint64_t* sid;             // id map
    const uint32_t* sent;
    long long n;
    const uint64_t* offs;            // [nlist + 1]
    int nlist;
    const uint8_t* codes;            // [n x m]
    int m, ksub, dsub;
    const float* cb;                 // [m x ksub x dsub]
    const float* cent;               // [nlist x dim]
    const float* rotT;               // R transposed, or null without a rotation
    uint32_t* ent;                   // [nq x P] scratch
    uint32_t* lst;                   // [nq x P] scratch
    float* dec;                      // [nq x P x dim] scratch (rotation only)
    float* rot_out;                  // [nq x P x dim] scratch (rotation only)
    float* exact_d;                  // [nq x P] scratch
    uint64_t* out_ids;               // [nq x k]
    float* out_d;                    // [nq x k]
    uint32_t* out_n;                 // [nq] or null
};
void launch_rerank(const RerankArgs& a, cudaStream_t st);

// ----------------------------------------------------------------------- index maintenance (index_ops.cu)
// out[i] = cent[list(i)] + rotT-rotated decode(codes[entry(i)]) in the reference's order;
// entry(i) = entries ? entries[i] : e0 + i, list(i) = lists ? lists[i] : list0; rotT may be
// null (no rotation).  tmp_dec / tmp_rot: [n x dim] scratch.
void launch_reconstruct_rows(const uint32_t* entries, unsigned long long e0, const uint32_t* lists, uint32_t list0,
                             long long n, const uint8_t* codes, int m, int ksub, int dsub, const float* cb,
                             const float* cent, const float* rotT, float* tmp_dec, float* tmp_rot, float* out,
                             cudaStream_t st);
// adc[e] = exact ADC distance of entry e from its list's table built from rres[list].
void launch_adc_all(const float* rres, int dim, int nlist, const float* cb, int m, int ksub, int dsub,
                    const uint64_t* offs, const uint8_t* codes, float* adc, cudaStream_t st);
void launch_count_less(const float* v, long long n, long long target, unsigned long long* count, cudaStream_t st);
// The index files' inverted-list section <-> CSR (lists_io.cu).  list_byte[l]: offset
// of list l's size field in raw (after the u32 list count).
void launch_unpack_lists(const uint8_t* raw, const uint64_t* list_byte, const uint64_t* offs, int nlist, int m,
                         uint64_t* ids, uint8_t* codes, cudaStream_t st);
void launch_pack_lists(const uint64_t* ids, const uint8_t* codes, const uint64_t* offs, int nlist, int m,
                       const uint64_t* list_byte, uint8_t* raw, cudaStream_t st);
// codes2 / ids2 in the new entry order (order[i] = old entry, 0xffffffff = the new entry).
void launch_gather_entries(const uint32_t* order, long long n, const uint8_t* codes, const uint64_t* ids, int m,
                           const uint8_t* new_code, uint64_t new_id, uint8_t* codes2, uint64_t* ids2,
                           cudaStream_t st);
// out[0] = first entry holding id (0xffffffff if none), out[1] = its list.
void launch_id_lookup(const uint64_t* sid, const uint32_t* sent, long long n, uint64_t id, const uint64_t* offs,
                      int nlist, uint32_t* out, cudaStream_t st);

}  // namespace vgpu
