// Exact rerank of an IVF-PQ candidate pool (src/index/ivf_pq.cpp:3995-4091).
//
// For the head of each query's ADC pool the reference finds the entry holding the
// candidate's id (the first one in list order), rebuilds its vector as
//     centroid[l] + apply_rotation_T(decode(code))          (rounded adds)
// and replaces the ADC distance by the squared L2 distance to the query, summed
// sequentially over the dimensions with a rounded product and a rounded add; then it
// re-sorts the head by distance and trims to k.  Here:
//   id_map_build      ids sorted with their entry index (stable radix sort, so the
//                     first entry holding an id comes first): the id -> entry lookup;
//   rerank_lookup     per candidate: entry (binary search) and list (binary search of
//                     the CSR offsets); with a rotation it also writes the decoded code;
//   residual_rotate   (ivfpq_kernels.cu) applies R^T in the reference's order;
//   rerank_dist       per candidate the sequential sum, 32 candidates per warp with the
//                     operands staged through shared memory in 32-dimension tiles;
//   rerank_select     per query the head sorted by (distance, position) and the output
//                     rows (the reference's std::sort leaves the order among exactly
//                     equal distances unspecified).
#include <cub/cub.cuh>

#include <cfloat>

#include "kernels.cuh"
#include "select.cuh"

namespace vgpu {

void launch_id_map_build(const uint64_t* ids, long long n, uint64_t* sorted_ids, uint32_t* sorted_entry,
                         DeviceBuffer<uint32_t>& iota, DeviceBuffer<unsigned char>& tmp, cudaStream_t st) {
    if (n <= 0) return;
    if (n > 0xffffffffLL) throw CudaError("id map: at most 2^32 entries");
    iota.reserve((size_t)n);
    launch_iota(iota.data(), n, st);
    size_t need = 0;
    check(cub::DeviceRadixSort::SortPairs(nullptr, need, ids, sorted_ids, iota.data(), sorted_entry, (int64_t)n, 0, 64,
                                          st),
          "cub::DeviceRadixSort::SortPairs(size)");
    tmp.reserve(need);
    check(cub::DeviceRadixSort::SortPairs(tmp.data(), need, ids, sorted_ids, iota.data(), sorted_entry, (int64_t)n, 0,
                                          64, st),
          "cub::DeviceRadixSort::SortPairs(id map)");
}

__global__ void entry_iota_kernel(uint32_t* __restrict__ out, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = (uint32_t)i;
}

void launch_iota(uint32_t* out, long long n, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    entry_iota_kernel<<<blocks, 256, 0, st>>>(out, n);
    VGPU_LAUNCH("entry_iota_kernel");
}

// One warp per pool slot (q, i) with i < head(q): entry e of the candidate's id (or
// 0xffffffff when absent), its list, and -- when dec != nullptr -- the decoded code.
__global__ void rerank_lookup_kernel(const uint64_t* __restrict__ pool_ids, const uint32_t* __restrict__ pool_n,
                                     long long nq, int P, int head_cap, const uint64_t* __restrict__ sid,
                                     const uint32_t* __restrict__ sent, long long n, const uint64_t* __restrict__ offs,
                                     int nlist, const uint8_t* __restrict__ codes, int m, int ksub, int dsub,
                                     const float* __restrict__ cb, uint32_t* __restrict__ ent,
                                     uint32_t* __restrict__ lst, float* __restrict__ dec) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    const int dim = m * dsub;
    for (long long slot = warp; slot < nq * P; slot += nw) {
        const long long q = slot / P;
        const int i = (int)(slot % P);
        const int head = min((int)pool_n[q], head_cap);
        if (i >= head) continue;
        uint32_t e = 0xffffffffu, l = 0;
        if (lane == 0) {
            const uint64_t id = pool_ids[slot];
            long long lo = 0, hi = n;  // first position with sid >= id
            while (lo < hi) {
                const long long mid = (lo + hi) >> 1;
                if (sid[mid] < id) lo = mid + 1; else hi = mid;
            }
            if (lo < n && sid[lo] == id) {
                e = sent[lo];
                int a = 0, b = nlist;  // last list with offs[list] <= e
                while (b - a > 1) {
                    const int mid = (a + b) >> 1;
                    if (offs[mid] <= (uint64_t)e) a = mid; else b = mid;
                }
                l = (uint32_t)a;
            }
            ent[slot] = e;
            lst[slot] = l;
        }
        e = __shfl_sync(0xffffffffu, e, 0);
        if (dec && e != 0xffffffffu) {
            const uint8_t* cd = codes + (long long)e * m;
            float* out = dec + slot * dim;
            for (int d = lane; d < dim; d += 32) {
                const int s = d / dsub;
                out[d] = cb[((long long)s * ksub + cd[s]) * dsub + (d - s * dsub)];
            }
        }
    }
}

// Squared distance of each head candidate, summed sequentially over d:
//     dist = sum_d (q[d] - (c_l[d] + r[d]))^2
// with r the rotated residual (res != nullptr) or the decoded code.  32 candidates per
// warp, one per lane: the elementwise part (q - (c + r), rounded) is formed with
// coalesced loads into a 32 x 32 shared tile, and each lane then adds its candidate's
// 32 squares in order.  Candidates whose id was not found keep the ADC distance.
constexpr int RD_NT = 256;
__global__ void __launch_bounds__(RD_NT) rerank_dist_kernel(
    const float* __restrict__ q, const uint32_t* __restrict__ pool_n, const float* __restrict__ pool_d, long long nq,
    int P, int head_cap, const uint32_t* __restrict__ ent, const uint32_t* __restrict__ lst,
    const float* __restrict__ cent, const float* __restrict__ res, const uint8_t* __restrict__ codes, int m, int ksub,
    int dsub, const float* __restrict__ cb, float* __restrict__ out_d) {
    __shared__ float td[RD_NT / 32][32][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int dim = m * dsub;
    const long long nslots = nq * P;
    const long long group = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long ngroups = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long g0 = group * 32; g0 < nslots; g0 += ngroups * 32) {
        const long long slot = g0 + lane;
        bool act = false;
        uint32_t e = 0xffffffffu, l = 0;
        long long qi = 0;
        if (slot < nslots) {
            qi = slot / P;
            const int i = (int)(slot % P);
            act = i < min((int)pool_n[qi], head_cap);
            if (act) { e = ent[slot]; l = lst[slot]; }
        }
        const bool found = act && e != 0xffffffffu;
        const unsigned any = __ballot_sync(0xffffffffu, found);
        float dist = 0.0f;
        if (any) {
            for (int d0 = 0; d0 < dim; d0 += 32) {
                const int d = d0 + lane;
                for (int c = 0; c < 32; ++c) {
                    const uint32_t ec = __shfl_sync(0xffffffffu, e, c);
                    const uint32_t lc = __shfl_sync(0xffffffffu, l, c);
                    const long long qc = __shfl_sync(0xffffffffu, qi, c);
                    float diff = 0.0f;
                    if (((any >> c) & 1u) && d < dim) {
                        float rv;
                        if (res) {
                            rv = res[(g0 + c) * dim + d];
                        } else {
                            const int s = d / dsub;
                            rv = cb[((long long)s * ksub + codes[(long long)ec * m + s]) * dsub + (d - s * dsub)];
                        }
                        const float rec = __fadd_rn(cent[(long long)lc * dim + d], rv);
                        diff = __fsub_rn(q[qc * dim + d], rec);
                    }
                    td[w][c][lane] = diff;
                }
                __syncwarp();
                if (found) {
                    const int dn = min(32, dim - d0);
                    for (int t = 0; t < dn; ++t) {
                        const float df = td[w][lane][t];
                        dist = __fadd_rn(dist, __fmul_rn(df, df));
                    }
                }
                __syncwarp();
            }
        }
        if (act) out_d[slot] = found ? dist : pool_d[slot];
    }
}

// Per query: the head sorted by (exact distance, position), then the ADC tail; rows
// padded like the other search paths (id 0, the last real distance).
constexpr int RS_NT = 256;
__global__ void __launch_bounds__(RS_NT) rerank_select_kernel(const uint64_t* __restrict__ pool_ids,
                                                              const float* __restrict__ pool_d,
                                                              const uint32_t* __restrict__ pool_n, int P, int head_cap,
                                                              const float* __restrict__ exact_d, int k,
                                                              uint64_t* __restrict__ out_ids, float* __restrict__ out_d,
                                                              uint32_t* __restrict__ out_n) {
    __shared__ unsigned long long keys[kMaxK];
    const long long q = blockIdx.x;
    const int cnt = (int)pool_n[q];
    const int head = min(cnt, head_cap);
    const int p2 = next_pow2(head < 2 ? 2 : head);
    for (int i = threadIdx.x; i < p2; i += RS_NT)
        keys[i] = i < head ? ((unsigned long long)float_key(exact_d[q * P + i]) << 32) | (uint32_t)i : ~0ull;
    bitonic_sort_u64<RS_NT>(keys, p2);
    const int take = min(cnt, k);
    float last = 0.0f;
    if (take > 0) {
        const int j = take - 1;
        last = j < head ? key_float((uint32_t)(keys[j] >> 32)) : pool_d[q * P + j];
    }
    for (int j = threadIdx.x; j < k; j += RS_NT) {
        uint64_t id = 0;
        float d = last;
        if (j < take) {
            if (j < head) {
                const uint32_t pos = (uint32_t)(keys[j] & 0xffffffffull);
                id = pool_ids[q * P + pos];
                d = key_float((uint32_t)(keys[j] >> 32));
            } else {
                id = pool_ids[q * P + j];
                d = pool_d[q * P + j];
            }
        }
        out_ids[q * k + j] = id;
        out_d[q * k + j] = d;
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)take;
}

void launch_rerank(const RerankArgs& a, cudaStream_t st) {
    if (a.nq <= 0) return;
    if (a.P > kMaxK) throw CudaError("rerank: candidate pool above 1024");
    const long long slots = a.nq * a.P;
    const int dim = a.m * a.dsub;
    {
        const int blocks = (int)std::min<long long>((slots * 32 + 255) / 256, 148LL * 32);
        rerank_lookup_kernel<<<blocks, 256, 0, st>>>(a.pool_ids, a.pool_n, a.nq, a.P, a.head_cap, a.sid, a.sent, a.n,
                                                     a.offs, a.nlist, a.codes, a.m, a.ksub, a.dsub, a.cb, a.ent, a.lst,
                                                     a.rotT ? a.dec : nullptr);
        VGPU_LAUNCH("rerank_lookup_kernel");
    }
    const float* res = nullptr;
    if (a.rotT) {
        launch_residual_rotate(a.dec, nullptr, nullptr, nullptr, slots, dim, a.rotT, a.rot_out, st);
        res = a.rot_out;
    }
    {
        const long long groups = (slots + 31) / 32;
        const int blocks = (int)std::min<long long>((groups * 32 + RD_NT - 1) / RD_NT, 148LL * 8);
        rerank_dist_kernel<<<blocks, RD_NT, 0, st>>>(a.q, a.pool_n, a.pool_d, a.nq, a.P, a.head_cap, a.ent, a.lst,
                                                     a.cent, res, a.codes, a.m, a.ksub, a.dsub, a.cb, a.exact_d);
        VGPU_LAUNCH("rerank_dist_kernel");
    }
    rerank_select_kernel<<<(unsigned)a.nq, RS_NT, 0, st>>>(a.pool_ids, a.pool_d, a.pool_n, a.P, a.head_cap, a.exact_d,
                                                           a.k, a.out_ids, a.out_d, a.out_n);
    VGPU_LAUNCH("rerank_select_kernel");
}

}  // namespace vgpu
