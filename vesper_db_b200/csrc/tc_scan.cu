// List-major tensor-core PQ scan (FAST search): screen every (query, entry) pair of a
// query batch with tcgen05 bf16 products, keep the pairs that can still be in a query's
// top k, and re-score only those with the FAST lookup-table arithmetic.
//
// The FAST distance of entry x of list l for query q is
//     d = (base(q,l) + u(x)) + sum_s T_q[s][c_s(x)],   T_q[s][c] = -2 <(Rq)_s, y_s,c>,
// and sum_s T_q[s][c_s(x)] = -2 <Rq, xhat> with xhat the decoded (rotated-space)
// residual.  The screen computes S = <bf16(Rq), bf16(xhat)> on the tensor cores, so
//     approx = (base + u) - 2 S,   |approx - d| <= slack(q, x)
// with the bound below.  A pair is kept when approx - slack <= tau(q), where tau(q) is
// an upper bound of q's k-th FAST distance (its k-th distance over its nearest list).
// Every entry whose FAST distance is <= tau(q) is therefore kept, the refine computes
// its FAST distance and scan position exactly as the blocked scan does, and the k
// smallest (distance, position) keys are the blocked scan's result, bit for bit.
//
// Work layout.  The (query, probe) pairs of the batch are grouped by list.  A unit is
// (list, 128-entry tile, group of up to QG x N queries).  A persistent CTA per SM takes
// units from a global counter:
//   * warps 0-7 decode the tile's 128 entries (codes -> bf16 codebook rows) straight
//     into tensor memory (A operand, 128 lanes x dim/2 columns);
//   * warps 4-7 stream the queries' bf16 rows (B operand, N x 64 per stage, 128-byte
//     swizzle) through an S-stage shared-memory ring with cp.async;
//   * one thread of warp 8 issues tcgen05.mma.kind::f16 (M = 128, N, K = 16, A from
//     TMEM) into one of two TMEM accumulators;
//   * warps 0-3 read the accumulator (thread = entry row), apply the keep rule and
//     append survivors to per-query candidate lists.
// Every wait is bounded; on timeout the kernel records an error code, stops issuing
// work at the next unit boundary, drains its tensor-core work and frees its TMEM.
#include <cub/cub.cuh>
#include <cuda.h>
#include <cuda_bf16.h>

#include <cfloat>
#include <cstdlib>
#include <string>

#include "kernels.cuh"
#include "kernels_tc.cuh"
#include "select.cuh"
#include "tc_common.cuh"

namespace vgpu {

CUtensorMap make_tile_map_bf16(const void* base, long long rows, int dim, int box_rows);

namespace {
constexpr int TL_M = 128;          // entries per tile (TMEM lanes)
constexpr uint32_t kSkipPair = 0xffffffffu;  // probe entry left out of a pair grouping
constexpr int TL_THREADS = 224;    // 7 warps: 0-3 decode + epilogue, 4 TMA, 5 MMA, 6 scheduler
constexpr int TL_QG = 1024;        // query chunks per unit (a unit is normally a whole list tile)
constexpr float kSlackMul = 0.03125f;           // 2^-5: bf16 products + tensor-core accumulation
constexpr float kSlackAbs = 9.5367431640625e-07f;  // 2^-20: fp32 rounding of both formulas

// Instruction descriptor for kind::f16: D f32, A and B bf16, both K-major, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TL_M >> 4) << 24);
}

// tcgen05.mma (A from shared memory / from TMEM) and tcgen05.commit, issued by one
// elected lane of a converged warp.
__device__ __forceinline__ void mma_bf16_ss_elect(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void commit_elect(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
        ::"r"(tc::smem_u32(bar))
        : "memory");
}

// OR of `v` over the 128 epilogue threads (named barrier 1); also a barrier for them.
__device__ __forceinline__ bool group_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// A box of 64 bf16 columns x 128 rows at (x, y) of the map's matrix, 128B-swizzled.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct UnitInfo {
    uint32_t list, tile, pair_begin, pair_end, n_chunks, list_len, valid;
    unsigned long long entry_base;
};

}  // namespace

struct TlParams {
    const __nv_bfloat16* rqb;   // [nq x dim] rotated queries, bf16
    const float* rqn;           // [nq] ||Rq||
    const float* pbase;         // [nq x nprobe]
    const float* tau;           // [nq] upper bound of the k-th FAST distance (-FLT_MAX: no screen)
    const uint32_t* probe;      // [nq x nprobe]
    const uint64_t* offs;       // [nlist + 1]
    const uint8_t* codes;       // [n_vectors x m]
    const float* vterm;         // [n_vectors]
    const float* xnorm;         // [n_vectors] ||xhat||
    const __nv_bfloat16* cbb;   // [m x 256 x dsub] codebooks, bf16
    const uint32_t* seg_off;    // [nlist + 1] pair segments per list
    const uint32_t* unit_list;  // [total units] list of each unit
    const uint4* seg_meta;      // [nq x nprobe] grouped by list: {q << 10 | probe, base, tau, ||Rq||}
    const uint32_t* unit_off;   // [nlist + 1]
    uint32_t* unit_counter;
    unsigned long long* cand;   // [nq x cap] (probe << 32 | position)
    float* mins;                // threshold pass: per (query, tile, warp) minimum upper bound (else null)
    const uint32_t* mins_off;   // [nq] first slot of each query's minima
    uint32_t* cand_cnt;         // [nq]
    int* err;
    int nlist, nprobe, dim, m, k, cap;
};

// 64 bf16 of dims [64 kc, 64 kc + 64) of the decoded entry whose codes start at crow
// (shared memory).
template <int DS>
__device__ __forceinline__ void decode_kchunk_smem(uint32_t (&v)[32], const uint8_t* crow,
                                                   const __nv_bfloat16* __restrict__ cbb, int kc, bool valid) {
    constexpr int SPK = 64 / DS;  // sub-spaces per 64-dim chunk
    if (!valid) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
        return;
    }
    const int s0 = kc * SPK;
    uint32_t cw[(SPK + 3) / 4];
#pragma unroll
    for (int w = 0; w < (SPK + 3) / 4; ++w) cw[w] = reinterpret_cast<const uint32_t*>(crow + s0)[w];
#pragma unroll
    for (int i = 0; i < SPK; ++i) {
        const uint32_t code = (cw[i >> 2] >> ((i & 3) * 8)) & 0xffu;
        const __nv_bfloat16* y = cbb + ((size_t)(s0 + i) * 256 + code) * DS;
        if constexpr (DS == 4) {
            const uint2 t = __ldg(reinterpret_cast<const uint2*>(y));
            v[2 * i] = t.x; v[2 * i + 1] = t.y;
        } else if constexpr (DS == 8) {
            const uint4 t = __ldg(reinterpret_cast<const uint4*>(y));
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        } else {
            const uint4 t0 = __ldg(reinterpret_cast<const uint4*>(y));
            const uint4 t1 = __ldg(reinterpret_cast<const uint4*>(y) + 1);
            v[8 * i] = t0.x; v[8 * i + 1] = t0.y; v[8 * i + 2] = t0.z; v[8 * i + 3] = t0.w;
            v[8 * i + 4] = t1.x; v[8 * i + 5] = t1.y; v[8 * i + 6] = t1.z; v[8 * i + 7] = t1.w;
        }
    }
}

// Decode DB consecutive 64-dim chunks (kc0 .. kc0+DB-1, those < KC) of one entry into TMEM
// columns [32 kc, 32 kc + 32) of this thread's lane.  crow: the entry's codes (shared
// memory); all codebook gathers of the batch are issued before the first store.
// Chunks kc < KT go to this thread's TMEM lane; chunks kc >= KT go to row `row` of the
// 128B-swizzled shared-memory tile a_smem (16 KB per 64-dim chunk).
template <int DS, int DB>
__device__ __forceinline__ void decode_batch(uint32_t tlane, unsigned char* a_smem, int row, const uint8_t* crow,
                                             const __nv_bfloat16* __restrict__ cbb, int kc0, int KC, int KT,
                                             bool valid) {
    uint32_t v[DB][32];
#pragma unroll
    for (int b = 0; b < DB; ++b)
        if (kc0 + b < KC) decode_kchunk_smem<DS>(v[b], crow, cbb, kc0 + b, valid);
#pragma unroll
    for (int b = 0; b < DB; ++b) {
        const int kc = kc0 + b;
        if (kc < KT) {
            tc::tmem_st32(tlane + (uint32_t)(kc * 32), v[b]);
        } else if (kc < KC) {
            unsigned char* atom = a_smem + (size_t)(kc - KT) * (TL_M * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(atom + tc::sw128_offset(row, c)) =
                    make_uint4(v[b][4 * c], v[b][4 * c + 1], v[b][4 * c + 2], v[b][4 * c + 3]);
        }
    }
}

template <int N, int S, int DS>
__global__ void __launch_bounds__(TL_THREADS, 1) tc_list_scan_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                     const TlParams P) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int STAGE_BYTES = N * 128;
    constexpr uint32_t kDcol = 512u - 2u * N;  // two accumulators at the top of TMEM
    const int KC = P.dim / 64;
    // The first KT 64-dim chunks of the tile live in TMEM (columns [0, 32 KT)), the
    // rest in a shared-memory tile after the B ring.
    const int KT = min(KC, (int)(kDcol / 32));
    unsigned char* a_smem = smem + S * STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(a_smem + (KC - KT) * (TL_M * 128));
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;
    uint64_t* acce = accf + 2;
    uint64_t* ufull = acce + 2;   // unit ring: scheduler -> roles
    uint64_t* uempty = ufull + 2; // unit ring: roles -> scheduler
    uint64_t* afull = uempty + 2; // decoded tile in TMEM -> MMA
    uint64_t* drain = afull + 1;
    uint4* meta = reinterpret_cast<uint4*>(drain + 1);    // [2][N] column metadata (16-byte aligned)
    float2* mtest = reinterpret_cast<float2*>(meta + 2 * N);      // [2][N] (||Rq||, keep threshold)
    UnitInfo* units = reinterpret_cast<UnitInfo*>(mtest + 2 * N);  // [2]
    unsigned char* ucodes = reinterpret_cast<unsigned char*>(units + 2);  // [2][128 * m], 16-byte aligned
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ucodes + 2 * TL_M * P.m);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr uint32_t kIdesc = idesc_bf16(N);

    if (tid == 0) {
        for (int s = 0; s < S; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&accf[b], 1);
            tc::mbar_init(&acce[b], 128);
            tc::mbar_init(&ufull[b], 1);
            tc::mbar_init(&uempty[b], 6);  // TMA warp + MMA + 4 decoder warps
        }
        tc::mbar_init(afull, 128);
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tc::smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&](int code) {
        *abort_flag = 1;
        atomicExch(P.err, code);
    };

    if (warp == 6) {
        // ---- scheduler: unit info and the tile's codes into a 2-slot ring.
        const uint32_t total = P.unit_off[P.nlist];
        for (uint32_t it = 0;; ++it) {
            const uint32_t slot = it & 1;
            if (it >= 2 && !tc::mbar_wait(&uempty[slot], ((it >> 1) - 1) & 1)) { fail(21); break; }
            UnitInfo ui{};
            uint32_t u = total;
            if (lane == 0 && !*abort_flag) u = atomicAdd(P.unit_counter, 1u);
            u = __shfl_sync(0xffffffffu, u, 0);
            if (u < total) {
                const uint32_t l = P.unit_list[u];
                const uint32_t r = u - P.unit_off[l];
                const uint32_t s0 = P.seg_off[l], s1 = P.seg_off[l + 1];
                const uint64_t o0 = P.offs[l], o1 = P.offs[l + 1];
                const uint32_t nqg = (s1 - s0 + N * TL_QG - 1) / (N * TL_QG);
                ui.list = l;
                ui.tile = r / nqg;
                ui.pair_begin = s0 + (r % nqg) * (uint32_t)(N * TL_QG);
                ui.pair_end = min(s1, ui.pair_begin + (uint32_t)(N * TL_QG));
                ui.n_chunks = (ui.pair_end - ui.pair_begin + N - 1) / N;
                ui.list_len = (uint32_t)(o1 - o0);
                ui.entry_base = o0 + (unsigned long long)ui.tile * TL_M;
                ui.valid = 1;
                // the tile's codes are contiguous in the CSR array: rows * m bytes
                const uint32_t rows = min((uint32_t)TL_M, ui.list_len - ui.tile * TL_M);
                const uint32_t n16 = rows * (uint32_t)P.m / 16;
                const unsigned char* src = P.codes + ui.entry_base * (unsigned long long)P.m;
                const uint32_t dst = tc::smem_u32(ucodes + slot * TL_M * P.m);
                for (uint32_t i = lane; i < n16; i += 32) cp_async16(dst + i * 16, src + (size_t)i * 16);
                cp_async_commit();
                cp_async_wait<0>();
            }
            if (lane == 0) units[slot] = ui;
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ufull[slot]);
            if (!ui.valid) break;
        }
    } else if (warp == 4) {
        // ---- TMA producer: the chunk's 128 query rows are consecutive rows of the
        // list-ordered query matrix, so each stage is one 128 x 64 tile load.
        uint32_t it_prod = 0;
        if (lane == 0) {
            for (uint32_t it = 0; !*abort_flag; ++it) {
                const uint32_t slot = it & 1;
                if (!tc::mbar_wait(&ufull[slot], (it >> 1) & 1)) { fail(22); break; }
                const UnitInfo ui = units[slot];
                tc::mbar_arrive(&uempty[slot]);
                if (!ui.valid) break;
                bool ok = true;
                for (uint32_t c = 0; c < ui.n_chunks && ok; ++c) {
                    const int y = (int)(ui.pair_begin + c * N);
                    for (int kc = 0; kc < KC; ++kc) {
                        const uint32_t stage = it_prod % S;
                        if (it_prod >= (uint32_t)S && !tc::mbar_wait(&empty[stage], ((it_prod / S) - 1) & 1)) {
                            fail(11);
                            ok = false;
                            break;
                        }
                        tc::mbar_expect_tx(&full[stage], (uint32_t)STAGE_BYTES);
                        tma_load_2d(tc::smem_u32(smem + stage * STAGE_BYTES), &qmap, kc * 64, y, &full[stage]);
                        ++it_prod;
                    }
                }
            }
            // Every load issued has landed before the CTA can exit (normally the MMA
            // already waited for each of them).
            for (uint32_t i = it_prod > (uint32_t)S ? it_prod - S : 0; i < it_prod; ++i)
                if (!tc::mbar_wait(&full[i % S], (i / S) & 1)) { fail(16); break; }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---- MMA issuer: the whole warp runs the loop (uniform control flow keeps the
        // descriptors in uniform registers); one elected lane issues each tcgen05 op.
        uint32_t it_mma = 0, cg_mma = 0;
        auto wwait = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, tc::mbar_wait(bar, parity));
        };
        for (uint32_t it = 0; !*abort_flag; ++it) {
            const uint32_t slot = it & 1;
            if (!wwait(&ufull[slot], (it >> 1) & 1)) { if (lane == 0) fail(23); break; }
            const uint32_t nch = units[slot].n_chunks;
            const uint32_t valid = units[slot].valid;
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&uempty[slot]);
            if (!valid) break;
            if (!wwait(afull, it & 1)) { if (lane == 0) fail(24); break; }
            tc::fence_after_sync();
            bool ok = true;
            for (uint32_t c = 0; c < nch && ok; ++c) {
                const uint32_t buf = cg_mma & 1;
                if (cg_mma >= 2 && !wwait(&acce[buf], ((cg_mma >> 1) - 1) & 1)) {
                    if (lane == 0) fail(12);
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t dcol = tmem + kDcol + buf * (uint32_t)N;
                for (int kc = 0; kc < KC; ++kc) {
                    const uint32_t stage = it_mma % S;
                    if (!wwait(&full[stage], (it_mma / S) & 1)) {
                        if (lane == 0) fail(13);
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_u32(smem + stage * STAGE_BYTES));
                    if (kc < KT) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)  // K = 16 bf16 = 32 bytes per MMA
                            mma_bf16_ts_elect(dcol, tmem + (uint32_t)(kc * 32 + kk * 8), bd + (uint64_t)(kk * 2),
                                              kIdesc, (kc > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        const uint64_t ad =
                            tc::sw128_kmajor_desc(tc::smem_u32(a_smem + (size_t)(kc - KT) * (TL_M * 128)));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_bf16_ss_elect(dcol, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), kIdesc,
                                              (kc > 0 || kk > 0) ? 1u : 0u);
                    }
                    commit_elect(&empty[stage]);
                    ++it_mma;
                }
                commit_elect(&accf[buf]);
                ++cg_mma;
            }
            if (!ok) break;
        }
        // Every tensor-core operation issued has completed before TMEM is freed.
        commit_elect(drain);
        if (!wwait(drain, 0) && lane == 0) atomicExch(P.err, 15);
    } else if (warp < 4) {
        // ---- decoders + epilogue (warps 0-3): thread = entry row of the tile.
        const int row = tid;
        const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
        const uint4 pad = make_uint4(0xffffffffu, 0u, 0u, 0u);
        uint32_t cg_epi = 0;
        for (uint32_t it = 0;; ++it) {
            const uint32_t slot = it & 1;
            const bool got = !*abort_flag && tc::mbar_wait(&ufull[slot], (it >> 1) & 1);
            if (group_any(!got)) {
                if (!got && !*abort_flag) fail(25);
                break;
            }
            const UnitInfo ui = units[slot];
            if (!ui.valid) break;
            const uint32_t pb = ui.pair_begin, pe = ui.pair_end, nch = ui.n_chunks;
            const uint32_t e0 = ui.tile * TL_M;
            const bool vrow = e0 + (uint32_t)row < ui.list_len;
            const float u = vrow ? P.vterm[ui.entry_base + row] : 0.0f;
            const float xn = vrow ? P.xnorm[ui.entry_base + row] : 0.0f;
            uint4 next = pad;
            if (tid < N && pb + (uint32_t)tid < pe) next = P.seg_meta[pb + tid];
            // Decode the tile into TMEM.  This group waited for the previous unit's last
            // accumulator, so the MMAs that read the previous tile have completed.
            tc::fence_after_sync();
            const uint8_t* crow = ucodes + slot * TL_M * P.m + row * P.m;
            for (int kc0 = 0; kc0 < KC; kc0 += 3)
                decode_batch<DS, 3>(tlane, a_smem, row, crow, P.cbb, kc0, KC, KT, vrow);
            tc::tmem_st_wait();
            tc::fence_proxy_async_smem();  // the shared-memory part is read by the tensor core
            tc::fence_before_sync();
            tc::mbar_arrive(afull);
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&uempty[slot]);

            // Keep rule approx - slack <= tau, rearranged as
            //   -2 S - sx ||Rq||  <=  T_col + W_row,
            //   T_col = tau - base + 2^-20 (|base| + |tau|),  W_row = 2^-20 |u| - u,
            // (the extra 2^-20 |tau| covers the rounding of the rearrangement).
            const float sx = (kSlackMul + 2.0f * kSlackAbs) * xn;
            const float wrow = kSlackAbs * fabsf(u) - u;
            const uint32_t pos = e0 + (uint32_t)row;
            bool stop = false;
            for (uint32_t c = 0; c < nch; ++c) {
                const uint32_t buf = cg_epi & 1;
                uint4* bm = meta + buf * N;
                float2* bt = mtest + buf * N;
                if (tid < N) {
                    bm[tid] = next;
                    const float bj = __uint_as_float(next.y), tq = __uint_as_float(next.z);
                    bt[tid] = next.x == 0xffffffffu
                                  ? make_float2(0.0f, -FLT_MAX)
                                  : make_float2(__uint_as_float(next.w),
                                                (tq - bj) + kSlackAbs * (fabsf(bj) + fabsf(tq)));
                    const uint32_t pi = pb + (c + 1) * N + (uint32_t)tid;
                    next = (c + 1 < nch && pi < pe) ? P.seg_meta[pi] : pad;
                }
                // One decision for the whole group (the named barrier also publishes the
                // column metadata written above).
                const bool ok = !*abort_flag && tc::mbar_wait(&accf[buf], (cg_epi >> 1) & 1);
                if (group_any(!ok)) {
                    if (!ok && !*abort_flag) fail(14);
                    stop = true;
                    break;
                }
                tc::fence_after_sync();
#pragma unroll
                for (int h = 0; h < N / 32; ++h) {
                    uint32_t acc[32];
                    tc::tmem_ld32(tlane + kDcol + buf * (uint32_t)N + h * 32, acc);
                    tc::tmem_ld_wait();
                    if (h == N / 32 - 1) {
                        tc::fence_before_sync();
                        tc::mbar_arrive(&acce[buf]);
                    }
                    if (P.mins) {
                        // Threshold pass: lane j records, for column h*32+j, the smallest
                        // upper bound (approx + slack) among this warp's 32 rows.
                        float mine = FLT_MAX;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const uint4 md = bm[h * 32 + j];
                            const float bj = __uint_as_float(md.y);
                            float ub = FLT_MAX;
                            if (vrow) {
                                const float approx = fmaf(-2.0f, __uint_as_float(acc[j]), bj + u);
                                ub = approx + fmaf(sx, __uint_as_float(md.w), kSlackAbs * (fabsf(bj) + fabsf(u)));
                            }
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) ub = fminf(ub, __shfl_xor_sync(0xffffffffu, ub, o));
                            if (lane == j) mine = ub;
                        }
                        const uint32_t qt = bm[h * 32 + lane].x;
                        if (qt != 0xffffffffu)
                            P.mins[P.mins_off[qt >> 10] + ui.tile * 4 + warp] = mine;
                        continue;
                    }
                    uint32_t mask = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float2 t = bt[h * 32 + j];
                        const float lhs = fmaf(-sx, t.x, -2.0f * __uint_as_float(acc[j]));
                        mask |= (lhs <= t.y + wrow) ? (1u << j) : 0u;
                    }
                    if (!vrow) mask = 0;
                    while (mask) {
                        const int j = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const uint32_t qt = bm[h * 32 + j].x;
                        const uint32_t q = qt >> 10;
                        const uint32_t slot2 = atomicAdd(&P.cand_cnt[q], 1u);
                        if (slot2 < (uint32_t)P.cap)
                            P.cand[(size_t)q * P.cap + slot2] = ((unsigned long long)(qt & 1023u) << 32) | pos;
                    }
                }
                ++cg_epi;
            }
            if (stop) break;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

// ---------------------------------------------------------------------------------
// The same screen on CTA pairs (clusters of two, tcgen05 cta_group::2).  A unit covers
// two consecutive 128-entry tiles of a list; CTA r of the pair decodes tile 2p + r into
// its own tensor memory (rows 128 r .. 128 r + 127 of an M = 256 A operand) and streams
// half of each chunk's N query rows (N/2 rows per stage) into its own shared memory.
// The pair's leader (rank 0) issues tcgen05.mma.cta_group::2 M = 256: each SM reads only
// its half of the query tile, halving the shared-memory traffic per MMA, and each CTA's
// tensor memory receives the accumulator rows of its own tile.  Roles as in the
// single-CTA kernel; in addition the leader's scheduler picks the units and publishes
// them to the peer, the peer's TMA loads complete on the leader's stage barriers, the
// leader's commits arrive on the barriers of both CTAs, and the peer's decoders and
// epilogue arrive on the leader's barriers.
// ---------------------------------------------------------------------------------
namespace {
__device__ __forceinline__ void mma2_ss_elect(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma2_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Commit of this thread's earlier tcgen05 operations to the mbarrier at cluster address
// caddr (this CTA's or the peer's).
__device__ __forceinline__ void commit2_elect(uint32_t caddr) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
        ::"r"(caddr)
        : "memory");
}
// A box of 64 bf16 columns x (N/2) rows into this CTA's shared memory; the bytes complete
// on the mbarrier at cluster address mbar (the pair leader's stage barrier).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
        : "memory");
}
// Arrive on a barrier of the pair leader (local arrive on the leader itself).
__device__ __forceinline__ void arrive_leader(uint64_t* bar, bool leader) {
    if (leader) tc::mbar_arrive(bar);
    else tc::mbar_arrive_cluster(tc::peer_addr(bar, 0));
}
}  // namespace

template <int N, int S, int DS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TL_THREADS, 1)
    tc_list_scan2_kernel(const __grid_constant__ CUtensorMap qmap, const TlParams P) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int HN = N / 2;                 // query rows per CTA per chunk
    constexpr int STAGE_BYTES = HN * 128;
    constexpr uint32_t kDcol = 512u - 2u * N;
    const int KC = P.dim / 64;
    const int KT = min(KC, (int)(kDcol / 32));
    unsigned char* a_smem = smem + S * STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(a_smem + (KC - KT) * (TL_M * 128));
    uint64_t* empty = full + S;
    uint64_t* accf = empty + S;
    uint64_t* acce = accf + 2;
    uint64_t* ufull = acce + 2;
    uint64_t* uempty = ufull + 2;
    uint64_t* uann = uempty + 2;   // peer: unit published by the leader's scheduler
    uint64_t* ureq = uann + 2;     // leader: the peer released a unit slot
    uint64_t* afull = ureq + 2;
    uint64_t* drain = afull + 1;
    uint4* meta = reinterpret_cast<uint4*>(drain + 1);
    float2* mtest = reinterpret_cast<float2*>(meta + 2 * N);
    UnitInfo* units = reinterpret_cast<UnitInfo*>(mtest + 2 * N);
    unsigned char* ucodes = reinterpret_cast<unsigned char*>(units + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ucodes + 2 * TL_M * P.m);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = tc::cluster_rank();
    const bool leader = rank == 0;
    constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (16u << 24);  // M 256

    if (tid == 0) {
        for (int s = 0; s < S; ++s) { tc::mbar_init(&full[s], 1); tc::mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&accf[b], 1);
            tc::mbar_init(&acce[b], 2 * 128);
            tc::mbar_init(&ufull[b], 1);
            tc::mbar_init(&uempty[b], 6);  // TMA warp + MMA warp + 4 decoder warps
            tc::mbar_init(&uann[b], 1);
            tc::mbar_init(&ureq[b], 1);
        }
        tc::mbar_init(afull, 2 * 128);
        tc::mbar_init(drain, 1);
        *abort_flag = 0;
        tc::mbar_init_fence();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tc::smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::cluster_sync();  // the peer's barriers exist before anything arrives on them
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t peer = rank ^ 1u;

    auto fail = [&](int code) {
        *abort_flag = 1;
        tc::st_cluster_u32(tc::peer_addr((const void*)abort_flag, peer), 1u);
        atomicExch(P.err, code);
    };

    if (warp == 6) {
        // ---- scheduler.  The leader takes units from the global counter and publishes
        // each to the peer (unit slot copy + arrive on the peer's uann); each CTA then
        // prefetches the codes of its own tile.
        const uint32_t total = P.unit_off[P.nlist];
        for (uint32_t it = 0;; ++it) {
            const uint32_t slot = it & 1;
            UnitInfo ui{};
            if (leader) {
                if (it >= 2) {
                    const bool ok = tc::mbar_wait(&uempty[slot], ((it >> 1) - 1) & 1) &&
                                    tc::mbar_wait_cluster(&ureq[slot], ((it >> 1) - 1) & 1);
                    if (!__all_sync(0xffffffffu, ok)) { if (lane == 0) fail(31); break; }
                }
                uint32_t u = total;
                if (lane == 0 && !*abort_flag) u = atomicAdd(P.unit_counter, 1u);
                u = __shfl_sync(0xffffffffu, u, 0);
                if (u < total) {
                    const uint32_t l = P.unit_list[u];
                    const uint32_t r = u - P.unit_off[l];
                    const uint32_t s0 = P.seg_off[l], s1 = P.seg_off[l + 1];
                    const uint64_t o0 = P.offs[l], o1 = P.offs[l + 1];
                    const uint32_t nqg = (s1 - s0 + N * TL_QG - 1) / (N * TL_QG);
                    ui.list = l;
                    ui.tile = r / nqg;  // tile pair
                    ui.pair_begin = s0 + (r % nqg) * (uint32_t)(N * TL_QG);
                    ui.pair_end = min(s1, ui.pair_begin + (uint32_t)(N * TL_QG));
                    ui.n_chunks = (ui.pair_end - ui.pair_begin + N - 1) / N;
                    ui.list_len = (uint32_t)(o1 - o0);
                    ui.entry_base = o0;
                    ui.valid = 1;
                }
                // publish to the peer's slot, then signal it
                if (lane == 0) {
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(&ui);
                    const uint32_t dst = tc::peer_addr(&units[slot], peer);
                    for (int i = 0; i < (int)(sizeof(UnitInfo) / 4); ++i) tc::st_cluster_u32(dst + 4 * i, w[i]);
                    tc::mbar_arrive_cluster(tc::peer_addr(&uann[slot], peer));
                }
            } else {
                if (it >= 2) {
                    const bool ok = tc::mbar_wait(&uempty[slot], ((it >> 1) - 1) & 1);
                    if (!__all_sync(0xffffffffu, ok)) { if (lane == 0) fail(32); break; }
                    if (lane == 0) tc::mbar_arrive_cluster(tc::peer_addr(&ureq[slot], peer));
                }
                if (!__all_sync(0xffffffffu, tc::mbar_wait_cluster(&uann[slot], (it >> 1) & 1))) {
                    if (lane == 0) fail(33);
                    break;
                }
                ui = units[slot];
            }
            if (ui.valid) {
                // this CTA's tile of the pair: codes contiguous in the CSR array
                const uint32_t tile = 2 * ui.tile + rank;
                const uint32_t e0 = tile * TL_M;
                const uint32_t rows = e0 < ui.list_len ? min((uint32_t)TL_M, ui.list_len - e0) : 0u;
                const uint32_t n16 = rows * (uint32_t)P.m / 16;
                const unsigned char* src = P.codes + (ui.entry_base + e0) * (unsigned long long)P.m;
                const uint32_t dst = tc::smem_u32(ucodes + slot * TL_M * P.m);
                for (uint32_t i = lane; i < n16; i += 32) cp_async16(dst + i * 16, src + (size_t)i * 16);
                cp_async_commit();
                cp_async_wait<0>();
            }
            if (leader && lane == 0) units[slot] = ui;
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&ufull[slot]);
            if (!ui.valid) break;
        }
    } else if (warp == 4) {
        // ---- TMA producer: this CTA's N/2 query rows of each chunk, one 64 x N/2 tile
        // load per stage; the bytes complete on the leader's stage barrier.
        uint32_t it_prod = 0;
        if (lane == 0) {
            for (uint32_t it = 0; !*abort_flag; ++it) {
                const uint32_t slot = it & 1;
                if (!tc::mbar_wait(&ufull[slot], (it >> 1) & 1)) { fail(22); break; }
                const UnitInfo ui = units[slot];
                tc::mbar_arrive(&uempty[slot]);
                if (!ui.valid) break;
                bool ok = true;
                for (uint32_t c = 0; c < ui.n_chunks && ok; ++c) {
                    const int y = (int)(ui.pair_begin + c * N + rank * HN);
                    for (int kc = 0; kc < KC; ++kc) {
                        const uint32_t stage = it_prod % S;
                        if (it_prod >= (uint32_t)S && !tc::mbar_wait(&empty[stage], ((it_prod / S) - 1) & 1)) {
                            fail(11);
                            ok = false;
                            break;
                        }
                        if (leader) tc::mbar_expect_tx(&full[stage], 2u * STAGE_BYTES);
                        tma_load_2d_pair(tc::smem_u32(smem + stage * STAGE_BYTES), &qmap, kc * 64, y,
                                         leader ? tc::smem_u32(&full[stage]) : tc::peer_addr(&full[stage], 0));
                        ++it_prod;
                    }
                }
            }
            // The leader's last stages have landed (both halves) before the pair can exit.
            if (leader)
                for (uint32_t i = it_prod > (uint32_t)S ? it_prod - S : 0; i < it_prod; ++i)
                    if (!tc::mbar_wait(&full[i % S], (i / S) & 1)) { fail(16); break; }
        }
        __syncwarp();
    } else if (warp == 5) {
        // ---- MMA issuer (leader only); the peer's warp follows the unit ring.
        uint32_t it_mma = 0, cg_mma = 0;
        auto wwait = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, tc::mbar_wait_cluster(bar, parity));
        };
        for (uint32_t it = 0; !*abort_flag; ++it) {
            const uint32_t slot = it & 1;
            if (!wwait(&ufull[slot], (it >> 1) & 1)) { if (lane == 0) fail(23); break; }
            const uint32_t nch = units[slot].n_chunks;
            const uint32_t valid = units[slot].valid;
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&uempty[slot]);
            if (!valid) break;
            if (!leader) continue;
            if (!wwait(afull, it & 1)) { if (lane == 0) fail(24); break; }
            tc::fence_after_sync();
            bool ok = true;
            for (uint32_t c = 0; c < nch && ok; ++c) {
                const uint32_t buf = cg_mma & 1;
                if (cg_mma >= 2 && !wwait(&acce[buf], ((cg_mma >> 1) - 1) & 1)) {
                    if (lane == 0) fail(12);
                    ok = false;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t dcol = tmem + kDcol + buf * (uint32_t)N;
                for (int kc = 0; kc < KC; ++kc) {
                    const uint32_t stage = it_mma % S;
                    if (!wwait(&full[stage], (it_mma / S) & 1)) {
                        if (lane == 0) fail(13);
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint64_t bd = tc::sw128_kmajor_desc(tc::smem_u32(smem + stage * STAGE_BYTES));
                    if (kc < KT) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma2_ts_elect(dcol, tmem + (uint32_t)(kc * 32 + kk * 8), bd + (uint64_t)(kk * 2), kIdesc,
                                          (kc > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        const uint64_t ad =
                            tc::sw128_kmajor_desc(tc::smem_u32(a_smem + (size_t)(kc - KT) * (TL_M * 128)));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma2_ss_elect(dcol, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), kIdesc,
                                          (kc > 0 || kk > 0) ? 1u : 0u);
                    }
                    commit2_elect(tc::smem_u32(&empty[stage]));
                    commit2_elect(tc::peer_addr(&empty[stage], 1));
                    ++it_mma;
                }
                commit2_elect(tc::smem_u32(&accf[buf]));
                commit2_elect(tc::peer_addr(&accf[buf], 1));
                ++cg_mma;
            }
            if (!ok) break;
        }
        if (leader) {
            // Every tensor-core operation issued has completed before TMEM is freed.
            commit2_elect(tc::smem_u32(drain));
            if (!wwait(drain, 0) && lane == 0) atomicExch(P.err, 15);
        }
    } else if (warp < 4) {
        // ---- decoders + epilogue (warps 0-3): thread = entry row of this CTA's tile.
        const int row = tid;
        const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
        const uint4 pad = make_uint4(0xffffffffu, 0u, 0u, 0u);
        uint32_t cg_epi = 0;
        for (uint32_t it = 0;; ++it) {
            const uint32_t slot = it & 1;
            const bool got = !*abort_flag && tc::mbar_wait(&ufull[slot], (it >> 1) & 1);
            if (group_any(!got)) {
                if (!got && !*abort_flag) fail(25);
                break;
            }
            const UnitInfo ui = units[slot];
            if (!ui.valid) break;
            const uint32_t pb = ui.pair_begin, pe = ui.pair_end, nch = ui.n_chunks;
            const uint32_t tile = 2 * ui.tile + rank;
            const uint32_t e0 = tile * TL_M;
            const bool vrow = e0 + (uint32_t)row < ui.list_len;
            const unsigned long long ebase = ui.entry_base + e0;
            const float u = vrow ? P.vterm[ebase + row] : 0.0f;
            const float xn = vrow ? P.xnorm[ebase + row] : 0.0f;
            uint4 next = pad;
            if (tid < N && pb + (uint32_t)tid < pe) next = P.seg_meta[pb + tid];
            tc::fence_after_sync();
            const uint8_t* crow = ucodes + slot * TL_M * P.m + row * P.m;
            for (int kc0 = 0; kc0 < KC; kc0 += 3)
                decode_batch<DS, 3>(tlane, a_smem, row, crow, P.cbb, kc0, KC, KT, vrow);
            tc::tmem_st_wait();
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            arrive_leader(afull, leader);
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&uempty[slot]);

            const float sx = (kSlackMul + 2.0f * kSlackAbs) * xn;
            const float wrow = kSlackAbs * fabsf(u) - u;
            const uint32_t pos = e0 + (uint32_t)row;
            bool stop = false;
            for (uint32_t c = 0; c < nch; ++c) {
                const uint32_t buf = cg_epi & 1;
                uint4* bm = meta + buf * N;
                float2* bt = mtest + buf * N;
                if (tid < N) {
                    bm[tid] = next;
                    const float bj = __uint_as_float(next.y), tq = __uint_as_float(next.z);
                    bt[tid] = next.x == 0xffffffffu
                                  ? make_float2(0.0f, -FLT_MAX)
                                  : make_float2(__uint_as_float(next.w),
                                                (tq - bj) + kSlackAbs * (fabsf(bj) + fabsf(tq)));
                    const uint32_t pi = pb + (c + 1) * N + (uint32_t)tid;
                    next = (c + 1 < nch && pi < pe) ? P.seg_meta[pi] : pad;
                }
                const bool ok = !*abort_flag && tc::mbar_wait_cluster(&accf[buf], (cg_epi >> 1) & 1);
                if (group_any(!ok)) {
                    if (!ok && !*abort_flag) fail(14);
                    stop = true;
                    break;
                }
                tc::fence_after_sync();
#pragma unroll
                for (int h = 0; h < N / 32; ++h) {
                    uint32_t acc[32];
                    tc::tmem_ld32(tlane + kDcol + buf * (uint32_t)N + h * 32, acc);
                    tc::tmem_ld_wait();
                    if (h == N / 32 - 1) {
                        tc::fence_before_sync();
                        arrive_leader(&acce[buf], leader);
                    }
                    if (P.mins) {
                        float mine = FLT_MAX;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const uint4 md = bm[h * 32 + j];
                            const float bj = __uint_as_float(md.y);
                            float ub = FLT_MAX;
                            if (vrow) {
                                const float approx = fmaf(-2.0f, __uint_as_float(acc[j]), bj + u);
                                ub = approx + fmaf(sx, __uint_as_float(md.w), kSlackAbs * (fabsf(bj) + fabsf(u)));
                            }
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) ub = fminf(ub, __shfl_xor_sync(0xffffffffu, ub, o));
                            if (lane == j) mine = ub;
                        }
                        const uint32_t qt = bm[h * 32 + lane].x;
                        if (qt != 0xffffffffu && e0 < ui.list_len)
                            P.mins[P.mins_off[qt >> 10] + tile * 4 + warp] = mine;
                        continue;
                    }
                    uint32_t mask = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float2 t = bt[h * 32 + j];
                        const float lhs = fmaf(-sx, t.x, -2.0f * __uint_as_float(acc[j]));
                        mask |= (lhs <= t.y + wrow) ? (1u << j) : 0u;
                    }
                    if (!vrow) mask = 0;
                    while (mask) {
                        const int j = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const uint32_t qt = bm[h * 32 + j].x;
                        const uint32_t q = qt >> 10;
                        const uint32_t slot2 = atomicAdd(&P.cand_cnt[q], 1u);
                        if (slot2 < (uint32_t)P.cap)
                            P.cand[(size_t)q * P.cap + slot2] = ((unsigned long long)(qt & 1023u) << 32) | pos;
                    }
                }
                ++cg_epi;
            }
            if (stop) break;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::cluster_sync();  // neither CTA frees its TMEM or exits while the pair still works
    tc::fence_after_sync();
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
}

// ---------------------------------------------------------------------------------
// Batch preparation: bf16 queries and norms, pair grouping by list, unit counts.
// ---------------------------------------------------------------------------------
__global__ void query_prep_kernel(const float* __restrict__ rq, long long nq, int dim, __nv_bfloat16* __restrict__ rqb,
                                  float* __restrict__ rqn) {
    const int lane = threadIdx.x & 31;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long q = w; q < nq; q += nw) {
        float s = 0.0f;
        for (int d = lane; d < dim; d += 32) {
            const float v = rq[q * dim + d];
            rqb[q * dim + d] = __float2bfloat16_rn(v);
            s = fmaf(v, v, s);
        }
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) rqn[q] = sqrtf(s) * 1.0000005f;
    }
}

// Per query: nearest-list size L0; queries with L0 > small_max (and k <= 256) get their
// threshold from the tensor-core pass over that list (pair kept in p0, 4 minima per
// 128-entry tile), the others from the blocked scan (run flag).
// Queries outside this shard's share (q mod shards != shard) get no threshold pass:
// tau = -FLT_MAX (no bound) until the threshold exchange brings another shard's.  A
// query whose nearest list holds fewer than short_len entries here is bounded on every
// shard all the same: its owner's part of the list may hold fewer than k entries and
// give no bound, and such a pass is cheap.
__global__ void home_split_kernel(const uint32_t* __restrict__ probe, int nprobe, const float* __restrict__ pbase,
                                  const uint64_t* __restrict__ offs, long long nq, uint32_t small_max, int big_ok,
                                  uint32_t shard, uint32_t shards, uint64_t short_len, uint32_t* __restrict__ p0,
                                  float* __restrict__ pbase0, uint32_t* __restrict__ mcount,
                                  uint32_t* __restrict__ run_lut, float* __restrict__ tau) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        const uint32_t l = probe[q * nprobe];
        const uint64_t L0 = offs[l + 1] - offs[l];
        const bool mine = shards <= 1 || (uint32_t)(q % shards) == shard || L0 < short_len;
        const bool big = mine && big_ok && L0 > small_max;
        p0[q] = big ? l : kSkipPair;
        pbase0[q] = pbase[q * nprobe];
        mcount[q] = big ? (uint32_t)(4 * ((L0 + 127) / 128)) : 0u;
        run_lut[q] = (mine && !big) ? 1u : 0u;
        if (!mine) tau[q] = -FLT_MAX;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) mcount[nq] = 0;
}

// tau[q] = k-th smallest of the query's minima (radix select on order-preserving keys,
// one CTA per query with minima).
__global__ void __launch_bounds__(256) minima_select_kernel(const float* __restrict__ mins,
                                                            const uint32_t* __restrict__ mins_off,
                                                            const uint32_t* __restrict__ mcount, int k,
                                                            float* __restrict__ tau) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t remaining, thresh;
    const long long q = blockIdx.x;
    const uint32_t n = mcount[q];
    if (n == 0) return;
    const float* v = mins + mins_off[q];
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, mask = 0;
    if (threadIdx.x == 0) remaining = (uint32_t)min((uint32_t)k, n);
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += 256) hist[i] = 0;
        __syncthreads();
        for (uint32_t c0 = 0; c0 < n; c0 += 256) {
            const uint32_t c = c0 + threadIdx.x;
            uint32_t key = 0;
            bool part = false;
            if (c < n) {
                key = float_key(v[c]);
                part = (key & mask) == prefix;
            }
            const unsigned act = __ballot_sync(0xffffffffu, part);
            if (act) {
                const uint32_t bin = (key >> shift) & 255u;
                const uint32_t bin0 = __shfl_sync(0xffffffffu, bin, __ffs(act) - 1);
                const unsigned same = __ballot_sync(0xffffffffu, part && bin == bin0);
                if (lane == __ffs(act) - 1) atomicAdd(&hist[bin0], (uint32_t)__popc(same));
                if (part && bin != bin0) atomicAdd(&hist[bin], 1u);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t rem = remaining, acc = 0, b = 0;
            for (; b < 256; ++b) { const uint32_t h = hist[b]; if (acc + h >= rem) break; acc += h; }
            remaining = rem - acc;
            thresh = b;
        }
        __syncthreads();
        prefix |= thresh << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    // fewer than k finite minima: no usable threshold
    if (threadIdx.x == 0) {
        const float t = key_float(prefix);
        tau[q] = (n >= (uint32_t)k && t < FLT_MAX) ? t : -FLT_MAX;
    }
}

// tau from the blocked scan for the queries it ran on (run_lut), overflow marks.
__global__ void tau_merge_kernel(const float* __restrict__ p1_d, const uint32_t* __restrict__ p1_n,
                                 const uint32_t* __restrict__ run_lut, long long nq, int k, int cap,
                                 float* __restrict__ tau, uint32_t* __restrict__ cand_cnt) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        if (run_lut[q]) tau[q] = p1_n[q] == (uint32_t)k ? p1_d[q * k + k - 1] : -FLT_MAX;
        cand_cnt[q] = tau[q] > -FLT_MAX ? 0u : (uint32_t)cap + 1u;
    }
}

// Threshold exchange between shards: tau_x = tau where this shard has a bound, else
// +inf; after the element-wise minimum over the shards, every query whose minimum is
// finite takes it (and is screened, not sent to the fallback scan).  Any shard's bound
// is an upper bound of the k-th distance over the union of the shards, so every entry
// of the union's top k still passes each shard's keep rule.
__global__ void tau_export_kernel(const float* __restrict__ tau, long long nq, float* __restrict__ tau_x) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x)
        tau_x[q] = tau[q] > -FLT_MAX ? tau[q] : __int_as_float(0x7f800000);
}

__global__ void tau_import_kernel(const float* __restrict__ tau_x, long long nq, int cap, float* __restrict__ tau,
                                  uint32_t* __restrict__ cand_cnt) {
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        const float t = tau_x[q];
        if (t < __int_as_float(0x7f800000) && t > -FLT_MAX) tau[q] = fminf(tau[q] > -FLT_MAX ? tau[q] : t, t);
        cand_cnt[q] = tau[q] > -FLT_MAX ? 0u : (uint32_t)cap + 1u;
    }
}

__global__ void cand_stats_kernel(const uint32_t* __restrict__ cand_cnt, long long nq, uint32_t cap,
                                  unsigned long long* __restrict__ stats) {
    unsigned long long c = 0, f = 0;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < nq; q += (long long)gridDim.x * blockDim.x) {
        const uint32_t n = cand_cnt[q];
        if (n > cap) ++f; else c += n;
    }
    for (int o = 16; o > 0; o >>= 1) {
        c += __shfl_xor_sync(0xffffffffu, c, o);
        f += __shfl_xor_sync(0xffffffffu, f, o);
    }
    if ((threadIdx.x & 31) == 0 && (c | f)) {
        atomicAdd(&stats[0], c);
        atomicAdd(&stats[1], f);
    }
}

// qperm[i] = rqb[q(i)]: the bf16 query rows in the list-grouped pair order (one warp
// per row, 16-byte copies); *total = number of grouped pairs.
__global__ void qperm_kernel(const uint4* __restrict__ seg_meta, const uint32_t* __restrict__ total,
                             const uint4* __restrict__ rqb, int row16, uint4* __restrict__ qperm) {
    const long long npairs = *total;
    const int lane = threadIdx.x & 31;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long i = w; i < npairs; i += nw) {
        const uint32_t q = __ldg(&seg_meta[i].x) >> 10;
        for (int c = lane; c < row16; c += 32) qperm[i * row16 + c] = __ldg(&rqb[(long long)q * row16 + c]);
    }
}

__global__ void pair_hist_kernel(const uint32_t* __restrict__ probe, long long npairs, uint32_t* __restrict__ cnt) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npairs;
         i += (long long)gridDim.x * blockDim.x)
        if (probe[i] != kSkipPair) atomicAdd(&cnt[probe[i]], 1u);
}

// Pairs grouped by list, each with the metadata the screen's epilogue needs:
// {q << 10 | probe index, base term, tau(q), ||Rq||}.
__global__ void pair_scatter_kernel(const uint32_t* __restrict__ probe, long long npairs, int nprobe,
                                    const uint32_t* __restrict__ seg_off, uint32_t* __restrict__ cursor,
                                    const float* __restrict__ pbase, const float* __restrict__ tau,
                                    const float* __restrict__ rqn, uint4* __restrict__ seg_meta) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < npairs;
         i += (long long)gridDim.x * blockDim.x) {
        const uint32_t l = probe[i];
        if (l == kSkipPair) continue;
        const uint32_t q = (uint32_t)(i / nprobe), t = (uint32_t)(i - (long long)q * nprobe);
        seg_meta[seg_off[l] + atomicAdd(&cursor[l], 1u)] =
            make_uint4((q << 10) | t, __float_as_uint(pbase[i]), __float_as_uint(tau[q]), __float_as_uint(rqn[q]));
    }
}

// unit_list[u] = the list unit u belongs to (unit_off[l] <= u < unit_off[l + 1]).
__global__ void unit_fill_kernel(const uint32_t* __restrict__ unit_off, int nlist, uint32_t* __restrict__ unit_list) {
    const uint32_t total = unit_off[nlist];
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += gridDim.x * blockDim.x) {
        int lo = 0, hi = nlist;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (unit_off[mid] <= u) lo = mid; else hi = mid;
        }
        unit_list[u] = (uint32_t)lo;
    }
}

// unit_rows: entries per unit (128 for single CTAs, 256 for CTA pairs).
__global__ void unit_count_kernel(const uint32_t* __restrict__ cnt, const uint64_t* __restrict__ offs, int nlist,
                                  int n_cols, int unit_rows, uint32_t* __restrict__ units) {
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l > nlist) return;
    if (l == nlist) { units[l] = 0; return; }
    const uint32_t c = cnt[l];
    const uint64_t L = offs[l + 1] - offs[l];
    units[l] = (c == 0 || L == 0) ? 0u
                                  : (uint32_t)((L + unit_rows - 1) / unit_rows) *
                                        ((c + (uint32_t)(n_cols * TL_QG) - 1) / (uint32_t)(n_cols * TL_QG));
}

// ---------------------------------------------------------------------------------
// Refine: exact FAST distances of the candidates (the blocked scan's arithmetic and
// scan positions), then the k smallest keys.  Queries whose candidate list overflowed
// are left to the blocked scan.
//
// The blocked scan adds the query's lookup-table entries T[s][c] = -2 * (fma chain over
// t < dsub of rq[s dsub + t] * y[s][c][t], from 0, t ascending: every table kernel's
// arithmetic) in the lane-rotated sub-space order.  A query with more than table_min
// candidates reads its table (m x 256 floats, one bulk copy into shared memory); one with
// fewer computes just the entries its candidates use from the rotated query and the fp32
// codebook rows (m rows of dsub floats per candidate, L2-resident).  Both give the same
// floats, so the result is the blocked scan's bit for bit.  The table path is the default
// for every query: on the 10M x 768 benchmark batch the refine takes 0.7 ms with it and
// 1.2 ms with the computed entries below 64 candidates (each entry waits on a code load
// and then a codebook row from L2, m times in sequence per candidate).
// ---------------------------------------------------------------------------------
constexpr uint32_t kRefineTableMin = 0;   // VGPU_REFINE_TABLE_MIN overrides it

template <int MC, int G, int DS>
__global__ void __launch_bounds__(256) tl_refine_kernel(const float* __restrict__ T, const float* __restrict__ rq,
                                                        int dim, const float* __restrict__ cb,
                                                        const uint32_t* __restrict__ probe, int nprobe,
                                                        const float* __restrict__ pbase,
                                                        const uint64_t* __restrict__ offs,
                                                        const uint8_t* __restrict__ codes,
                                                        const float* __restrict__ vterm,
                                                        const uint64_t* __restrict__ ids,
                                                        const unsigned long long* __restrict__ cand,
                                                        const uint32_t* __restrict__ cand_cnt, int cap, int k,
                                                        uint64_t* __restrict__ out_ids, float* __restrict__ out_d,
                                                        uint32_t* __restrict__ out_n, int* __restrict__ err,
                                                        uint32_t table_min) {
    // Shared memory: [barrier, 16 B][region: the table, later the sort keys][rq][eprefix].
    // With the table, the keys (at most KPT per thread, in registers meanwhile) overwrite
    // it once every candidate is scored, so a CTA needs little more than one table.
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int m = MC;
    constexpr int KPT = 16;                                                          // keys per thread
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);
    const int tbytes = m * 256 * 4;
    const int region = tbytes > next_pow2(cap) * 8 ? tbytes : next_pow2(cap) * 8;
    float* lut = reinterpret_cast<float*>(smem_raw + 16);                             // [m * 256]
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw + 16);  // [next_pow2(cap)]
    float* rqs = reinterpret_cast<float*>(smem_raw + 16 + region);                    // [dim]
    uint32_t* eprefix = reinterpret_cast<uint32_t*>(rqs + ((dim + 3) & ~3));          // [nprobe + 1]
    const long long q = blockIdx.x;
    const uint32_t n = cand_cnt[q];
    if (n > (uint32_t)cap) return;
    const int p2 = next_pow2(n < 2 ? 2 : (int)n);
    const bool table = n > table_min;
    const float* tq = T + q * (long long)m * 256;
    if (table) tc::lut_stage_begin(lut, tq, (uint32_t)tbytes, bar);
    else for (int i = threadIdx.x; i < dim; i += 256) rqs[i] = rq[q * dim + i];
    if (threadIdx.x < 32) probe_prefixes_warp(probe + q * nprobe, nprobe, offs, nullptr, eprefix, nullptr);

    if (!table) {
        __syncthreads();
        for (int i = threadIdx.x; i < p2; i += 256) {
            unsigned long long key = ~0ull;
            if (i < (int)n) {
                const unsigned long long c = cand[q * cap + i];
                const uint32_t t = (uint32_t)(c >> 32), p = (uint32_t)c;
                const uint64_t e = offs[probe[q * nprobe + t]] + p;
                const uint8_t* cr = codes + e * m;
                const int lane = (int)((p & 127u) >> 2);
                float acc = 0.0f;
#pragma unroll 4
                for (int r = 0; r < m; ++r) {
                    const int sub = (r / G) * G + ((lane + r) & (G - 1));
                    const float4* y = reinterpret_cast<const float4*>(cb + ((long long)sub * 256 + cr[sub]) * DS);
                    const float* x = rqs + sub * DS;
                    float a = 0.0f;
#pragma unroll
                    for (int v = 0; v < DS / 4; ++v) {
                        const float4 yv = __ldg(y + v);
                        a = fmaf(x[4 * v + 0], yv.x, a);
                        a = fmaf(x[4 * v + 1], yv.y, a);
                        a = fmaf(x[4 * v + 2], yv.z, a);
                        a = fmaf(x[4 * v + 3], yv.w, a);
                    }
                    acc = __fadd_rn(acc, -2.0f * a);
                }
                const float dist = (pbase[q * nprobe + t] + vterm[e]) + acc;
                key = ((unsigned long long)float_key(dist) << 32) | (eprefix[t] + p);
            }
            keys[i] = key;
        }
    } else {
        // Candidate metadata while the table is in flight.
        const uint8_t* crow[KPT];
        float dbase[KPT];
        uint32_t slot[KPT], pos[KPT];
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = (int)threadIdx.x + j * 256;
            crow[j] = nullptr;
            dbase[j] = 0.0f;
            slot[j] = pos[j] = 0;
            if (i < (int)n) {
                const unsigned long long c = cand[q * cap + i];
                const uint32_t t = (uint32_t)(c >> 32), p = (uint32_t)c;
                const uint64_t e = offs[probe[q * nprobe + t]] + p;
                crow[j] = codes + e * m;
                dbase[j] = pbase[q * nprobe + t] + vterm[e];
                slot[j] = t;
                pos[j] = p;
            }
        }
        if (!tc::lut_stage_wait(lut, tq, (uint32_t)tbytes, bar) && threadIdx.x == 0 && err) atomicExch(err, 41);
        unsigned long long kr[KPT];
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            kr[j] = ~0ull;
            if (crow[j] != nullptr) {
                const int lane = (int)((pos[j] & 127u) >> 2);
                const uint8_t* cr = crow[j];
                float acc = 0.0f;
#pragma unroll 8
                for (int r = 0; r < m; ++r) {
                    const int g = r / G, s_lo = (lane + r) & (G - 1);
                    acc += lut[(g * 256 + cr[g * G + s_lo]) * G + s_lo];
                }
                const float dist = dbase[j] + acc;
                kr[j] = ((unsigned long long)float_key(dist) << 32) | (eprefix[slot[j]] + pos[j]);
            }
        }
        __syncthreads();  // every read of the table is done: the keys take its place
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = (int)threadIdx.x + j * 256;
            if (i < p2) keys[i] = kr[j];
        }
    }
    bitonic_sort_u64<256>(keys, p2);
    const int h = (int)n < k ? (int)n : k;
    for (int i = threadIdx.x; i < k; i += 256) {
        if (i < h) {
            const unsigned long long key = keys[i];
            const uint32_t sq = (uint32_t)(key & 0xffffffffull);
            int lo = 0, hi = nprobe;
            while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (eprefix[mid] <= sq) lo = mid; else hi = mid; }
            const uint32_t l = probe[q * nprobe + lo];
            out_ids[q * k + i] = ids[offs[l] + (sq - eprefix[lo])];
            out_d[q * k + i] = key_float((uint32_t)(key >> 32));
        } else {
            out_ids[q * k + i] = 0;
            out_d[q * k + i] = h > 0 ? key_float((uint32_t)(keys[h - 1] >> 32)) : 0.0f;
        }
    }
    if (threadIdx.x == 0 && out_n) out_n[q] = (uint32_t)h;
}

// ---------------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------------
namespace {
// One accumulator is 128 queries wide; with two of them 256 TMEM columns remain for the
// tile, so dims beyond 512 go to a shared-memory tile and the B ring shrinks.
template <int S, int N>
size_t tl_smem(int dim, int m) {
    const int kt = (512 - 2 * N) / 32, kc = dim / 64, ks = kc > kt ? kc - kt : 0;  // 32 TMEM columns per 64 dims
    return 1024 + (size_t)S * N * 128 + (size_t)ks * TL_M * 128 + (2 * S + 10) * 8 + 2 * N * 16 + 2 * N * 8 +
           2 * sizeof(UnitInfo) + 2 * (size_t)TL_M * m + 16;
}
// CTA-pair kernel: stages of N/2 query rows, four more unit-ring barriers.
template <int S>
size_t tl_smem2(int dim, int m) {
    constexpr int N = 128;
    const int kc = dim / 64, ks = kc > 8 ? kc - 8 : 0;
    return 1024 + (size_t)S * (N / 2) * 128 + (size_t)ks * TL_M * 128 + (2 * S + 14) * 8 + 2 * N * 16 + 2 * N * 8 +
           2 * sizeof(UnitInfo) + 2 * (size_t)TL_M * m + 16;
}
}  // namespace

bool tc_list_scan_supported(int dim, int m, int ksub) {
    const int dsub = m > 0 ? dim / m : 0;
    return ksub == 256 && dim % 64 == 0 && dim >= 64 && dim <= 768 && dim % m == 0 &&
           (dsub == 4 || dsub == 8 || dsub == 16) && scan_blocked_supported(m, ksub);
}

void launch_query_prep(const float* rq, long long nq, int dim, uint16_t* rqb, float* rqn, cudaStream_t st) {
    if (nq <= 0) return;
    const int blocks = (int)std::min<long long>((nq * 32 + 255) / 256, 148LL * 16);
    query_prep_kernel<<<blocks, 256, 0, st>>>(rq, nq, dim, reinterpret_cast<__nv_bfloat16*>(rqb), rqn);
    VGPU_LAUNCH("query_prep_kernel");
}

void TlWork::reserve(long long nq, int nprobe, int nlist, int dim, int k, int cap_, size_t n_vectors) {
    const long long np = nq * nprobe;
    // units <= (query groups per list) x (128-entry tiles over all lists)
    const size_t groups = (size_t)((nq + 128LL * TL_QG - 1) / (128LL * TL_QG));
    unit_list.reserve(groups * (n_vectors / TL_M + (size_t)nlist + 1));
    rqb.reserve((size_t)nq * dim);
    tau.reserve(nq);
    tau_x.reserve(nq);
    rqn.reserve(nq);
    cnt.reserve(nlist + 1);
    cursor.reserve(nlist + 1);
    seg_off.reserve(nlist + 1);
    units.reserve(nlist + 1);
    unit_off.reserve(nlist + 1);
    seg_meta.reserve((size_t)np * 4);
    p0.reserve(nq);
    pbase0.reserve(nq);
    mcount.reserve(nq + 1);
    mins_off.reserve(nq + 1);
    run_lut.reserve(nq);
    if (!host_u32) check(cudaMallocHost(&host_u32, sizeof(uint32_t)), "cudaMallocHost");
    qperm.reserve((size_t)np * dim);
    cand.reserve((size_t)nq * cap_);
    cand_cnt.reserve(nq);
    counter.reserve(1);
    stats.reserve(2);
    for (auto& e : ev)
        if (!e) check(cudaEventCreate(&e), "cudaEventCreate");
    p1_ids.reserve((size_t)nq * k);
    p1_d.reserve((size_t)nq * k);
    p1_n.reserve(nq);
    cap = cap_;
    size_t need = 0, need2 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, need, cnt.data(), seg_off.data(), nlist + 1);
    cub::DeviceScan::ExclusiveSum(nullptr, need2, mcount.data(), mins_off.data(), (int)(nq + 1));
    scan_tmp.reserve(std::max(need, need2) + 256);
}

namespace {
constexpr uint32_t kSmallHome = 8192;  // nearest lists up to this size get the blocked-scan threshold

// Group the pairs of probe [nq x np] (kSkipPair entries left out) by list with their
// epilogue metadata, build the unit table, and gather the list-ordered bf16 query rows.
void group_pairs(const TlScanArgs& a, TlWork& w, const uint32_t* probe, int np, const float* pbase,
                 cudaStream_t st) {
    constexpr int N = 128;
    const long long npairs = a.nq * np;
    check(cudaMemsetAsync(w.cnt.data(), 0, sizeof(uint32_t) * (a.nlist + 1), st), "memset");
    check(cudaMemsetAsync(w.cursor.data(), 0, sizeof(uint32_t) * (a.nlist + 1), st), "memset");
    const int gb = (int)std::min<long long>((npairs + 255) / 256, 148LL * 8);
    pair_hist_kernel<<<gb, 256, 0, st>>>(probe, npairs, w.cnt.data());
    VGPU_LAUNCH("pair_hist_kernel");
    size_t tmp = w.scan_tmp.size();
    check(cub::DeviceScan::ExclusiveSum(w.scan_tmp.data(), tmp, w.cnt.data(), w.seg_off.data(), a.nlist + 1, st),
          "cub::DeviceScan::ExclusiveSum(seg_off)");
    pair_scatter_kernel<<<gb, 256, 0, st>>>(probe, npairs, np, w.seg_off.data(), w.cursor.data(), pbase,
                                            w.tau.data(), w.rqn.data(), reinterpret_cast<uint4*>(w.seg_meta.data()));
    VGPU_LAUNCH("pair_scatter_kernel");
    unit_count_kernel<<<(a.nlist + 1 + 255) / 256, 256, 0, st>>>(w.cnt.data(), a.offs, a.nlist, N,
                                                                 TL_M * (w.pairs ? 2 : 1), w.units.data());
    VGPU_LAUNCH("unit_count_kernel");
    tmp = w.scan_tmp.size();
    check(cub::DeviceScan::ExclusiveSum(w.scan_tmp.data(), tmp, w.units.data(), w.unit_off.data(), a.nlist + 1, st),
          "cub::DeviceScan::ExclusiveSum(unit_off)");
    unit_fill_kernel<<<148 * 4, 256, 0, st>>>(w.unit_off.data(), a.nlist, w.unit_list.data());
    VGPU_LAUNCH("unit_fill_kernel");
    check(cudaMemsetAsync(w.counter.data(), 0, sizeof(uint32_t), st), "memset");
    qperm_kernel<<<148 * 16, 256, 0, st>>>(reinterpret_cast<const uint4*>(w.seg_meta.data()),
                                           w.seg_off.data() + a.nlist, reinterpret_cast<const uint4*>(w.rqb.data()),
                                           a.dim / 8, reinterpret_cast<uint4*>(w.qperm.data()));
    VGPU_LAUNCH("qperm_kernel");
}

// One launch of the screening kernel over the grouped pairs (mins != null: threshold pass).
void screen_pass(const TlScanArgs& a, TlWork& w, long long npairs, int np, float* mins, const uint32_t* mins_off,
                 cudaStream_t st) {
    constexpr int N = 128;
    const int dsub = a.dim / a.m;
    TlParams P;
    P.rqb = reinterpret_cast<const __nv_bfloat16*>(w.rqb.data()); P.rqn = w.rqn.data(); P.pbase = a.pbase;
    P.tau = w.tau.data();
    P.probe = a.probe; P.offs = a.offs; P.codes = a.codes; P.vterm = a.vterm; P.xnorm = a.xnorm;
    P.cbb = reinterpret_cast<const __nv_bfloat16*>(a.cbb);
    P.seg_off = w.seg_off.data(); P.seg_meta = reinterpret_cast<const uint4*>(w.seg_meta.data());
    P.unit_off = w.unit_off.data(); P.unit_list = w.unit_list.data();
    P.unit_counter = w.counter.data(); P.cand = w.cand.data(); P.cand_cnt = w.cand_cnt.data(); P.err = a.err;
    P.mins = mins; P.mins_off = mins_off;
    P.nlist = a.nlist; P.nprobe = np; P.dim = a.dim; P.m = a.m; P.k = a.k; P.cap = w.cap;
    int dev = 0, sms = 148;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
    if (w.pairs) {
        const CUtensorMap qmap2 = make_tile_map_bf16(w.qperm.data(), npairs, a.dim, N / 2);
#define VGPU_TL2(SV, DSV)                                                                                \
    do {                                                                                                 \
        const size_t smem = tl_smem2<SV>(a.dim, a.m);                                                    \
        if (smem > 227 * 1024) throw CudaError("tc_list_scan: shared-memory layout too large");          \
        check(cudaFuncSetAttribute(tc_list_scan2_kernel<N, SV, DSV>,                                     \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),             \
              "cudaFuncSetAttribute(tc_list_scan2)");                                                    \
        cudaLaunchConfig_t cfg = {};                                                                     \
        cfg.blockDim = dim3(TL_THREADS);                                                                 \
        cfg.dynamicSmemBytes = smem;                                                                     \
        cfg.stream = st;                                                                                 \
        cfg.gridDim = dim3(2 * (sms / 2));                                                               \
        int clusters = 0;                                                                                \
        check(cudaOccupancyMaxActiveClusters(&clusters, tc_list_scan2_kernel<N, SV, DSV>, &cfg),        \
              "cudaOccupancyMaxActiveClusters");                                                         \
        if (clusters < 1) throw CudaError("tc_list_scan: no CTA pair fits on an SM pair");               \
        tc_list_scan2_kernel<N, SV, DSV><<<2 * std::min(clusters, sms / 2), TL_THREADS, smem, st>>>(qmap2, P); \
    } while (0)
        if (a.dim > 512 && tl_smem2<16>(a.dim, a.m) > 227 * 1024) {
            if (dsub == 4) VGPU_TL2(12, 4); else if (dsub == 8) VGPU_TL2(12, 8); else VGPU_TL2(12, 16);
        } else if (a.dim > 512) {
            if (dsub == 4) VGPU_TL2(16, 4); else if (dsub == 8) VGPU_TL2(16, 8); else VGPU_TL2(16, 16);
        } else {
            if (dsub == 4) VGPU_TL2(16, 4); else if (dsub == 8) VGPU_TL2(16, 8); else VGPU_TL2(16, 16);
        }
#undef VGPU_TL2
        VGPU_LAUNCH("tc_list_scan2_kernel");
        return;
    }
    const CUtensorMap qmap = make_tile_map_bf16(w.qperm.data(), npairs, a.dim, N);
#define VGPU_TL(NV, SV, DSV)                                                                             \
    do {                                                                                                 \
        const size_t smem = tl_smem<SV, NV>(a.dim, a.m);                                                 \
        if (smem > 227 * 1024) throw CudaError("tc_list_scan: shared-memory layout too large");          \
        check(cudaFuncSetAttribute(tc_list_scan_kernel<NV, SV, DSV>,                                     \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),             \
              "cudaFuncSetAttribute(tc_list_scan)");                                                     \
        tc_list_scan_kernel<NV, SV, DSV><<<sms, TL_THREADS, smem, st>>>(qmap, P);                        \
    } while (0)
    if (a.dim > 512) {  // part of the tile in shared memory: 8 B stages
        if (dsub == 4) VGPU_TL(128, 8, 4); else if (dsub == 8) VGPU_TL(128, 8, 8); else VGPU_TL(128, 8, 16);
    } else {
        if (dsub == 4) VGPU_TL(128, 10, 4); else if (dsub == 8) VGPU_TL(128, 10, 8); else VGPU_TL(128, 10, 16);
    }
#undef VGPU_TL
    VGPU_LAUNCH("tc_list_scan_kernel");
}
}  // namespace

void launch_tc_list_scan(const TlScanArgs& a, TlWork& w, cudaStream_t st) {
    const long long npairs = a.nq * a.nprobe;
    if (a.nq <= 0 || npairs <= 0) return;
    if (!tc_list_scan_supported(a.dim, a.m, 256)) throw CudaError("tc_list_scan: unsupported shape");
    if (a.k > kMaxK) throw CudaError("tc_list_scan: k exceeds the supported maximum");
    if (npairs > 0xffffffffLL || a.nq > (1LL << 22) || a.nprobe > 1024)
        throw CudaError("tc_list_scan: batch too large (at most 2^22 queries and 1024 probes)");

    // VGPU_LIST_CTA=2 selects the CTA-pair screen (M = 256); default single CTAs (the
    // pair kernel halves the query bytes each SM streams but measures slower: its stage
    // recycling crosses the pair twice per stage).
    w.pairs = false;
    if (const char* v = std::getenv("VGPU_LIST_CTA")) w.pairs = std::string(v) == "2";
    check(cudaEventRecord(w.ev[0], st), "cudaEventRecord");
    launch_query_prep(a.rq, a.nq, a.dim, w.rqb.data(), w.rqn.data(), st);
    // Thresholds.  A query whose nearest list is long gets tau from a tensor-core pass
    // over that list: the k-th smallest of per-warp minima of the pairs' proven upper
    // bounds (k distinct entries, so an upper bound of its k-th FAST distance).  The
    // others take the k-th FAST distance over their nearest list (blocked scan).
    const int gq = (int)std::min<long long>((a.nq + 255) / 256, 148LL * 4);
    // VGPU_LIST_THRESHOLD=tc / lut forces one threshold source for every query.
    uint32_t small_max = kSmallHome;
    if (const char* v = std::getenv("VGPU_LIST_THRESHOLD")) {
        if (std::string(v) == "tc") small_max = 0;
        if (std::string(v) == "lut") small_max = 0xffffffffu;
    }
    const uint32_t shards = a.tau_fn ? std::max(a.tau_shards, 1u) : 1u;
    home_split_kernel<<<gq, 256, 0, st>>>(a.probe, a.nprobe, a.pbase, a.offs, a.nq, small_max, a.k <= 256 ? 1 : 0,
                                          a.tau_shard, shards, (uint64_t)4 * (uint64_t)a.k, w.p0.data(),
                                          w.pbase0.data(), w.mcount.data(),
                                          w.run_lut.data(), w.tau.data());
    VGPU_LAUNCH("home_split_kernel");
    size_t tmp = w.scan_tmp.size();
    check(cub::DeviceScan::ExclusiveSum(w.scan_tmp.data(), tmp, w.mcount.data(), w.mins_off.data(), (int)(a.nq + 1), st),
          "cub::DeviceScan::ExclusiveSum(mins_off)");
    check(cudaMemcpyAsync(w.host_u32, w.mins_off.data() + a.nq, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "d2h");
    // Any k entries of the nearest list bound the k-th distance; scanning a prefix of the
    // list trades a looser tau for a cheaper threshold pass (VGPU_LIST_HOME_BLOCKS caps it
    // in 128-entry blocks, at least enough blocks to hold k entries).
    uint32_t home_blocks = 0xffffffffu;
    if (const char* v = std::getenv("VGPU_LIST_HOME_BLOCKS"))
        home_blocks = std::max<uint32_t>((uint32_t)std::strtoul(v, nullptr, 10), (uint32_t)((a.k + 127) / 128));
    launch_scan_blocked_split(a.T, a.nq, a.pbase, a.probe, a.nprobe, 1, a.m, a.offs, a.blk_off, a.bcodes, a.bvterm,
                              a.ids, a.k, w.p1_ids.data(), w.p1_d.data(), w.p1_n.data(), w.run_lut.data(), 0u,
                              w.split, st, home_blocks);  // synchronizes the stream: host_u32 is ready
    const uint32_t n_mins = *w.host_u32;
    if (n_mins > 0) {
        w.mins.reserve(n_mins);
        group_pairs(a, w, w.p0.data(), 1, w.pbase0.data(), st);
        screen_pass(a, w, a.nq, 1, w.mins.data(), w.mins_off.data(), st);
        minima_select_kernel<<<(unsigned)a.nq, 256, 0, st>>>(w.mins.data(), w.mins_off.data(), w.mcount.data(), a.k,
                                                             w.tau.data());
        VGPU_LAUNCH("minima_select_kernel");
    }
    tau_merge_kernel<<<gq, 256, 0, st>>>(w.p1_d.data(), w.p1_n.data(), w.run_lut.data(), a.nq, a.k, w.cap,
                                         w.tau.data(), w.cand_cnt.data());
    VGPU_LAUNCH("tau_merge_kernel");
    if (a.tau_fn) {
        tau_export_kernel<<<gq, 256, 0, st>>>(w.tau.data(), a.nq, w.tau_x.data());
        VGPU_LAUNCH("tau_export_kernel");
        if (a.tau_fn(w.tau_x.data(), (size_t)a.nq, st, a.tau_user) != 0)
            throw CudaError("tc_list_scan: the threshold exchange failed");
        tau_import_kernel<<<gq, 256, 0, st>>>(w.tau_x.data(), a.nq, w.cap, w.tau.data(), w.cand_cnt.data());
        VGPU_LAUNCH("tau_import_kernel");
    }
    check(cudaEventRecord(w.ev[1], st), "cudaEventRecord");

    // Pairs grouped by list; units per list; list-ordered query rows.
    group_pairs(a, w, a.probe, a.nprobe, a.pbase, st);
    check(cudaEventRecord(w.ev[2], st), "cudaEventRecord");
    screen_pass(a, w, npairs, a.nprobe, nullptr, nullptr, st);
    check(cudaEventRecord(w.ev[3], st), "cudaEventRecord");

    // Refine the candidates; overflowed queries fall back to the blocked scan.
    // [barrier][table, then the sort keys][rotated query][probe prefixes] (tl_refine_kernel)
    if (next_pow2(w.cap) > 256 * 16) throw CudaError("tc_list_scan: candidate cap above 4096");
    if (a.cb == nullptr) throw CudaError("tc_list_scan: the fp32 codebooks are required");
    const size_t rsmem = 16 + std::max((size_t)a.m * 256 * 4, (size_t)next_pow2(w.cap) * 8) +
                         (size_t)((a.dim + 3) & ~3) * 4 + (size_t)(a.nprobe + 1) * 4;
    if (rsmem > 227 * 1024) throw CudaError("tc_list_scan: refine buffers do not fit in shared memory");
    uint32_t table_min = kRefineTableMin;
    if (const char* v = std::getenv("VGPU_REFINE_TABLE_MIN")) table_min = (uint32_t)std::strtoul(v, nullptr, 10);
#define VGPU_RF(MCV, GV, DSV)                                                                               \
    do {                                                                                                    \
        check(cudaFuncSetAttribute(tl_refine_kernel<MCV, GV, DSV>,                                          \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem),               \
              "cudaFuncSetAttribute(tl_refine)");                                                           \
        tl_refine_kernel<MCV, GV, DSV><<<(unsigned)a.nq, 256, rsmem, st>>>(                                 \
            a.T, a.rq, a.dim, a.cb, a.probe, a.nprobe, a.pbase, a.offs, a.codes, a.vterm, a.ids,            \
            w.cand.data(), w.cand_cnt.data(), w.cap, a.k, a.out_ids, a.out_d, a.out_n, a.err, table_min);  \
    } while (0)
    // (m, dsub) pairs of tc_list_scan_supported: dim = m dsub <= 768, a multiple of 64
    const int rdsub = a.dim / a.m;
    if (a.m == 16 && rdsub == 4) VGPU_RF(16, 16, 4);
    else if (a.m == 16 && rdsub == 8) VGPU_RF(16, 16, 8);
    else if (a.m == 16) VGPU_RF(16, 16, 16);
    else if (a.m == 32 && rdsub == 4) VGPU_RF(32, 32, 4);
    else if (a.m == 32 && rdsub == 8) VGPU_RF(32, 32, 8);
    else if (a.m == 32) VGPU_RF(32, 32, 16);
    else if (a.m == 64 && rdsub == 4) VGPU_RF(64, 32, 4);
    else if (a.m == 64 && rdsub == 8) VGPU_RF(64, 32, 8);
    else if (a.m == 96 && rdsub == 4) VGPU_RF(96, 32, 4);
    else if (a.m == 96 && rdsub == 8) VGPU_RF(96, 32, 8);
    else if (a.m == 128 && rdsub == 4) VGPU_RF(128, 32, 4);
    else throw CudaError("tc_list_scan: no refine kernel for this sub-quantizer shape");
#undef VGPU_RF
    VGPU_LAUNCH("tl_refine_kernel");
    check(cudaEventRecord(w.ev[4], st), "cudaEventRecord");
    launch_scan_blocked_split(a.T, a.nq, a.pbase, a.probe, a.nprobe, a.nprobe, a.m, a.offs, a.blk_off, a.bcodes,
                              a.bvterm, a.ids, a.k, a.out_ids, a.out_d, a.out_n, w.cand_cnt.data(), (uint32_t)w.cap,
                              w.split, st);
    check(cudaEventRecord(w.ev[5], st), "cudaEventRecord");
    cand_stats_kernel<<<(int)std::min<long long>((a.nq + 255) / 256, 148LL * 4), 256, 0, st>>>(
        w.cand_cnt.data(), a.nq, (uint32_t)w.cap, w.stats.data());
    VGPU_LAUNCH("cand_stats_kernel");
}

// ---------------------------------------------------------------------------------
// Per-index preparation: bf16 codebooks and per-entry decoded norms.
// ---------------------------------------------------------------------------------
__global__ void codebook_bf16_kernel(const float* __restrict__ cb, long long n, __nv_bfloat16* __restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __float2bfloat16_rn(cb[i]);
}

void launch_codebook_bf16(const float* cb, long long n, uint16_t* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 8);
    codebook_bf16_kernel<<<blocks, 256, 0, st>>>(cb, n, reinterpret_cast<__nv_bfloat16*>(out));
    VGPU_LAUNCH("codebook_bf16_kernel");
}

// xnorm[e] = ||xhat_e|| = sqrt(sum_s ||y_s,c_s||^2) (fp64 sum, rounded up slightly).
__global__ void entry_norm_kernel(const uint8_t* __restrict__ codes, long long n, const float* __restrict__ cb, int m,
                                  int dsub, float* __restrict__ xnorm) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        double s = 0.0;
        for (int j = 0; j < m; ++j) {
            const float* y = cb + ((long long)j * 256 + codes[e * m + j]) * dsub;
            for (int t = 0; t < dsub; ++t) s += (double)y[t] * y[t];
        }
        xnorm[e] = (float)(sqrt(s) * (1.0 + 1e-6));
    }
}

void launch_entry_norms(const uint8_t* codes, long long n, const float* cb, int m, int dsub, float* xnorm,
                        cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    entry_norm_kernel<<<blocks, 256, 0, st>>>(codes, n, cb, m, dsub, xnorm);
    VGPU_LAUNCH("entry_norm_kernel");
}

}  // namespace vgpu
