// Tensor-core (tcgen05, kind::tf32) screening of query-centroid distances, followed
// by an exact refine, for the coarse probe, add() assignment and the k-means E-step.
//
// Stage 1 (tc_screen_kernel): S = X * C^T on the 5th-generation tensor cores.  One CTA
// computes a 128 x 256 tile: a TMA producer thread streams 128x32 and 256x32 fp32 tiles
// (128-byte swizzle) through a 4-stage shared-memory ring, one thread issues
// tcgen05.mma.kind::tf32 (M=128, N=256, K=8) into a TMEM accumulator (256 columns),
// and the four warps read it back with tcgen05.ld and write
//     Dt = ||x||^2 + ||c||^2 - 2 S
// to global memory.  TF32 operands are truncated to 10 mantissa bits, so Dt is only a
// screen: |Dt - d_ref| <= eps(x, c) (bound below), with d_ref the reference-order
// distance of common.cuh.
//
// Stage 2 (screen_select_kernel): per row, U* = the k-th smallest upper bound
// Dt + eps; every centroid whose lower bound Dt - eps is <= U* is recomputed exactly
// (l2 in the reference's lane order) and the k smallest (exact distance, index) pairs
// are selected.  A centroid outside the band cannot be among the k nearest, so the
// result equals the exact top-k / arg-min (ties to the lowest index; with `keep`, the
// current assignment wins a tie, as in KmeansElkan::assign_with_bounds).
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code, stops
// issuing work, and still frees its TMEM before returning.
#include <cuda.h>
#include <cfloat>

#include "kernels.cuh"
#include "kernels_tc.cuh"
#include "select.cuh"
#include "tc_common.cuh"
#include "tc_screen.cuh"

namespace vgpu {
namespace {

constexpr int BM = 128, BN = 256, BK = 32, STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;            // 16 KB
constexpr int B_BYTES = BN * BK * 4;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLS = 256;

using tc::kSpinLimit;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_u32;
using tc::sw128_kmajor_desc;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) { tc::commit(bar); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    tc::tmem_ld32(taddr, r);
    tc::tmem_ld_wait();
}

}  // namespace

// MODE 0: Dt = ||x||^2 + ||c||^2 - 2S (L2 screen), 1: Dt = -2S (inner-product screen),
// 2 / 3: the same values are not stored; column c of row r is appended to the row's
// candidate list when its lower bound (value - eps) is <= tau[r] (flat top-k filter).
template <int MODE>
__global__ void __launch_bounds__(128, 1) tc_screen_kernel(const __grid_constant__ CUtensorMap map_x,
                                                           const __grid_constant__ CUtensorMap map_c, int nx,
                                                           int nc, int dim, const float* __restrict__ xn,
                                                           const float* __restrict__ cn, float* __restrict__ Dt,
                                                           long long ldd, int* __restrict__ err,
                                                           const float* __restrict__ tau,
                                                           uint2* __restrict__ cand, uint32_t* __restrict__ cand_cnt,
                                                           int cap, uint32_t col_off, int qfast,
                                                           const float* __restrict__ cs) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    __shared__ int s_fail;
    __shared__ float s_cn[BN], s_cs[BN];  // filter modes: the tile's column norms and their square roots

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // qfast: consecutive CTAs share a column tile (columns streamed from HBM once while
    // the row tiles stay in L2); otherwise they share a row tile.
    const int m0 = (qfast ? blockIdx.x : blockIdx.y) * BM, n0 = (qfast ? blockIdx.y : blockIdx.x) * BN;
    const int kt = (dim + BK - 1) / BK;

    if constexpr (MODE >= 2) {
        for (int j = threadIdx.x; j < BN; j += blockDim.x) {
            const int col = n0 + j;
            s_cn[j] = col < nc ? cn[col] : 0.0f;
            s_cs[j] = col < nc ? cs[col] : 0.0f;
        }
    }
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer.
        for (int t = 0; t < kt; ++t) {
            const int s = t % STAGES;
            if (t >= STAGES && !mbar_wait(&empty[s], ((t / STAGES) - 1) & 1)) { s_fail = 1; break; }
            unsigned char* a = smem + s * STAGE_BYTES;
            mbar_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(a, &map_x, t * BK, m0, &full[s]);
            tma_load_2d(a + A_BYTES, &map_c, t * BK, n0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        bool ok = true;
        for (int t = 0; t < kt && ok; ++t) {
            const int s = t % STAGES;
            if (!mbar_wait(&full[s], (t / STAGES) & 1)) { s_fail = 2; ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a = smem_u32(smem + s * STAGE_BYTES);
            const uint64_t ad = sw128_kmajor_desc(a), bd = sw128_kmajor_desc(a + A_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk)  // K = 8 tf32 = 32 bytes per MMA
                mma_tf32(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), (t > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&empty[s]);
        }
        mma_commit(accum);
    }
    __syncwarp();
    // Epilogue: thread (warp w, lane l) owns accumulator row 32w + l.
    const bool acc_ok = mbar_wait(accum, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!acc_ok) s_fail = 3;
    __syncthreads();
    if (s_fail == 0) {
        const int row = m0 + warp * 32 + lane;
        const float rn = (row < nx && xn != nullptr) ? xn[row] : 0.0f;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        if constexpr (MODE <= 1) {
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint32_t r[32];
                tmem_ld32(trow + (uint32_t)(ch * 32), r);
                if (row < nx) {
                    float* out = Dt + (long long)row * ldd + n0 + ch * 32;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int col = n0 + ch * 32 + j;
                        if (col < nc)
                            out[j] = MODE == 0 ? (rn + cn[col]) - 2.0f * __uint_as_float(r[j])
                                               : -2.0f * __uint_as_float(r[j]);
                    }
                }
            }
        } else {
            // Keep column c when value - eps <= tau (screen_eps / screen_eps_ip with
            // sqrt(xn * cn) taken as sqrt(xn) * sqrt(cn); the bounds' factor-2 margin
            // covers the extra rounding), rearranged so that no division or square root
            // runs per element.  Two passes over the accumulator: keep masks first, then
            // one slot reservation per row and the appends, so that each row waits for
            // one returning atomic per tile instead of one per kept column.
            const float t = row < nx ? tau[row] : -FLT_MAX;
            const float xs = sqrtf(rn);
            const float a = 1.953125e-3f + (float)(dim + 8) * 1.1920929e-7f;
            const float rr = (float)(dim / 8 + 8) * 1.1920929e-7f;
            // IP: keep iff S >= -t/2 - w sqrt(cn), w = 2 (a + rr + 2.4e-7) sqrt(xn) (+2^-10)
            const float w_ip = 2.0f * (a + rr + 2.4e-7f) * xs * 1.0009765625f;
            const float t_ip = -0.5f * t;
            auto screen_value = [&](float S, int cj) -> float {
                if constexpr (MODE == 2) return (rn + s_cn[cj]) - 2.0f * S;
                else return -2.0f * S;
            };
            auto keep_of = [&](float S, int cj) -> bool {
                if constexpr (MODE == 2) {
                    const float c2 = s_cn[cj];
                    const float xc = xs * s_cs[cj];
                    const float dt = (rn + c2) - 2.0f * S;
                    const float e = 4.0f * a * xc + 4.768e-7f * (rn + c2 + 2.0f * xc) + 2.0f * rr * fabsf(dt);
                    return dt - 1.0009765625f * e <= t;
                } else {
                    return S >= fmaf(-w_ip, s_cs[cj], t_ip);
                }
            };
            uint32_t mask[BN / 32];
            uint32_t total = 0;
#pragma unroll
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint32_t r[32];
                tmem_ld32(trow + (uint32_t)(ch * 32), r);
                uint32_t mk = 0;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int cj = ch * 32 + j;
                    if (keep_of(__uint_as_float(r[j]), cj) && n0 + cj < nc) mk |= 1u << j;
                }
                mask[ch] = row < nx ? mk : 0u;
                total += __popc(mask[ch]);
            }
            uint32_t slot = 0;
            if (total) slot = atomicAdd(&cand_cnt[row], total);
            uint2* dst = cand + (long long)row * cap;
#pragma unroll
            for (int ch = 0; ch < BN / 32; ++ch) {
                if (!__any_sync(0xffffffffu, mask[ch] != 0u)) continue;
                uint32_t r[32];
                tmem_ld32(trow + (uint32_t)(ch * 32), r);
                uint32_t mk = mask[ch];
                while (mk) {
                    const int j = __ffs(mk) - 1;
                    mk &= mk - 1u;
                    const int cj = ch * 32 + j;
                    if (slot < (uint32_t)cap) {
                        // r[] is indexed by a run-time j here; pick it with a small select
                        float S = 0.0f;
#pragma unroll
                        for (int u = 0; u < 32; ++u) S = (u == j) ? __uint_as_float(r[u]) : S;
                        dst[slot] = make_uint2((uint32_t)(n0 + cj) + col_off, __float_as_uint(screen_value(S, cj)));
                    }
                    ++slot;
                }
            }
        }
    } else if (threadIdx.x == 0) {
        atomicExch(err, s_fail);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ---------------------------------------------------------------------------------
// Host: tensor maps through the driver entry point (no libcuda link dependency).
// ---------------------------------------------------------------------------------
namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q), "cudaGetDriverEntryPoint");
        if (!p || q != cudaDriverEntryPointSuccess) throw CudaError("cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

CUtensorMap make_map(const float* base, long long rows, int dim, int box_rows, long long row_stride = 0) {
    CUtensorMap m;
    const cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)(row_stride ? row_stride : dim) * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim, gstride,
                                   box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed");
    return m;
}
}  // namespace

// Tile map over a bf16 matrix [rows x dim] (row stride dim * 2 bytes): boxes of 64
// columns x box_rows rows with 128-byte swizzle (K-major UMMA operand tiles).
CUtensorMap make_tile_map_bf16(const void* base, long long rows, int dim, int box_rows) {
    if (dim % 64 != 0) throw CudaError("tile map: dim must be a multiple of 64");
    CUtensorMap m;
    const cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
    const cuuint64_t gstride[1] = {(cuuint64_t)dim * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box,
                                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled (tile map) failed");
    return m;
}

bool tc_screen_supported(int dim) {
    return dim % 4 == 0 && dim >= 32;
}

namespace {
template <int MODE>
void tc_screen_launch(const float* x, long long nx, const float* c, long long nc, long long c_stride, int dim,
                      const float* xn, const float* cn, float* Dt, long long ldd, int* err, const float* tau,
                      uint2* cand, uint32_t* cand_cnt, int cap, uint32_t col_off, cudaStream_t st,
                      const float* cs = nullptr) {
    if (nx <= 0 || nc <= 0) return;
    if (!tc_screen_supported(dim)) throw CudaError("tc_screen: dim must be a multiple of 4 and >= 32");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(c)) & 15)
        throw CudaError("tc_screen: operands must be 16-byte aligned");
    if (nc > 0x7fffffffLL) throw CudaError("tc_screen: too many columns");
    const CUtensorMap mx = make_map(x, nx, dim, BM);
    const CUtensorMap mc = make_map(c, nc, dim, BN, c_stride);
    check(cudaFuncSetAttribute(tc_screen_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
          "cudaFuncSetAttribute(tc_screen)");
    // Columns larger than a quarter of L2 are streamed once, row tiles fastest.
    const long long row_bytes = (long long)dim * sizeof(float);
    const int qfast = (nc * row_bytes > (32LL << 20) && ceil_div(nc, BN) <= 65535) ? 1 : 0;
    if (!qfast && ceil_div(nx, BM) > 65535) throw CudaError("tc_screen: too many rows for one launch");
    dim3 grid = qfast ? dim3((unsigned)ceil_div(nx, BM), (unsigned)ceil_div(nc, BN))
                      : dim3((unsigned)ceil_div(nc, BN), (unsigned)ceil_div(nx, BM));
    tc_screen_kernel<MODE><<<grid, 128, SMEM_BYTES, st>>>(mx, mc, (int)nx, (int)nc, dim, xn, cn, Dt, ldd, err, tau,
                                                          cand, cand_cnt, cap, col_off, qfast, cs);
    VGPU_LAUNCH("tc_screen_kernel");
}
}  // namespace

void launch_tc_screen(const float* x, long long nx, const float* c, int nc, int dim, const float* xn, const float* cn,
                      float* Dt, long long ldd, int* err, cudaStream_t st) {
    tc_screen_launch<0>(x, nx, c, nc, 0, dim, xn, cn, Dt, ldd, err, nullptr, nullptr, nullptr, 0, 0, st);
}

void launch_tc_screen_op(bool ip, const float* x, long long nx, const float* c, long long nc, long long c_stride,
                         int dim, const float* xn, const float* cn, float* Dt, long long ldd, int* err,
                         cudaStream_t st) {
    if (ip)
        tc_screen_launch<1>(x, nx, c, nc, c_stride, dim, xn, cn, Dt, ldd, err, nullptr, nullptr, nullptr, 0, 0, st);
    else
        tc_screen_launch<0>(x, nx, c, nc, c_stride, dim, xn, cn, Dt, ldd, err, nullptr, nullptr, nullptr, 0, 0, st);
}

void launch_tc_filter(bool ip, const float* x, long long nx, const float* c, long long nc, long long c_stride,
                      int dim, const float* xn, const float* cn, const float* cs, const float* tau, uint32_t col_off,
                      uint2* cand, uint32_t* cand_cnt, int cap, int* err, cudaStream_t st) {
    if (ip)
        tc_screen_launch<3>(x, nx, c, nc, c_stride, dim, xn, cn, nullptr, 0, err, tau, cand, cand_cnt, cap, col_off,
                            st, cs);
    else
        tc_screen_launch<2>(x, nx, c, nc, c_stride, dim, xn, cn, nullptr, 0, err, tau, cand, cand_cnt, cap, col_off,
                            st, cs);
}

// ---------------------------------------------------------------------------------
// Fused nearest centroid (k = 1): tc_argmin_kernel.
// One persistent CTA per 128-row block walks every 256-column centroid tile:
//   warp 4 (one lane)  TMA producer of the 128x32 / 256x32 fp32 operand tiles (4-stage ring);
//   warp 5 (one lane)  tcgen05.mma.kind::tf32 into two 256-column TMEM accumulators, so
//                      the next tile's products run while the epilogue reads the last;
//   warps 0..3         epilogue, thread = row: for every column the screen value
//                      Dt = ||x||^2 - 2S' and its proven error eps (screen_eps), a
//                      running minimum U of the upper bounds Dt + eps,
//                      and the columns whose lower bound Dt - eps is <= U kept in a
//                      per-row list of ARG_CAP (compacted against the current U when it
//                      fills).
// Then each warp re-scores its rows' surviving columns exactly (reference lane order)
// and keeps the smallest (distance, index) -- the exact arg-min, ties to the lowest
// index, or, with `keep`, to the current assignment (KmeansElkan's rule).  No screen
// value ever reaches global memory.  A row whose list overflows is appended to `over`
// for the caller to redo.  Every wait is bounded; on timeout the kernel records an
// error code, stops, and frees its TMEM.
// ---------------------------------------------------------------------------------
// The augmented screen.  The tensor cores compute S' = <x, c> - ||c||^2 / 2 directly:
// the centroid operand carries one more 32-column K-slice holding (-hi, -lo, 0, ...),
// hi = tf32(||c||^2 / 2) and lo = tf32(||c||^2 / 2 - hi) (truncations, so both are
// exact tf32 values and hi + lo is within 2^-21 ||c||^2 of ||c||^2 / 2), and the row
// operand of that slice is a constant shared-memory tile of rows (1, 1, 0, ...).  One
// extra K = 8 MMA per tile; the epilogue's screen value is Dt = fl(||x||^2 - 2 S'), and
// a 32-column chunk is dismissed on fl(||x||^2 - 2 max S') alone (the rounding is
// monotone, so that is the chunk's smallest Dt): one max per column on the common path.
// screen_eps bounds the augmented value (screen_a, screen_r2).
// ---------------------------------------------------------------------------------
namespace {
constexpr int ARG_CAP = 16;
constexpr int ARG_THREADS = 192;
constexpr int ONES_OFF = STAGES * STAGE_BYTES;   // the augmented slice's row operand (A_BYTES)
constexpr int BAR_OFF = ONES_OFF + A_BYTES;      // barriers (256 bytes), then per-kernel arrays
constexpr int ARG_SMEM = BAR_OFF + 256 + ARG_CAP * BM * 8 + 1024;
constexpr int FILT_SMEM = BAR_OFF + 256 + 2 * BN * 4 + 1024;
static_assert(ARG_SMEM <= 232448 && FILT_SMEM <= 232448, "shared memory per CTA");

// Row r of the augmented slice's row operand, (1, 1, 0, ..., 0), in the 128-byte
// swizzled K-major layout a TMA tile load produces (16-byte chunk j of row r at chunk
// j ^ (r & 7)); then a proxy fence so the tensor cores see the generic-proxy stores.
__device__ __forceinline__ void write_ones_row(unsigned char* ones, int r) {
    uint4* row = reinterpret_cast<uint4*>(ones + r * 128);
#pragma unroll
    for (int j = 0; j < 8; ++j)
        row[j ^ (r & 7)] = j == 0 ? make_uint4(0x3f800000u, 0x3f800000u, 0u, 0u) : make_uint4(0u, 0u, 0u, 0u);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// AND of v over the 128 epilogue threads (warps 0..3, named barrier 1); also a barrier
// for them that publishes their earlier shared-memory writes.
__device__ __forceinline__ bool epilogue_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
constexpr uint32_t ARG_TMEM_COLS = 512;

// The two pipeline roles of the persistent screens (tc_argmin_kernel, tc_filter_kernel),
// each run by one lane.  Producer: the 128-row block at m0 with column tiles
// jt0 .. jt0 + ntiles - 1, K-slices in order, through the STAGES-deep ring.  MMA: tile t
// into TMEM accumulator t & 1 (256 columns each), after the epilogue has released the
// accumulator's previous tile.  A failed (bounded) wait sets *fail and ends the role.
__device__ __forceinline__ void screen_producer(unsigned char* smem, uint64_t* full, uint64_t* empty,
                                                const CUtensorMap* map_x, const CUtensorMap* map_c, int m0,
                                                int jt0, int ntiles, int kt, bool aug, volatile int* fail) {
    int it = 0;
    const int kslices = kt + (aug ? 1 : 0);
    for (int j = 0; j < ntiles && !*fail; ++j) {
        for (int t = 0; t < kslices; ++t, ++it) {
            const int s = it % STAGES;
            if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1)) { *fail = 1; return; }
            unsigned char* a = smem + s * STAGE_BYTES;
            if (t < kt) {
                mbar_expect_tx(&full[s], STAGE_BYTES);
                tma_load_2d(a, map_x, t * BK, m0, &full[s]);
            } else {
                mbar_expect_tx(&full[s], B_BYTES);   // the augmented slice: centroid side only
            }
            tma_load_2d(a + A_BYTES, map_c, t * BK, (jt0 + j) * BN, &full[s]);
        }
    }
}

__device__ __forceinline__ void screen_mma(unsigned char* smem, uint64_t* full, uint64_t* empty, uint64_t* acc_full,
                                           uint64_t* acc_empty, uint32_t tmem, int ntiles, int kt, bool aug,
                                           volatile int* fail) {
    int it = 0;
    const int kslices = kt + (aug ? 1 : 0);
    const uint64_t ones_desc = sw128_kmajor_desc(smem_u32(smem + ONES_OFF));
    for (int j = 0; j < ntiles && !*fail; ++j) {
        const int acc = j & 1;
        if (j >= 2 && !mbar_wait(&acc_empty[acc], ((j >> 1) - 1) & 1)) { *fail = 4; return; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t td = tmem + (uint32_t)(acc * BN);
        for (int t = 0; t < kslices; ++t, ++it) {
            const int s = it % STAGES;
            if (!mbar_wait(&full[s], (it / STAGES) & 1)) { *fail = 2; return; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a = smem_u32(smem + s * STAGE_BYTES);
            const uint64_t ad = sw128_kmajor_desc(a), bd = sw128_kmajor_desc(a + A_BYTES);
            if (t < kt) {
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk)
                    mma_tf32(td, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), (t > 0 || kk > 0) ? 1u : 0u);
            } else {
                mma_tf32(td, ones_desc, bd, 1u);   // only K columns 0 and 1 of the slice are nonzero
            }
            mma_commit(&empty[s]);
        }
        mma_commit(&acc_full[acc]);
    }
}
}  // namespace

__global__ void __launch_bounds__(ARG_THREADS, 1) tc_argmin_kernel(
    const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_c, int nx, int nc, int dim,
    const float* __restrict__ x, const float* __restrict__ cent, const float* __restrict__ xn,
    const float* __restrict__ cn, const float* __restrict__ cs, const float* __restrict__ cmax,
    const uint32_t* __restrict__ keep, uint32_t* __restrict__ out_idx, float* __restrict__ out_val,
    uint32_t* __restrict__ over, uint32_t* __restrict__ n_over, int* __restrict__ err) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;     // [2]
    uint64_t* acc_empty = acc_full + 2;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    // barriers in the first 256 bytes past the ring and the ones tile, then the
    // candidate lists (the last 1024 bytes of ARG_SMEM absorb the 1024-byte alignment)
    uint32_t* cand_col = reinterpret_cast<uint32_t*>(smem + BAR_OFF + 256);  // [ARG_CAP][BM]
    float* cand_lb = reinterpret_cast<float*>(cand_col + ARG_CAP * BM);      // [ARG_CAP][BM]
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM;
    const int kt = (dim + BK - 1) / BK;
    const int ntiles = (nc + BN - 1) / BN;

    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], 4); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ARG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp < 4) write_ones_row(smem + ONES_OFF, threadIdx.x);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0)
            screen_producer(smem, full, empty, &map_x, &map_c, m0, 0, ntiles, kt, true, (volatile int*)&s_fail);
    } else if (warp == 5) {
        if (lane == 0)
            screen_mma(smem, full, empty, acc_full, acc_empty, tmem, ntiles, kt, true, (volatile int*)&s_fail);
    } else {
        // Epilogue: thread (warp w < 4, lane l) owns row 32w + l.
        const int r = warp * 32 + lane;
        const int row = m0 + r;
        const bool live = row < nx;
        const float rn = live ? xn[row] : 0.0f;
        const float xs = sqrtf(rn);
        const float a = screen_a(dim), r2 = screen_r2(dim);
        const float rr = (float)(dim / 8 + 8) * 1.1920929e-7f;
        // e(col) <= E0 + 2.002 rr |dt| over every column (cmax = the largest ||c||^2 and
        // ||c||), so dt > T = (U + E0)(1 + 4 rr) proves dt - e > U: most columns are
        // dismissed on dt alone.  U >= 0 (an upper bound of an exact distance), so such
        // a dt is positive.
        const float c2max = cmax[0], csmax = cmax[1];
        const float E0 = 1.0009765625f * (4.0f * a * xs * csmax + 4.0f * r2 * c2max +
                                          4.768e-7f * (rn + c2max + 2.0f * xs * csmax));
        const float tgrow = 1.0f + 4.0f * rr + 1e-5f;   // + slack for the fp32 rounding of this test
        float U = FLT_MAX, T = FLT_MAX;
        int cnt = 0;
        bool overflow = false;
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        for (int j = 0; j < ntiles; ++j) {
            const int acc = j & 1;
            const int n0 = j * BN;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (j >> 1) & 1));
            if (!got) { s_fail = 3; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint32_t v[32];
                __syncwarp();   // reconverge after the divergent screen before the collective load
                tmem_ld32(trow + (uint32_t)(acc * BN + ch * 32), v);
                const int cb = n0 + ch * 32;
                if (cb >= nc) continue;   // uniform: the last tile's padding columns
                // Fast screen: the chunk's smallest screen value is fl(rn - 2 max S')
                // (monotone rounding); a chunk above T is dismissed, otherwise each
                // column passes when its screen value can reach T.
                float mx = -FLT_MAX;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) mx = fmaxf(mx, __uint_as_float(v[jj]));
                if (!live || !(__fmaf_rn(-2.0f, mx, rn) <= T)) continue;
                float dts[32];
                uint32_t mask = 0;
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) {
                    dts[jj] = __fmaf_rn(-2.0f, __uint_as_float(v[jj]), rn);
                    mask |= (dts[jj] <= T ? 1u : 0u) << jj;
                }
                if (nc - cb < 32) mask &= (1u << (nc - cb)) - 1u;   // columns past nc never pass
                if (!live) mask = 0;
                // Slow path for the (few) passing columns: the exact bound and the list.
                while (mask) {
                    const int jj = __ffs(mask) - 1;
                    mask &= mask - 1u;
                    const int col = cb + jj;
                    float dt = 0.0f;
#pragma unroll
                    for (int u = 0; u < 32; ++u) dt = (u == jj) ? dts[u] : dt;
                    const float c2 = __ldg(cn + col);
                    const float xc = xs * __ldg(cs + col);
                    const float e = 1.0009765625f * (4.0f * a * xc + 4.0f * r2 * c2 +
                                                     4.768e-7f * (rn + c2 + 2.0f * xc) + 2.0f * rr * fabsf(dt));
                    const float lb = dt - e;
                    if (lb > U) continue;
                    if (dt + e < U) {
                        U = dt + e;
                        T = (U + E0) * tgrow;
                    }
                    if (overflow) continue;
                    if (cnt == ARG_CAP) {
                        int w = 0;
                        for (int i = 0; i < ARG_CAP; ++i) {
                            const float l = cand_lb[i * BM + r];
                            if (l <= U) {
                                cand_lb[w * BM + r] = l;
                                cand_col[w * BM + r] = cand_col[i * BM + r];
                                ++w;
                            }
                        }
                        cnt = w;
                        if (cnt == ARG_CAP) { overflow = true; continue; }
                    }
                    cand_lb[cnt * BM + r] = lb;
                    cand_col[cnt * BM + r] = (uint32_t)col;
                    ++cnt;
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        // Exact refine, warp by warp: each of the warp's 32 rows in turn, four kept
        // columns at a time (eight lanes each, the reference's lane order).
        __syncwarp();
        const int ccnt = overflow ? 0 : cnt;
        const bool failed = __shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&s_fail), 0) != 0;
        const uint32_t kc = (live && keep) ? keep[row] : 0xffffffffu;
        for (int q = 0; q < 32; ++q) {
            const int rq = warp * 32 + q;
            const int rowq = m0 + rq;
            const int nq_c = __shfl_sync(0xffffffffu, ccnt, q);
            const float Uq = __shfl_sync(0xffffffffu, U, q);
            const bool ovq = __shfl_sync(0xffffffffu, (int)overflow, q) != 0;
            const uint32_t kcq = __shfl_sync(0xffffffffu, kc, q);
            if (rowq >= nx || failed) continue;
            if (ovq) {
                if (lane == 0) over[atomicAdd(n_over, 1u)] = (uint32_t)rowq;
                continue;
            }
            unsigned long long best = ~0ull;
            float keep_v = FLT_MAX;
            const float* xr = x + (long long)rowq * dim;
            for (int b = 0; b < nq_c; b += 4) {
                const int ci = b + (lane >> 3);
                const bool act = ci < nq_c && cand_lb[ci * BM + rq] <= Uq;
                const uint32_t col = act ? cand_col[ci * BM + rq] : 0u;
                const float vv = warp_l2_group(xr, cent + (long long)col * dim, dim, act);
                if (act && (lane & 7) == 0) {
                    const unsigned long long key = ((unsigned long long)float_key(vv) << 32) | col;
                    best = key < best ? key : best;
                    if (col == kcq) keep_v = vv;
                }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
                best = y < best ? y : best;
                keep_v = fminf(keep_v, __shfl_xor_sync(0xffffffffu, keep_v, o));
            }
            if (lane == 0) {
                uint32_t id = (uint32_t)(best & 0xffffffffull);
                const float v = key_float((uint32_t)(best >> 32));
                if (keep && kcq != id && keep_v == v) id = kcq;
                out_idx[rowq] = id;
                out_val[rowq] = v;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && s_fail) atomicExch(err, s_fail);
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ARG_TMEM_COLS) : "memory");
}

// ---------------------------------------------------------------------------------
// Persistent filter screen (flat top-k pass 2, the coarse probe's filter): the
// pipeline of tc_argmin_kernel over the column tiles [jt0, jt0 + tiles) of blockIdx.y's
// share, and the filter modes' keep rule: column c of row r is kept when its proven
// lower bound can reach tau[r] (L2: Dt - eps <= tau; IP: -2 S' - eps <= tau, i.e.
// S' >= -tau / 2 - w ||c||).  Kept columns are appended to the row's list (col +
// col_off, screen value), one atomic reservation per row per tile; a row's count may
// exceed cap (the refine treats that as an overflow).  Most columns are dismissed on a
// column-independent bound first (L2: Dt > (tau + E0)(1 + 4 rr + 1e-5); IP: S' below
// the threshold at the largest ||c||), the exact test runs only for the rest.  AUG (L2
// only): map_c is the augmented centroid operand and the screen value is ||x||^2 - 2 S';
// otherwise the tile's column norms are staged in shared memory.
// ---------------------------------------------------------------------------------
template <bool IP, bool AUG>
__global__ void __launch_bounds__(ARG_THREADS, 1) tc_filter_kernel(
    const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_c, int nx, int nc, int dim,
    int tiles_per_cta, const float* __restrict__ xn, const float* __restrict__ cn, const float* __restrict__ cs,
    const float* __restrict__ cmax, const float* __restrict__ tau, uint32_t col_off, uint2* __restrict__ cand,
    uint32_t* __restrict__ cand_cnt, int cap, int* __restrict__ err) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    float* c2s = reinterpret_cast<float*>(smem + BAR_OFF + 256);   // [2][BN] (L2 without AUG)
    __shared__ int s_fail;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM;
    const int kt = (dim + BK - 1) / BK;
    const int all_tiles = (nc + BN - 1) / BN;
    const int jt0 = blockIdx.y * tiles_per_cta;
    const int ntiles = max(0, min(tiles_per_cta, all_tiles - jt0));

    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int s2 = 0; s2 < STAGES; ++s2) { mbar_init(&full[s2], 1); mbar_init(&empty[s2], 1); }
        for (int a2 = 0; a2 < 2; ++a2) { mbar_init(&acc_full[a2], 1); mbar_init(&acc_empty[a2], 4); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ARG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (AUG && warp < 4) write_ones_row(smem + ONES_OFF, threadIdx.x);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0)
            screen_producer(smem, full, empty, &map_x, &map_c, m0, jt0, ntiles, kt, AUG, (volatile int*)&s_fail);
    } else if (warp == 5) {
        if (lane == 0)
            screen_mma(smem, full, empty, acc_full, acc_empty, tmem, ntiles, kt, AUG, (volatile int*)&s_fail);
    } else {
        const int r = warp * 32 + lane;
        const int row = m0 + r;
        const bool live = row < nx;
        const float rn = live ? xn[row] : 0.0f;
        const float xs = sqrtf(rn);
        const float t = live ? tau[row] : -FLT_MAX;
        const float a = screen_a(dim), r2 = screen_r2(dim);
        const float rr = (float)(dim / 8 + 8) * 1.1920929e-7f;
        const float c2max = cmax[0], csmax = cmax[1];
        // L2 fast bound (as in tc_argmin_kernel, with the fixed tau in place of U)
        const float E0 = 1.0009765625f * (4.0f * a * xs * csmax + 4.0f * r2 * c2max +
                                          4.768e-7f * (rn + c2max + 2.0f * xs * csmax));
        const float T = (t + E0) * (1.0f + 4.0f * rr + 1e-5f);
        // IP: keep iff S >= t_ip - w cs; below S_lo no column can be kept (w cs <= w csmax)
        const float w_ip = 2.0f * (a + rr + 2.4e-7f) * xs * 1.0009765625f;
        const float t_ip = -0.5f * t;
        const float S_lo = fmaf(-w_ip, csmax, t_ip);
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        for (int j = 0; j < ntiles; ++j) {
            const int acc = j & 1;
            const int n0 = (jt0 + j) * BN;
            float* c2t = c2s + acc * BN;
            if constexpr (!IP && !AUG)
                for (int i = r; i < BN; i += BM) c2t[i] = n0 + i < nc ? __ldg(cn + n0 + i) : FLT_MAX;
            const bool got = epilogue_all(mbar_wait(&acc_full[acc], (j >> 1) & 1));
            if (!got) { s_fail = 3; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t keepm[BN / 32];
            uint32_t total = 0;
#pragma unroll
            for (int ch = 0; ch < BN / 32; ++ch) {
                uint32_t v[32];
                __syncwarp();   // reconverge after the divergent screen before the collective load
                tmem_ld32(trow + (uint32_t)(acc * BN + ch * 32), v);
                keepm[ch] = 0u;
                const int cb = n0 + ch * 32;
                if (cb >= nc) continue;
                uint32_t mask = 0;
                if constexpr (IP) {
                    // dismiss the chunk when its largest dot product is below S_lo
                    float mx = -FLT_MAX;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) mx = fmaxf(mx, __uint_as_float(v[jj]));
                    if (!live || !(mx >= S_lo)) continue;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) mask |= (__uint_as_float(v[jj]) >= S_lo ? 1u : 0u) << jj;
                } else if constexpr (AUG) {
                    // the chunk's smallest screen value is fl(rn - 2 max S')
                    float mx = -FLT_MAX;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) mx = fmaxf(mx, __uint_as_float(v[jj]));
                    if (!live || !(__fmaf_rn(-2.0f, mx, rn) <= T)) continue;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        mask |= (__fmaf_rn(-2.0f, __uint_as_float(v[jj]), rn) <= T ? 1u : 0u) << jj;
                } else {
                    const float* cc = c2t + ch * 32;
                    float dts[32];
                    float mn = FLT_MAX;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) {
                        dts[jj] = __fmaf_rn(-2.0f, __uint_as_float(v[jj]), __fadd_rn(rn, cc[jj]));
                        mn = fminf(mn, dts[jj]);
                    }
                    if (!live || !(mn <= T)) continue;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) mask |= (dts[jj] <= T ? 1u : 0u) << jj;
                }
                if (nc - cb < 32) mask &= (1u << (nc - cb)) - 1u;
                if (!live) mask = 0;
                uint32_t km = 0;
                while (mask) {
                    const int jj = __ffs(mask) - 1;
                    mask &= mask - 1u;
                    const int col = cb + jj;
                    float S = 0.0f;
#pragma unroll
                    for (int u2 = 0; u2 < 32; ++u2) S = (u2 == jj) ? __uint_as_float(v[u2]) : S;
                    bool kp;
                    if constexpr (IP) {
                        kp = S >= fmaf(-w_ip, __ldg(cs + col), t_ip);
                    } else {
                        const float c2 = __ldg(cn + col);
                        const float xc = xs * __ldg(cs + col);
                        const float dt = AUG ? __fmaf_rn(-2.0f, S, rn) : (rn + c2) - 2.0f * S;
                        const float e = 4.0f * a * xc + 4.0f * r2 * c2 + 4.768e-7f * (rn + c2 + 2.0f * xc) +
                                        2.0f * rr * fabsf(dt);
                        kp = dt - 1.0009765625f * e <= t;
                    }
                    if (kp) km |= 1u << jj;
                }
                keepm[ch] = km;
                total += __popc(km);
            }
            uint32_t slot = 0;
            if (total) slot = atomicAdd(&cand_cnt[row], total);
            uint2* dst = cand + (long long)row * cap;
#pragma unroll
            for (int ch = 0; ch < BN / 32; ++ch) {
                if (!__any_sync(0xffffffffu, keepm[ch] != 0u)) continue;
                uint32_t v[32];
                tmem_ld32(trow + (uint32_t)(acc * BN + ch * 32), v);
                uint32_t km = keepm[ch];
                while (km) {
                    const int jj = __ffs(km) - 1;
                    km &= km - 1u;
                    const int col = n0 + ch * 32 + jj;
                    if (slot < (uint32_t)cap) {
                        float S = 0.0f;
#pragma unroll
                        for (int u2 = 0; u2 < 32; ++u2) S = (u2 == jj) ? __uint_as_float(v[u2]) : S;
                        const float val = IP    ? -2.0f * S
                                          : AUG ? __fmaf_rn(-2.0f, S, rn)
                                                : (rn + __ldg(cn + col)) - 2.0f * S;
                        dst[slot] = make_uint2((uint32_t)col + col_off, __float_as_uint(val));
                    }
                    ++slot;
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && s_fail) atomicExch(err, s_fail);
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ARG_TMEM_COLS) : "memory");
}

namespace {
// cmax[0] = max ||c||^2, cmax[1] = max ||c|| (non-negative floats order as their bits);
// cmax must be zeroed first.
__global__ void col_max_kernel(const float* __restrict__ cn, const float* __restrict__ cs, int nc,
                               float* __restrict__ cmax) {
    float a = 0.0f, b = 0.0f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nc; i += gridDim.x * blockDim.x) {
        a = fmaxf(a, cn[i]);
        b = fmaxf(b, cs[i]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(reinterpret_cast<unsigned int*>(cmax), __float_as_uint(a));
        atomicMax(reinterpret_cast<unsigned int*>(cmax + 1), __float_as_uint(b));
    }
}

// Row i of the augmented centroid operand: c_i (dim values, then zeros up to the next
// multiple of BK), then the slice (-hi, -lo, 0, ...) of ||c_i||^2 / 2.
__global__ void aug_cols_kernel(const float* __restrict__ c, long long nc, int dim, long long c_ld,
                                const float* __restrict__ cn, float* __restrict__ out, int ldo) {
    const int kd = ldo - BK;
    const long long total = nc * (long long)ldo;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / ldo;
        const int j = (int)(i - row * ldo);
        float v = 0.0f;
        if (j < dim) {
            v = c[row * c_ld + j];
        } else if (j == kd || j == kd + 1) {
            const float h = 0.5f * cn[row];
            const float hi = __uint_as_float(__float_as_uint(h) & 0xffffe000u);   // tf32 truncation
            const float lo = __uint_as_float(__float_as_uint(h - hi) & 0xffffe000u);
            v = j == kd ? -hi : -lo;
        }
        out[i] = v;
    }
}

__global__ void scatter_top1_kernel(const uint32_t* __restrict__ rows, int n, const uint32_t* __restrict__ idx,
                                    const float* __restrict__ val, uint32_t* __restrict__ out_idx,
                                    float* __restrict__ out_val) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        out_idx[rows[i]] = idx[i];
        out_val[rows[i]] = val[i];
    }
}
}  // namespace

bool tc_argmin_supported(int dim) { return tc_screen_supported(dim); }

int aug_ld(int dim) { return (dim + BK - 1) / BK * BK + BK; }

void launch_aug_cols(const float* c, long long nc, int dim, long long c_ld, const float* cn, float* out,
                     cudaStream_t st) {
    if (nc <= 0) return;
    const long long total = nc * (long long)aug_ld(dim);
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    aug_cols_kernel<<<blocks, 256, 0, st>>>(c, nc, dim, c_ld, cn, out, aug_ld(dim));
    VGPU_LAUNCH("aug_cols_kernel");
}

void launch_col_max(const float* cn, const float* cs, int nc, float* cmax, cudaStream_t st) {
    check(cudaMemsetAsync(cmax, 0, 2 * sizeof(float), st), "memset");
    if (nc <= 0) return;
    col_max_kernel<<<std::min(ceil_div(nc, 256), 148), 256, 0, st>>>(cn, cs, nc, cmax);
    VGPU_LAUNCH("col_max_kernel");
}

void launch_tc_argmin(const float* x, long long nx, const float* c, int nc, int dim, const float* xn, const float* cn,
                      const float* cs, const float* cmax, const uint32_t* keep, uint32_t* out_idx, float* out_val,
                      uint32_t* over, uint32_t* n_over, float* caug, int* err, cudaStream_t st) {
    if (nx <= 0 || nc <= 0) return;
    if (!tc_screen_supported(dim)) throw CudaError("tc_argmin: dim must be a multiple of 4 and >= 32");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(caug)) & 15)
        throw CudaError("tc_argmin: operands must be 16-byte aligned");
    if (nx > 0x7fffffffLL) throw CudaError("tc_argmin: too many rows");
    launch_aug_cols(c, nc, dim, dim, cn, caug, st);
    const CUtensorMap mx = make_map(x, nx, dim, BM);
    const CUtensorMap mc = make_map(caug, nc, aug_ld(dim), BN);
    check(cudaFuncSetAttribute(tc_argmin_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ARG_SMEM),
          "cudaFuncSetAttribute(tc_argmin)");
    tc_argmin_kernel<<<(unsigned)ceil_div(nx, BM), ARG_THREADS, ARG_SMEM, st>>>(
        mx, mc, (int)nx, nc, dim, x, c, xn, cn, cs, cmax, keep, out_idx, out_val, over, n_over, err);
    VGPU_LAUNCH("tc_argmin_kernel");
}

void launch_tc_filter_persistent(bool ip, const float* x, long long nx, const float* c, long long nc,
                                 long long c_stride, int dim, const float* xn, const float* cn, const float* cs,
                                 const float* cmax, const float* tau, uint32_t col_off, uint2* cand,
                                 uint32_t* cand_cnt, int cap, int* err, cudaStream_t st, const float* caug) {
    if (nx <= 0 || nc <= 0) return;
    if (!tc_screen_supported(dim)) throw CudaError("tc_filter: dim must be a multiple of 4 and >= 32");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(caug)) & 15)
        throw CudaError("tc_filter: operands must be 16-byte aligned");
    if (nc > 0x7fffffffLL || nx > 0x7fffffffLL) throw CudaError("tc_filter: too many rows or columns");
    const bool aug = !ip && caug;
    const CUtensorMap mx = make_map(x, nx, dim, BM);
    const CUtensorMap mc = aug ? make_map(caug, nc, aug_ld(dim), BN) : make_map(c, nc, dim, BN, c_stride);
    const long long row_blocks = ceil_div(nx, BM);
    const long long col_tiles = ceil_div(nc, BN);
    // Column shares: enough CTAs for a few waves of the SMs, at least 8 tiles per CTA so
    // that the pipeline's fill and drain stay small next to its steady state.
    long long splits = std::max<long long>(1, (148LL * 4 + row_blocks - 1) / row_blocks);
    splits = std::min(splits, std::max<long long>(1, col_tiles / 8));
    splits = std::min<long long>(splits, 65535);
    const int per = (int)((col_tiles + splits - 1) / splits);
    splits = (col_tiles + per - 1) / per;
    if (row_blocks > 0x7fffffffLL) throw CudaError("tc_filter: too many row blocks");
    dim3 grid((unsigned)row_blocks, (unsigned)splits);
#define VGPU_FILTER_LAUNCH(IPV, AUGV)                                                                            \
    do {                                                                                                         \
        check(cudaFuncSetAttribute(tc_filter_kernel<IPV, AUGV>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                   FILT_SMEM),                                                                   \
              "cudaFuncSetAttribute(tc_filter)");                                                                \
        tc_filter_kernel<IPV, AUGV><<<grid, ARG_THREADS, FILT_SMEM, st>>>(mx, mc, (int)nx, (int)nc, dim, per, xn, \
                                                                         cn, cs, cmax, tau, col_off, cand,       \
                                                                         cand_cnt, cap, err);                    \
    } while (0)
    if (ip) VGPU_FILTER_LAUNCH(true, false);
    else if (aug) VGPU_FILTER_LAUNCH(false, true);
    else VGPU_FILTER_LAUNCH(false, false);
#undef VGPU_FILTER_LAUNCH
    VGPU_LAUNCH("tc_filter_kernel");
}

void launch_scatter_top1(const uint32_t* rows, int n, const uint32_t* idx, const float* val, uint32_t* out_idx,
                         float* out_val, cudaStream_t st) {
    if (n <= 0) return;
    scatter_top1_kernel<<<std::min(ceil_div(n, 256), 148 * 8), 256, 0, st>>>(rows, n, idx, val, out_idx, out_val);
    VGPU_LAUNCH("scatter_top1_kernel");
}

__global__ void sqrt_kernel(const float* __restrict__ in, long long n, float* __restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = sqrtf(in[i]);
}

// ---------------------------------------------------------------------------------
// OPQ rotation of a query batch as one tensor-core GEMM (3xTF32).
//
// out = X W^T (W = R^T: the x R of apply_rotation) with every fp32 operand split as
// v = hi(v) + lo(v): hi(v) = v rounded to tf32 (10 mantissa bits, exact in a tf32
// operand), lo(v) = v - hi(v) (exact in fp32, |lo| <= 2^-11 |v|).
// X W^T ~= hi(X) hi(W)^T + hi(X) lo(W)^T + lo(X) hi(W)^T is one K = 3 dim contraction of
// X3 = [hi(X) | hi(X) | lo(X)] with W3 = [hi(W) | lo(W) | hi(W)] on tc_screen_kernel
// (MODE 1 stores -2 S, so W3 carries a factor -1/2, which is exact).
// Per term the error is about 2^-20 |x| |r| (the dropped lo lo product and the tf32
// rounding of lo), against 2^-24 for an fp32 product, so the rotated query differs from
// the sequential fp32 rotation by a few 1e-7 relative: well inside the 1e-4 relative
// distance tolerance of FAST search, which is the only path that uses it.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float tf32_hi(float v) {
    const uint32_t b = __float_as_uint(v);
    const float r = __uint_as_float((b + 0x1000u) & 0xffffe000u);  // round half away from zero on the magnitude
    return isfinite(r) ? r : __uint_as_float(b & 0xffffe000u);
}

// order 0: [hi | hi | lo] (the row operand), 1: scale [hi | lo | hi] (the rotation).
__global__ void tf32_split3_kernel(const float* __restrict__ x, long long n, int dim, int order, float scale,
                                   float* __restrict__ out) {
    const long long total = n * dim;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long row = e / dim;
        const int c = (int)(e - row * dim);
        const float v = x[e];
        const float hi = tf32_hi(v), lo = v - hi;
        float* o = out + row * 3 * dim + c;
        if (order == 0) {
            o[0] = hi; o[dim] = hi; o[2 * dim] = lo;
        } else {
            o[0] = scale * hi; o[dim] = scale * lo; o[2 * dim] = scale * hi;
        }
    }
}

bool rotate_3xtf32_supported(int dim) { return tc_screen_supported(3 * dim) && dim >= 32; }

void prepare_rotation_3xtf32(const float* W, int dim, float* W3, cudaStream_t st) {
    const long long total = (long long)dim * dim;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    tf32_split3_kernel<<<blocks, 256, 0, st>>>(W, dim, dim, 1, -0.5f, W3);
    VGPU_LAUNCH("tf32_split3_kernel");
}

void launch_rotate_3xtf32(const float* x, long long n, int dim, const float* R3, float* x3, float* out, int* err,
                          cudaStream_t st) {
    if (n <= 0) return;
    if (!rotate_3xtf32_supported(dim)) throw CudaError("rotate_3xtf32: unsupported dimension");
    const long long total = n * dim;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    tf32_split3_kernel<<<blocks, 256, 0, st>>>(x, n, dim, 0, 1.0f, x3);
    VGPU_LAUNCH("tf32_split3_kernel");
    tc_screen_launch<1>(x3, n, R3, dim, 0, 3 * dim, nullptr, nullptr, out, dim, err, nullptr, nullptr, nullptr, 0, 0,
                        st);
}

void launch_sqrt(const float* in, long long n, float* out, cudaStream_t st) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    sqrt_kernel<<<blocks, 256, 0, st>>>(in, n, out);
    VGPU_LAUNCH("sqrt_kernel");
}

// ---------------------------------------------------------------------------------
// Row norms (fp64 accumulate, one rounding) for the screen.
// ---------------------------------------------------------------------------------
__global__ void row_norms_kernel(const float* __restrict__ x, long long n, int dim, long long ld,
                                 float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long i = warp; i < n; i += nw) {
        double s = 0.0;
        for (int d = lane; d < dim; d += 32) { const double v = x[i * ld + d]; s += v * v; }
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) out[i] = (float)s;
    }
}

void launch_row_norms(const float* x, long long n, int dim, float* out, cudaStream_t st, long long ld) {
    if (n <= 0) return;
    const int blocks = (int)std::min<long long>((n * 32 + 255) / 256, 148LL * 32);
    row_norms_kernel<<<blocks, 256, 0, st>>>(x, n, dim, ld > 0 ? ld : dim, out);
    VGPU_LAUNCH("row_norms_kernel");
}

// ---------------------------------------------------------------------------------
// Stage 2: band selection, exact refine, top-k.
// ---------------------------------------------------------------------------------
namespace {
constexpr int SS_NT = 256;
constexpr int SS_CAP = 1024;   // columns per candidate chunk (at most this many candidates)
constexpr int SS_SMEM_KEYS = 16384;  // rows up to this width keep their upper-bound keys in shared memory

struct ScreenSmem {
    unsigned long long keys[4096];   // (exact key << 32 | index): carried winners + a chunk's candidates
    uint32_t cidx[SS_CAP];           // the chunk's candidate indices (in arrival order)
    uint32_t hist[256];
    uint32_t remaining, thresh, count;
    float keep_val;
};
}  // namespace

// IP: Dt holds -2 S (inner-product screen); the exact score is the reference-order
// inner product, larger first (ties to the lower index); out_val receives it.
// Column c of the screen is row c * cent_ld of cent.
template <bool IP>
__global__ void __launch_bounds__(SS_NT) screen_select_kernel(
    const float* __restrict__ Dt, long long ldd, int nc, const float* __restrict__ x, int dim,
    const float* __restrict__ cent, long long cent_ld, const float* __restrict__ xn, const float* __restrict__ cn,
    int k, const uint32_t* __restrict__ keep, uint32_t* __restrict__ out_idx, float* __restrict__ out_val, int* err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ScreenSmem& S = *reinterpret_cast<ScreenSmem*>(smem_raw);
    const long long row = blockIdx.x;
    const float* drow = Dt + row * ldd;
    const float* xr = x + row * dim;
    const float rn = xn[row];
    const int kk = k < nc ? k : nc;
    const uint32_t kc = keep ? keep[row] : 0xffffffffu;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) S.keep_val = FLT_MAX;
    (void)err;
    // Upper-bound keys computed once into shared memory when the row fits.
    uint32_t* ukeys = reinterpret_cast<uint32_t*>(smem_raw + sizeof(ScreenSmem));
    const bool cached = nc <= SS_SMEM_KEYS;
    float eps_max = 0.0f;
    if (cached) {
        // 8 columns per thread in flight at a time
        for (int c0 = threadIdx.x; c0 < nc; c0 += 8 * SS_NT) {
            float dt[8], cv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * SS_NT;
                dt[u] = c < nc ? drow[c] : 0.0f;
                cv[u] = c < nc ? cn[c] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * SS_NT;
                if (c < nc) {
                    const float e = IP ? screen_eps_ip(rn, cv[u], dim) : screen_eps(rn, cv[u], dt[u], dim);
                    ukeys[c] = float_key(dt[u] + e);
                    eps_max = fmaxf(eps_max, e);
                }
            }
        }
        for (int o = 16; o > 0; o >>= 1) eps_max = fmaxf(eps_max, __shfl_xor_sync(0xffffffffu, eps_max, o));
        if (lane == 0) S.hist[warp] = __float_as_uint(eps_max);
        __syncthreads();
        eps_max = 0.0f;
        for (int w = 0; w < SS_NT / 32; ++w) eps_max = fmaxf(eps_max, __uint_as_float(S.hist[w]));
        __syncthreads();
    }

    // 1) U* = kk-th smallest upper bound (4-pass radix select on order-preserving keys;
    //    histogram updates aggregated per warp, since the keys of one row share most
    //    of their leading bits).
    uint32_t prefix = 0, mask = 0;
    if (threadIdx.x == 0) S.remaining = (uint32_t)kk;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += SS_NT) S.hist[i] = 0;
        __syncthreads();
        for (int c0 = 0; c0 < nc; c0 += SS_NT) {
            const int c = c0 + threadIdx.x;
            uint32_t key = 0;
            bool part = false;
            if (c < nc) {
                if (cached) {
                    key = ukeys[c];
                } else {
                    const float dt = drow[c];
                    key = float_key(dt + (IP ? screen_eps_ip(rn, cn[c], dim) : screen_eps(rn, cn[c], dt, dim)));
                }
                part = (key & mask) == prefix;
            }
            // lanes sharing the first participating lane's bin add once, the rest alone
            const unsigned act = __ballot_sync(0xffffffffu, part);
            if (act) {
                const uint32_t bin = (key >> shift) & 255u;
                const uint32_t bin0 = __shfl_sync(0xffffffffu, bin, __ffs(act) - 1);
                const unsigned same = __ballot_sync(0xffffffffu, part && bin == bin0);
                if (lane == __ffs(act) - 1) atomicAdd(&S.hist[bin0], (uint32_t)__popc(same));
                if (part && bin != bin0) atomicAdd(&S.hist[bin], 1u);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t rem = S.remaining, acc = 0, b = 0;
            for (; b < 256; ++b) { const uint32_t h = S.hist[b]; if (acc + h >= rem) break; acc += h; }
            S.remaining = rem - acc;
            S.thresh = b;
        }
        __syncthreads();
        prefix |= S.thresh << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    const float ustar = key_float(prefix);
    // With cached keys, a column can only be a candidate (lower bound <= U*) if its
    // upper bound is <= U* + 2 max eps (+ a rounding margin).
    const uint32_t ukey_cut = float_key(ustar + 2.0f * eps_max + fabsf(ustar) * 1e-6f + 1e-30f);

    // 2) Column chunks of SS_CAP: candidates (lower bound <= U*) refined exactly, then
    //    the kk smallest (exact distance, index) of carried winners + candidates.
    // With cached keys, count the candidate superset first: when it fits, one chunk
    // spans the whole row.
    int chunk = SS_CAP;
    if (cached) {
        if (threadIdx.x == 0) S.count = 0;
        __syncthreads();
        uint32_t mine = 0;
        for (int c = threadIdx.x; c < nc; c += SS_NT) mine += ukeys[c] <= ukey_cut ? 1u : 0u;
        for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
        if (lane == 0 && mine) atomicAdd(&S.count, mine);
        __syncthreads();
        if (S.count <= (uint32_t)SS_CAP) chunk = nc;
        __syncthreads();
    }
    int carry = 0;
    for (int cb = 0; cb < nc; cb += chunk) {
        const int ce = min(nc, cb + chunk);
        if (threadIdx.x == 0) S.count = 0;
        __syncthreads();
        for (int c0 = cb; c0 < ce; c0 += SS_NT) {
            const int c = c0 + threadIdx.x;
            bool cand = false;
            if (c < ce && (!cached || ukeys[c] <= ukey_cut)) {
                const float dt = drow[c];
                cand = (dt - (IP ? screen_eps_ip(rn, cn[c], dim) : screen_eps(rn, cn[c], dt, dim))) <= ustar;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, cand);
            if (bal) {
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(&S.count, (uint32_t)__popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (cand) S.cidx[base + __popc(bal & ((1u << lane) - 1u))] = (uint32_t)c;
            }
        }
        __syncthreads();
        const int nnew = (int)S.count;
        // exact distances, 4 candidates per warp per step
        for (int b0 = warp * 4; b0 < nnew; b0 += (SS_NT / 32) * 4) {
            const int ci = b0 + (lane >> 3);
            const bool act = ci < nnew;
            const uint32_t c = act ? S.cidx[ci] : 0u;
            const float* crow = cent + (long long)c * cent_ld;
            const float v = IP ? warp_ip_group(xr, crow, dim, act) : warp_l2_group(xr, crow, dim, act);
            if (act && (lane & 7) == 0) {
                // inner products order by -v (zero canonicalised so -0 and +0 tie)
                const float ordv = IP ? (v == 0.0f ? 0.0f : -v) : v;
                S.keys[carry + ci] = ((unsigned long long)float_key(ordv) << 32) | c;
                if (c == kc) S.keep_val = v;
            }
        }
        const int total = carry + nnew;
        const int p2 = next_pow2(total < 2 ? 2 : total);
        __syncthreads();
        for (int i = total + threadIdx.x; i < p2; i += SS_NT) S.keys[i] = ~0ull;
        bitonic_sort_u64<SS_NT>(S.keys, p2);
        carry = total < kk ? total : kk;
    }
    // 3) Output in (exact distance, index) order; with `keep`, a tie with the current
    //    assignment keeps it.
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += SS_NT) {
        uint32_t id = 0u;
        float v = FLT_MAX;
        if (i < carry) {
            id = (uint32_t)(S.keys[i] & 0xffffffffull);
            v = key_float((uint32_t)(S.keys[i] >> 32));
            if (IP) v = v == 0.0f ? 0.0f : -v;
            if (i == 0 && keep && S.keep_val == v) id = kc;
        } else if (IP) {
            v = -FLT_MAX;
        }
        out_idx[row * k + i] = id;
        if (out_val) out_val[row * k + i] = v;
    }
}

namespace {
template <bool IP>
void screen_select_launch(const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                          const float* cent, long long cent_ld, const float* xn, const float* cn, int k,
                          const uint32_t* keep, uint32_t* out_idx, float* out_val, int* err, cudaStream_t st) {
    if (n_rows <= 0) return;
    if (k > kMaxK) throw CudaError("screen_select: k exceeds the supported maximum");
    const size_t smem = sizeof(ScreenSmem) + (nc <= SS_SMEM_KEYS ? (size_t)nc * sizeof(uint32_t) : 0);
    check(cudaFuncSetAttribute(screen_select_kernel<IP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute(screen_select)");
    screen_select_kernel<IP><<<(unsigned)n_rows, SS_NT, smem, st>>>(Dt, ldd, nc, x, dim, cent, cent_ld, xn, cn, k,
                                                                    keep, out_idx, out_val, err);
    VGPU_LAUNCH("screen_select_kernel");
}
}  // namespace

void launch_screen_select(const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                          const float* cent, const float* xn, const float* cn, int k, const uint32_t* keep,
                          uint32_t* out_idx, float* out_val, int* err, cudaStream_t st) {
    screen_select_launch<false>(Dt, n_rows, ldd, nc, x, dim, cent, dim, xn, cn, k, keep, out_idx, out_val, err, st);
}

void launch_screen_select_op(bool ip, const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                             const float* cent, long long cent_ld, const float* xn, const float* cn, int k,
                             uint32_t* out_idx, float* out_val, int* err, cudaStream_t st) {
    if (ip) screen_select_launch<true>(Dt, n_rows, ldd, nc, x, dim, cent, cent_ld, xn, cn, k, nullptr, out_idx,
                                       out_val, err, st);
    else screen_select_launch<false>(Dt, n_rows, ldd, nc, x, dim, cent, cent_ld, xn, cn, k, nullptr, out_idx,
                                     out_val, err, st);
}

}  // namespace vgpu
