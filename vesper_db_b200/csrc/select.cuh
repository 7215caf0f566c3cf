// Block-wide top-k selection in shared memory.
//
// Selects the k smallest entries of a float array under the total order
// (value, position): equal values are ordered by their position in the array, so a
// caller that lays candidates out in scan order gets "earlier candidate wins ties",
// and one that lays them out by index gets "smaller index wins" -- the tie rule of
// the reference's fused top-k (include/vesper/kernels/batch_distances.hpp:362-369)
// and of its coarse probe (partial_sort of (distance, list) pairs,
// src/index/ivf_pq.cpp:3449-3463).
//
// Method: 4-pass 8-bit radix select on order-preserving uint32 keys finds the k-th
// key T; every entry below T is taken; entries equal to T are taken in position
// order until k are chosen; the chosen (key, position) pairs are bitonic-sorted.
#pragma once

#include "common.cuh"

namespace vgpu {

struct SelectSmem {
    uint32_t hist[256];
    uint32_t scan_tmp[33];
    uint32_t counter;
    uint32_t thresh;
    uint32_t remaining;
};

// Bitonic sort of `p2` (power of two) uint64 keys in shared memory, ascending.
template <int NT>
__device__ void bitonic_sort_u64(unsigned long long* a, int p2) {
    for (int size = 2; size <= p2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < (p2 >> 1); i += NT) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = ((lo & size) == 0);
                const unsigned long long x = a[lo], y = a[hi];
                if ((x > y) == up) { a[lo] = y; a[hi] = x; }
            }
        }
    }
    __syncthreads();
}

__host__ __device__ inline int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Block-wide exclusive prefix of a per-thread flag, in thread order.  Returns this
// thread's rank among flagged threads; *total receives the block total.
template <int NT>
__device__ uint32_t block_rank(bool flag, uint32_t* warp_tmp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ballot = __ballot_sync(0xffffffffu, flag);
    const uint32_t in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_tmp[warp] = __popc(ballot);
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t run = 0;
        for (int w = 0; w < NT / 32; ++w) { const uint32_t c = warp_tmp[w]; warp_tmp[w] = run; run += c; }
        warp_tmp[32] = run;
    }
    __syncthreads();
    const uint32_t r = warp_tmp[warp] + in_warp;
    *total = warp_tmp[32];
    __syncthreads();
    return r;
}

// Select the k smallest of vals[0..n) by (value, position).  Writes the chosen
// (key << 32 | position) pairs, sorted ascending, to out[0..min(k,n)) and returns
// min(k, n).  `out` must hold next_pow2(min(k, n)) entries.  All threads of the
// block must call it; vals lives in shared or global memory.
template <int NT>
__device__ int block_select_k(const float* vals, int n, int k, unsigned long long* out,
                              SelectSmem& sm) {
    const int take = n < k ? n : k;
    if (take <= 0) return 0;
    const int p2 = next_pow2(take);
    if (n <= k) {
        for (int i = threadIdx.x; i < p2; i += NT)
            out[i] = i < n ? ((unsigned long long)float_key(vals[i]) << 32) | (uint32_t)i : ~0ull;
        bitonic_sort_u64<NT>(out, p2);
        return take;
    }
    // Radix select of the k-th smallest key.
    uint32_t prefix = 0, mask = 0;
    if (threadIdx.x == 0) sm.remaining = (uint32_t)k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) sm.hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += NT) {
            const uint32_t key = float_key(vals[i]);
            if ((key & mask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t rem = sm.remaining, acc = 0, b = 0;
            for (; b < 256; ++b) {
                const uint32_t h = sm.hist[b];
                if (acc + h >= rem) break;
                acc += h;
            }
            sm.remaining = rem - acc;
            sm.thresh = b;
        }
        __syncthreads();
        prefix |= sm.thresh << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t T = prefix;
    const uint32_t ties_needed = sm.remaining;       // entries equal to T to take
    const uint32_t n_less = (uint32_t)k - ties_needed;
    if (threadIdx.x == 0) sm.counter = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += NT) {
        const uint32_t key = float_key(vals[i]);
        if (key < T) {
            const uint32_t slot = atomicAdd(&sm.counter, 1u);
            out[slot] = ((unsigned long long)key << 32) | (uint32_t)i;
        }
    }
    __syncthreads();
    // Ties in position order.
    uint32_t taken = 0;
    for (int base = 0; base < n && taken < ties_needed; base += NT) {
        const int i = base + threadIdx.x;
        const bool tie = i < n && float_key(vals[i]) == T;
        uint32_t tot;
        const uint32_t r = block_rank<NT>(tie, sm.scan_tmp, &tot);
        if (tie && taken + r < ties_needed)
            out[n_less + taken + r] = ((unsigned long long)T << 32) | (uint32_t)i;
        taken += tot;
    }
    for (int i = take + threadIdx.x; i < p2; i += NT) out[i] = ~0ull;
    __syncthreads();
    bitonic_sort_u64<NT>(out, p2);
    return take;
}

// Per-probe prefix sums of one query's probed lists, run by one whole warp (a shuffle
// scan per 32 probes instead of one thread walking them): eprefix[t] = entries of
// probes 0..t-1, eprefix[nscan] = their total; the same for 128-entry blocks when
// bprefix is given.  Integer sums: the values equal a sequential walk's.
__device__ __forceinline__ void probe_prefixes_warp(const uint32_t* __restrict__ prow, int nscan,
                                                    const uint64_t* __restrict__ offs,
                                                    const uint64_t* __restrict__ blk_off, uint32_t* eprefix,
                                                    uint32_t* bprefix) {
    const int lane = threadIdx.x & 31;
    uint32_t ec = 0, bc = 0;
    for (int t0 = 0; t0 < nscan; t0 += 32) {
        const int t = t0 + lane;
        uint32_t e = 0, b = 0;
        if (t < nscan) {
            const uint32_t l = prow[t];
            e = (uint32_t)(offs[l + 1] - offs[l]);
            if (bprefix) b = (uint32_t)(blk_off[l + 1] - blk_off[l]);
        }
        uint32_t ie = e, ib = b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t ye = __shfl_up_sync(0xffffffffu, ie, o);
            const uint32_t yb = __shfl_up_sync(0xffffffffu, ib, o);
            if (lane >= o) { ie += ye; ib += yb; }
        }
        if (t < nscan) {
            eprefix[t] = ec + ie - e;
            if (bprefix) bprefix[t] = bc + ib - b;
        }
        ec += __shfl_sync(0xffffffffu, ie, 31);
        bc += __shfl_sync(0xffffffffu, ib, 31);
    }
    if (lane == 0) {
        eprefix[nscan] = ec;
        if (bprefix) bprefix[nscan] = bc;
    }
}

}  // namespace vgpu
