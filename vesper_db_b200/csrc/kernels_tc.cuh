// Tensor-core screening + exact refine for nearest-centroid search (tc_coarse.cu).
#pragma once

#include "common.cuh"

namespace vgpu {

// tcgen05 needs dim % 4 == 0 (16-byte TMA rows) and at least one 32-wide K tile.
bool tc_screen_supported(int dim);
// Dt[i][j] = ||x_i||^2 + ||c_j||^2 - 2 <x_i, c_j> with tf32 tensor-core products.
// err receives a nonzero code if a bounded wait timed out.
void launch_tc_screen(const float* x, long long nx, const float* c, int nc, int dim, const float* xn,
                      const float* cn, float* Dt, long long ldd, int* err, cudaStream_t st);
// out[i] = ||x_i||^2 (fp64 accumulation).
void launch_row_norms(const float* x, long long n, int dim, float* out, cudaStream_t st);
// Per row: exact k nearest centroids (reference-order distances, ties to the lowest
// index; `keep` applies Elkan's keep-on-tie rule to the nearest).  Dt from
// launch_tc_screen bounds which centroids need the exact recomputation.
void launch_screen_select(const float* Dt, long long n_rows, long long ldd, int nc, const float* x, int dim,
                          const float* cent, const float* xn, const float* cn, int k, const uint32_t* keep,
                          uint32_t* out_idx, float* out_val, int* err, cudaStream_t st);

}  // namespace vgpu
