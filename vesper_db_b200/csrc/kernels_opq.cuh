// fp64 helpers for OPQ training (definitions in opq_kernels.cu).
#pragma once

#include "common.cuh"

namespace vgpu {

// C = sum_i (a_i - ma)(b_i - mb)^T over n rows of d floats (fp64 accumulate);
// ma / mb may be null.
void launch_cross_fp64(const float* A, const float* B, long long n, int d, const double* ma,
                       const double* mb, double* C, cudaStream_t st);
// C[j][k] = sum_i A[i][j] * B[i][k] with every product and sum rounded separately, in
// row order (no fused multiply-add): the Procrustes matrix as the reference forms it.
void launch_cross_fp64_unfused(const float* A, const float* B, long long n, int d, double* C, cudaStream_t st);
void launch_col_mean(const float* X, long long n, int d, double* mean, cudaStream_t st);
// C = alpha * op(A) op(B) + beta * C, square d x d row-major; ta/tb transpose flags.
void launch_dgemm(const double* A, const double* B, double* C, int d, int ta, int tb, double alpha,
                  double beta, cudaStream_t st);
void launch_daxpby(double* y, const double* x, long long n, double a, double b, cudaStream_t st);
// Power iteration with deflation for all d eigenvectors of the symmetric C (rows of E).
// work must hold 3*d + 2 doubles.
void power_iteration_pca(const double* C, int d, int max_iters, double tol, double* E,
                         double* work, cudaStream_t st);

}  // namespace vgpu
