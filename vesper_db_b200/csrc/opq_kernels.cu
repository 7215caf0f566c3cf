// fp64 kernels for OPQ training on the GPU.
//
// learn_opq_rotation (src/index/ivf_pq.cpp:2769-2945): mean and covariance of the
// residual sample in fp64, then one power iteration per eigenvector with deflation
// against the previous ones; the eigenvectors become the rows of R.
// The OPQ alternation (:2540-2721) updates R by orthogonal Procrustes on
// C = X^T Y / n; the reference takes R = U V^T from a one-sided Jacobi SVD of C, which
// is the orthogonal polar factor of C.  Here the polar factor is computed by the
// Newton-Schulz iteration X <- 1.5 X - 0.5 X X^T X (fp64 GEMMs), which converges to
// the same matrix.
#include "kernels_opq.cuh"

namespace vgpu {

// C[j][k] += sum_i (a_i[j] - ma[j]) * (b_i[k] - mb[k]) over rows [0, n), fp64.
// 32x32 output tile per CTA, rows staged 32 at a time.  ma/mb may be null (no centring).
template <bool UNFUSED>
__global__ void __launch_bounds__(256) cross_fp64_kernel(const float* __restrict__ A,
                                                         const float* __restrict__ B, long long n,
                                                         int d, const double* __restrict__ ma,
                                                         const double* __restrict__ mb,
                                                         double* __restrict__ C) {
    __shared__ double As[32][33];
    __shared__ double Bs[32][33];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 2x2 outputs each
    const int j0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    double acc[2][2] = {{0, 0}, {0, 0}};
    for (long long r0 = 0; r0 < n; r0 += 32) {
        for (int e = threadIdx.x; e < 32 * 32; e += 256) {
            const int r = e / 32, c = e % 32;
            const long long g = r0 + r;
            double av = 0.0, bv = 0.0;
            if (g < n) {
                if (j0 + c < d) av = (double)A[g * d + j0 + c] - (ma ? ma[j0 + c] : 0.0);
                if (k0 + c < d) bv = (double)B[g * d + k0 + c] - (mb ? mb[k0 + c] : 0.0);
            }
            As[r][c] = av;
            Bs[r][c] = bv;
        }
        __syncthreads();
        for (int r = 0; r < 32; ++r) {
            const double a0 = As[r][ty * 2], a1 = As[r][ty * 2 + 1];
            const double b0 = Bs[r][tx * 2], b1 = Bs[r][tx * 2 + 1];
            if constexpr (UNFUSED) {   // rounded product, then rounded sum
                acc[0][0] = __dadd_rn(acc[0][0], __dmul_rn(a0, b0));
                acc[0][1] = __dadd_rn(acc[0][1], __dmul_rn(a0, b1));
                acc[1][0] = __dadd_rn(acc[1][0], __dmul_rn(a1, b0));
                acc[1][1] = __dadd_rn(acc[1][1], __dmul_rn(a1, b1));
            } else {
                acc[0][0] += a0 * b0; acc[0][1] += a0 * b1;
                acc[1][0] += a1 * b0; acc[1][1] += a1 * b1;
            }
        }
        __syncthreads();
    }
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            const int row = j0 + ty * 2 + i, col = k0 + tx * 2 + j;
            if (row < d && col < d) C[(long long)row * d + col] = acc[i][j];
        }
}

void launch_cross_fp64(const float* A, const float* B, long long n, int d, const double* ma,
                       const double* mb, double* C, cudaStream_t st) {
    dim3 grid(ceil_div(d, 32), ceil_div(d, 32));
    cross_fp64_kernel<false><<<grid, 256, 0, st>>>(A, B, n, d, ma, mb, C);
    VGPU_LAUNCH("cross_fp64_kernel");
}

void launch_cross_fp64_unfused(const float* A, const float* B, long long n, int d, double* C, cudaStream_t st) {
    dim3 grid(ceil_div(d, 32), ceil_div(d, 32));
    cross_fp64_kernel<true><<<grid, 256, 0, st>>>(A, B, n, d, nullptr, nullptr, C);
    VGPU_LAUNCH("cross_fp64_kernel");
}

__global__ void col_mean_kernel(const float* __restrict__ X, long long n, int d,
                                double* __restrict__ mean) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    double s = 0.0;
    for (long long i = 0; i < n; ++i) s += X[i * d + j];
    mean[j] = s / (double)n;
}

void launch_col_mean(const float* X, long long n, int d, double* mean, cudaStream_t st) {
    col_mean_kernel<<<ceil_div(d, 128), 128, 0, st>>>(X, n, d, mean);
    VGPU_LAUNCH("col_mean_kernel");
}

// C = alpha * op(A) * op(B) + beta * C for square d x d row-major fp64 matrices.
__global__ void __launch_bounds__(256) dgemm_kernel(const double* __restrict__ A,
                                                    const double* __restrict__ B, double* C, int d,
                                                    int ta, int tb, double alpha, double beta) {
    __shared__ double As[32][33];
    __shared__ double Bs[32][33];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
    double acc[2][2] = {{0, 0}, {0, 0}};
    for (int k0 = 0; k0 < d; k0 += 32) {
        for (int e = threadIdx.x; e < 1024; e += 256) {
            const int r = e / 32, c = e % 32;
            const int ai = i0 + r, ak = k0 + c;   // A(ai, ak)
            const int bk = k0 + r, bj = j0 + c;   // B(bk, bj)
            As[r][c] = (ai < d && ak < d) ? (ta ? A[(long long)ak * d + ai] : A[(long long)ai * d + ak]) : 0.0;
            Bs[r][c] = (bk < d && bj < d) ? (tb ? B[(long long)bj * d + bk] : B[(long long)bk * d + bj]) : 0.0;
        }
        __syncthreads();
        for (int k = 0; k < 32; ++k) {
            const double a0 = As[ty * 2][k], a1 = As[ty * 2 + 1][k];
            const double b0 = Bs[k][tx * 2], b1 = Bs[k][tx * 2 + 1];
            acc[0][0] += a0 * b0; acc[0][1] += a0 * b1;
            acc[1][0] += a1 * b0; acc[1][1] += a1 * b1;
        }
        __syncthreads();
    }
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            const int r = i0 + ty * 2 + i, c = j0 + tx * 2 + j;
            if (r < d && c < d) {
                const long long o = (long long)r * d + c;
                C[o] = alpha * acc[i][j] + (beta != 0.0 ? beta * C[o] : 0.0);
            }
        }
}

void launch_dgemm(const double* A, const double* B, double* C, int d, int ta, int tb, double alpha,
                  double beta, cudaStream_t st) {
    dim3 grid(ceil_div(d, 32), ceil_div(d, 32));
    dgemm_kernel<<<grid, 256, 0, st>>>(A, B, C, d, ta, tb, alpha, beta);
    VGPU_LAUNCH("dgemm_kernel");
}

__global__ void daxpby_kernel(double* y, const double* x, long long n, double a, double b) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        y[i] = a * x[i] + b * y[i];
}

void launch_daxpby(double* y, const double* x, long long n, double a, double b, cudaStream_t st) {
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 8);
    daxpby_kernel<<<blocks, 256, 0, st>>>(y, x, n, a, b);
    VGPU_LAUNCH("daxpby_kernel");
}

// ------------------------------------------------------------------ power iteration
// State per eigenvector: v (current iterate), Av, scalars {prev, done}.  One launch
// sequence per iteration; every kernel returns immediately once `done` is set, so
// the host can enqueue max_iters iterations without reading anything back.
struct PowerState {
    double prev;
    double lambda;
    int done;
};

// Av[i] = sum_j C[i][j] v[j]  (one warp per row)
__global__ void pi_matvec_kernel(const double* __restrict__ C, const double* __restrict__ v,
                                 double* __restrict__ Av, int d, const PowerState* ps) {
    if (ps->done) return;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= d) return;
    double s = 0.0;
    for (int j = lane; j < d; j += 32) s += C[(long long)row * d + j] * v[j];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) Av[row] = s;
}

// dots[p] = <w, E_p> for p < np (one warp per previous eigenvector)
__global__ void pi_dots_kernel(const double* __restrict__ E, const double* __restrict__ w,
                               double* __restrict__ dots, int d, int np, const PowerState* ps) {
    if (ps && ps->done) return;
    const int lane = threadIdx.x & 31;
    const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (p >= np) return;
    double s = 0.0;
    for (int j = lane; j < d; j += 32) s += w[j] * E[(long long)p * d + j];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) dots[p] = s;
}

// w[j] -= sum_p dots[p] * E_p[j]
__global__ void pi_deflate_kernel(const double* __restrict__ E, double* __restrict__ w,
                                  const double* __restrict__ dots, int d, int np,
                                  const PowerState* ps) {
    if (ps && ps->done) return;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    double s = w[j];
    for (int p = 0; p < np; ++p) s -= dots[p] * E[(long long)p * d + j];
    w[j] = s;
}

// Rayleigh quotient, convergence test and normalisation, one CTA.
__global__ void __launch_bounds__(1024) pi_update_kernel(double* __restrict__ v,
                                                         const double* __restrict__ Av, int d,
                                                         double tol, PowerState* ps) {
    if (ps->done) return;
    __shared__ double r1[32], r2[32], r3[32];
    double a = 0.0, b = 0.0, c = 0.0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        a += v[j] * Av[j];
        b += v[j] * v[j];
        c += Av[j] * Av[j];
    }
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { r1[w] = a; r2[w] = b; r3[w] = c; }
    __syncthreads();
    __shared__ int conv;
    __shared__ double inv_norm;
    if (threadIdx.x == 0) {
        double A = 0, B = 0, Cc = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { A += r1[i]; B += r2[i]; Cc += r3[i]; }
        const double lam = A / B;
        conv = fabs(lam - ps->prev) < tol;
        if (conv) {
            ps->done = 1;
        } else {
            ps->prev = lam;
        }
        ps->lambda = lam;
        inv_norm = 1.0 / sqrt(Cc);
    }
    __syncthreads();
    if (conv) return;
    for (int j = threadIdx.x; j < d; j += blockDim.x) v[j] = Av[j] * inv_norm;
}

__global__ void pi_init_kernel(double* v, int d, int idx, PowerState* ps) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    // The reference writes `0.1 * (i % 3 - 1)` with a std::size_t index, so for
    // i % 3 == 0 the subtraction wraps to SIZE_MAX (src/index/ivf_pq.cpp:2837-2840).
    if (j < d) v[j] = (j == idx) ? 1.0 : 0.1 * (double)((unsigned long long)j % 3ull - 1ull);
    if (j == 0) { ps->prev = 0.0; ps->lambda = 0.0; ps->done = 0; }
}

__global__ void __launch_bounds__(1024) pi_normalize_kernel(double* v, int d) {
    __shared__ double r[32];
    double s = 0.0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) s += v[j] * v[j];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = s;
    __syncthreads();
    __shared__ double nrm;
    if (threadIdx.x == 0) {
        double t = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += r[i];
        nrm = sqrt(t);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < d; j += blockDim.x) v[j] /= nrm;
}

__global__ void copy_row_kernel(double* E, const double* v, int d, int row) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < d) E[(long long)row * d + j] = v[j];
}

void power_iteration_pca(const double* C, int d, int max_iters, double tol, double* E,
                         double* work, cudaStream_t st) {
    // work: v[d], Av[d], dots[d], PowerState
    double* v = work;
    double* Av = work + d;
    double* dots = work + 2 * (size_t)d;
    PowerState* ps = reinterpret_cast<PowerState*>(work + 3 * (size_t)d);
    const int tb = 256;
    for (int e = 0; e < d; ++e) {
        pi_init_kernel<<<ceil_div(d, tb), tb, 0, st>>>(v, d, e, ps);
        if (e > 0) {
            pi_dots_kernel<<<ceil_div(e, 8), 256, 0, st>>>(E, v, dots, d, e, nullptr);
            pi_deflate_kernel<<<ceil_div(d, tb), tb, 0, st>>>(E, v, dots, d, e, nullptr);
        }
        pi_normalize_kernel<<<1, 1024, 0, st>>>(v, d);
        for (int it = 0; it < max_iters; ++it) {
            pi_matvec_kernel<<<ceil_div(d, 8), 256, 0, st>>>(C, v, Av, d, ps);
            if (e > 0) {
                pi_dots_kernel<<<ceil_div(e, 8), 256, 0, st>>>(E, Av, dots, d, e, ps);
                pi_deflate_kernel<<<ceil_div(d, tb), tb, 0, st>>>(E, Av, dots, d, e, ps);
            }
            pi_update_kernel<<<1, 1024, 0, st>>>(v, Av, d, tol, ps);
        }
        copy_row_kernel<<<ceil_div(d, tb), tb, 0, st>>>(E, v, d, e);
        VGPU_LAUNCH("power_iteration_pca");
    }
}

}  // namespace vgpu
