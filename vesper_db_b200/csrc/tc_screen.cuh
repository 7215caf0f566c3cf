// Bounds and exact scores shared by the tf32 tensor-core screens (tc_coarse.cu) and
// the flat top-k refine (flat_topk.cu).
#pragma once

#include "common.cuh"

namespace vgpu {

// Relative error of a tf32 dot product against ||x|| ||c||: truncation of both operands
// (2^-10 each) and fp32 accumulation over up to dim + 16 terms (the products and the
// two norm terms of the augmented screen below), with 0.4 % headroom.
__host__ __device__ __forceinline__ float screen_a(int dim) {
    return 1.953125e-3f + (float)(dim + 16) * 1.1920929e-7f * 1.00390625f;
}
// The augmented L2 screen folds -||c||^2 / 2 into the product as two tf32 terms
// (hi + lo, residual below 2^-21 ||c||^2) that are accumulated with the others: their
// share of the accumulation error plus the residual, per unit of ||c||^2.
__host__ __device__ __forceinline__ float screen_r2(int dim) {
    return (float)(dim + 16) * 5.9604645e-8f * 1.00390625f + 4.7683716e-7f;
}

// Screening error bound of an L2 screen value Dt (||x||^2 + ||c||^2 - 2 S, or
// ||x||^2 - 2 S' with the augmented S' = S - ||c||^2 / 2): the tf32 product, the
// augmented norm terms, fp32 rounding of the epilogue and of the norms, and the
// reference-order rounding of d_ref; times a safety factor of 2.
__device__ __forceinline__ float screen_eps(float xn, float cn, float dt, int dim) {
    const float a = screen_a(dim);
    const float xc = sqrtf(xn * cn);
    const float e = 2.0f * a * xc + 2.0f * screen_r2(dim) * cn + 2.384e-7f * (xn + cn + 2.0f * xc) +
                    (float)(dim / 8 + 8) * 1.1920929e-7f * fabsf(dt);
    return 2.0f * e + 1e-30f;
}

// Exact l2 for up to 4 candidates per warp: lane group g = lane / 8 takes candidate g,
// lane (lane % 8) plays AVX2 lane l, then an 8-lane hsum in the reference order.
__device__ __forceinline__ float warp_l2_group(const float* __restrict__ x, const float* __restrict__ c, int dim,
                                               bool active) {
    const int lane = threadIdx.x & 31, l = lane & 7;
    const int simd_end = dim & ~7;
    float acc = 0.0f;
    if (active) {
#pragma unroll 8
        for (int t = l; t < simd_end; t += 8) {
            const float d = __fsub_rn(x[t], c[t]);
            acc = __fmaf_rn(d, d, acc);
        }
    }
    const float a4 = __shfl_down_sync(0xffffffffu, acc, 4, 8);
    const float s = __fadd_rn(a4, acc);
    const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
    const float s2 = __shfl_down_sync(0xffffffffu, s, 2, 8);
    const float s3 = __shfl_down_sync(0xffffffffu, s, 3, 8);
    float r = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
    if (active)
        for (int t = simd_end; t < dim; ++t) {
            const float d = __fsub_rn(x[t], c[t]);
            r = __fadd_rn(r, __fmul_rn(d, d));
        }
    return r;  // valid in lane l == 0 of each group
}

// Screening bound for inner products: the screen value is -2 S' with S' the tf32 dot;
// |S' - S| <= a ||x|| ||c|| and |S - s_ref| <= (dim/8 + 8) 2^-23 ||x|| ||c|| (the
// reference's lane sums), doubled for the -2 factor, times a safety factor of 2.
__device__ __forceinline__ float screen_eps_ip(float xn, float cn, int dim) {
    const float a = 1.953125e-3f + (float)(dim + 8) * 1.1920929e-7f;
    const float r = (float)(dim / 8 + 8) * 1.1920929e-7f;
    return 4.0f * (a + r + 2.4e-7f) * sqrtf(xn * cn) + 1e-30f;
}

// Exact inner product (reference lane order) for up to 4 candidates per warp, as
// warp_l2_group.
__device__ __forceinline__ float warp_ip_group(const float* __restrict__ x, const float* __restrict__ c, int dim,
                                               bool active) {
    const int lane = threadIdx.x & 31, l = lane & 7;
    const int simd_end = dim & ~7;
    float acc = 0.0f;
    if (active) {
#pragma unroll 8
        for (int t = l; t < simd_end; t += 8) acc = __fmaf_rn(x[t], c[t], acc);
    }
    const float a4 = __shfl_down_sync(0xffffffffu, acc, 4, 8);
    const float s = __fadd_rn(a4, acc);
    const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
    const float s2 = __shfl_down_sync(0xffffffffu, s, 2, 8);
    const float s3 = __shfl_down_sync(0xffffffffu, s, 3, 8);
    float r = __fadd_rn(__fadd_rn(s, s1), __fadd_rn(s2, s3));
    if (active)
        for (int t = simd_end; t < dim; ++t) r = __fadd_rn(r, __fmul_rn(x[t], c[t]));
    return r;  // valid in lane l == 0 of each group
}

}  // namespace vgpu
