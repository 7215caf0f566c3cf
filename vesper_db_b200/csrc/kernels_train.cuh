// Training-time kernels (definitions in train_kernels.cu).
#pragma once

#include "common.cuh"

namespace vgpu {

void launch_fill(float* p, long long n, float v, cudaStream_t st);

// Batched k-means++ over the m PQ sub-spaces: mind [m x n].
void launch_pq_kpp_update(const float* x, long long n, int dim, int m, int dsub,
                          const float* picks, float* mind, cudaStream_t st);
void launch_pq_gather_picks(const float* x, int dim, int m, int dsub, const uint32_t* idx, int slot,
                            int ksub, float* picks, float* cb, cudaStream_t st);
// E-step of all sub-space k-means; codes/mind are [m x n]; keep = Elkan tie rule.
void launch_pq_assign(const float* x, long long n, int dim, int m, int ksub, int dsub,
                      const float* cb, uint32_t* codes, float* mind, int keep, const int* active,
                      cudaStream_t st);
void launch_pq_keys(const uint32_t* codes, long long n, int m, int ksub, uint32_t* keys,
                    cudaStream_t st);
void launch_pq_segment_mean(const float* x, long long n, int dim, int m, int dsub, int ksub,
                            const uint32_t* order, const uint32_t* seg, const int* active, float* cb,
                            cudaStream_t st);

// Scratch for group_by_key (grow-only).
struct GroupWork {
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    uint32_t* keys_out = nullptr;
    uint32_t* vals_in = nullptr;
    size_t cap = 0;
    GroupWork() = default;
    GroupWork(const GroupWork&) = delete;
    GroupWork& operator=(const GroupWork&) = delete;
    ~GroupWork();
};
// order = item indices grouped by key (item order kept inside a key);
// seg[0..nkeys] = segment offsets.
void group_by_key(const uint32_t* keys, long long n, int nkeys, uint32_t* order, uint32_t* seg,
                  GroupWork& w, cudaStream_t st);

void launch_pq_decode(const uint8_t* codes, long long n, int m, int ksub, int dsub, const float* cb,
                      float* out, cudaStream_t st);
void launch_row_l2(const float* a, const float* b, long long n, int dim, float* out, cudaStream_t st);
void launch_transpose(const float* in, int d, float* out, cudaStream_t st);
void launch_gather_rows(const float* x, int dim, const uint32_t* idx, long long n, float* out,
                        cudaStream_t st);
void launch_gather_u32(const uint32_t* src, const uint32_t* idx, long long n, uint32_t* out, cudaStream_t st);
void launch_d2f(const double* in, long long n, float* out, cudaStream_t st);

}  // namespace vgpu
