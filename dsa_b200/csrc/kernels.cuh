// Host-side launchers of the indexer kernels (one definition per .cu file).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace tdsa {

constexpr int kTopkSegment = 32768;    // keys one top-k CTA holds in shared memory
constexpr int kTopkMaxSorted = 8192;   // largest k sorted in shared memory

int launch_score_dense_tc(const void* q, int64_t q_bs, const float* w, int64_t w_bs,
                          const void* k, int64_t k_bs, int64_t k_rs, int dtype, int batch,
                          int length, float* out, int64_t o_bs, cudaStream_t stream,
                          int* status);

int launch_score_dense_f32(const float* q, int64_t q_bs, const float* w, int64_t w_bs,
                           const float* k, int64_t k_bs, int64_t k_rs, int batch, int length,
                           float* out, int64_t o_bs, cudaStream_t stream);

size_t topk_workspace_bytes(int batch, int length, int k);
int topk_check(int length, int k, int sorted);
int launch_topk(const float* scores, int64_t s_stride, const int32_t* idx, int64_t idx_stride,
                int batch, int length, int k, int sorted, void* out_idx, int idx_bytes,
                int64_t oi_stride, float* out_val, int64_t ov_stride, void* ws, size_t ws_bytes,
                cudaStream_t stream);

int launch_qprep(const void* qraw, int64_t qraw_stride, const float* wraw, int64_t wraw_stride,
                 const int64_t* positions, void* q, int64_t q_stride, float* w,
                 int64_t w_stride, int dtype, int batch, int rope_dim, float theta,
                 float scale, cudaStream_t stream);

// Device status word of the current device (allocated with the module, never freed).
int* device_status_ptr();

}  // namespace tdsa
