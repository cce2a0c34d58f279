// Small companions of the block-structured scoring kernels.
//
// compact_blocks_kernel: the compact output of the progressive H8 path (reference
// progressive_kernel.py:335-340, :468-474).  The reference hands out output slots with an
// atomic counter, so its candidate order varies run to run and the ragged last block can
// leave unwritten slots inside candidate_count.  Here one CTA per sequence scans the
// accepted flags in block order and packs every valid key of the accepted blocks: the same
// candidate set, in ascending key order, with an exact count.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 1024;

__global__ void __launch_bounds__(kThreads)
    compact_blocks_kernel(const float* __restrict__ scores, int64_t s_stride,
                          const int8_t* __restrict__ accepted, int64_t a_stride, int length,
                          int bs, float* __restrict__ out_scores, int32_t* __restrict__ out_idx,
                          int64_t o_stride, int32_t* __restrict__ out_count) {
  __shared__ uint32_t warp_tot[32];
  __shared__ uint32_t carry;
  const int seq = blockIdx.x;
  const float* srow = scores + static_cast<int64_t>(seq) * s_stride;
  const int8_t* arow = accepted + static_cast<int64_t>(seq) * a_stride;
  float* os = out_scores + static_cast<int64_t>(seq) * o_stride;
  int32_t* oi = out_idx + static_cast<int64_t>(seq) * o_stride;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  // Keys in chunks of 1024, ordered compaction with a block-wide exclusive scan.
  for (int base = 0; base < length; base += kThreads) {
    const int key = base + threadIdx.x;
    const bool take = key < length && arow[key / bs] != 0;
    const unsigned ballot = __ballot_sync(0xffffffffu, take);
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    uint32_t before = 0, chunk = 0;
    for (int w = 0; w < 32; ++w) {
      const uint32_t c = warp_tot[w];
      if (w < warp) before += c;
      chunk += c;
    }
    before += __popc(ballot & ((1u << lane) - 1u));
    const uint32_t pos = carry + before;
    if (take) {
      os[pos] = srow[key];
      oi[pos] = key;
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += chunk;
    __syncthreads();
  }
  if (threadIdx.x == 0) out_count[seq] = static_cast<int32_t>(carry);
}

}  // namespace

int launch_compact_blocks(const float* scores, int64_t s_stride, const int8_t* accepted,
                          int64_t a_stride, int batch, int length, int block_size,
                          float* out_scores, int32_t* out_indices, int64_t o_stride,
                          int32_t* out_count, cudaStream_t stream) {
  compact_blocks_kernel<<<batch, kThreads, 0, stream>>>(scores, s_stride, accepted, a_stride,
                                                         length, block_size, out_scores,
                                                         out_indices, o_stride, out_count);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
