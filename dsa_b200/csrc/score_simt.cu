// Dense indexer scoring for float32 queries and keys on the FP32 CUDA cores.
//
// The tensor-core kinds take 16-bit (or TF32) operands; TF32 alone misses the 1e-5 float32
// tolerance, so the float32 key cache uses exact FP32 FMAs.  Block tile: 128 keys x
// 64 heads, 128 threads; thread (ty, tx) owns keys 8*ty..8*ty+7 and heads 8*tx..8*tx+7
// (64 accumulators) and walks the 128 dims out of shared memory.  The ReLU-weighted head
// sum is reduced over the 8 tx lanes of a key with a fixed butterfly (deterministic).
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kKeys = 128;
constexpr int kThreads = 128;
constexpr int kKPad = kHeadDim + 1;  // key rows padded: conflict-free column reads
constexpr int kSmemBytes = (kKeys * kKPad + kHeadDim * kHeads) * 4;

__global__ void __launch_bounds__(kThreads)
    score_dense_f32_kernel(const float* __restrict__ q, int64_t q_bs,
                           const float* __restrict__ w, int64_t w_bs,
                           const float* __restrict__ keys, int64_t k_bs, int64_t k_rs,
                           int length, float* __restrict__ out, int64_t o_bs) {
  extern __shared__ float sm[];
  float* ks = sm;                      // [128 keys][129]
  float* qt = sm + kKeys * kKPad;      // [128 dims][64 heads]
  const int b = blockIdx.y;
  const int key0 = blockIdx.x * kKeys;
  const int tid = threadIdx.x;
  const float* qb = q + static_cast<int64_t>(b) * q_bs;
  const float* kb = keys + static_cast<int64_t>(b) * k_bs;

  // q transposed to [dim][head]; consecutive threads take consecutive heads.
  for (int i = tid; i < kHeads * kHeadDim; i += kThreads) {
    const int h = i & (kHeads - 1), d = i >> 6;
    qt[d * kHeads + h] = __ldg(qb + h * kHeadDim + d);
  }
  // Key tile, one row per warp iteration (coalesced), rows beyond `length` are zero.
  for (int i = tid; i < kKeys * (kHeadDim / 4); i += kThreads) {
    const int r = i >> 5, c4 = i & 31;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (key0 + r < length) {
      const float* src = kb + static_cast<int64_t>(key0 + r) * k_rs + 4 * c4;
      if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0u) {
        v = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        v = make_float4(__ldg(src), __ldg(src + 1), __ldg(src + 2), __ldg(src + 3));
      }
    }
    float* dst = ks + r * kKPad + 4 * c4;
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  }
  __syncthreads();

  const int tx = tid & 7, ty = tid >> 3;
  float acc[8][8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;

#pragma unroll 4
  for (int d = 0; d < kHeadDim; ++d) {
    float kv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) kv[j] = ks[(8 * ty + j) * kKPad + d];
    const float4 qa = *reinterpret_cast<const float4*>(qt + d * kHeads + 8 * tx);
    const float4 qc = *reinterpret_cast<const float4*>(qt + d * kHeads + 8 * tx + 4);
    const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qc.x, qc.y, qc.z, qc.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[j][i] = fmaf(kv[j], qv[i], acc[j][i]);
  }

  float wv[8];
  const float* wb = w + static_cast<int64_t>(b) * w_bs;
#pragma unroll
  for (int i = 0; i < 8; ++i) wv[i] = __ldg(wb + 8 * tx + i);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = fmaf(wv[i], fmaxf(acc[j][i], 0.f), s);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    const int row = key0 + 8 * ty + j;
    if (tx == 0 && row < length) out[static_cast<int64_t>(b) * o_bs + row] = s;
  }
}

}  // namespace

int launch_score_dense_f32(const float* q, int64_t q_bs, const float* w, int64_t w_bs,
                           const float* k, int64_t k_bs, int64_t k_rs, int batch, int length,
                           float* out, int64_t o_bs, cudaStream_t stream) {
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(score_dense_f32_kernel),
                                      kSmemBytes));
  const dim3 grid((length + kKeys - 1) / kKeys, batch);
  score_dense_f32_kernel<<<grid, kThreads, kSmemBytes, stream>>>(q, q_bs, w, w_bs, k, k_bs,
                                                                  k_rs, length, out, o_bs);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
