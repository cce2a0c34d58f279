// The per-key epilogue shared by every scoring kernel: ReLU, head weight, head sum.
// One fixed summation order (four interleaved partial sums over h mod 4, combined as
// (s0 + s1) + (s2 + s3)) makes every kernel that calls it produce bit-identical scores
// for the same head dots -- the exact progressive path relies on this to return the
// dense path's top-k.
#pragma once

#include <cstdint>

namespace tdsa {

__device__ __forceinline__ void load_head_weights(const float* w, float (&wr)[64]) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
  if ((reinterpret_cast<uintptr_t>(w) & 15u) == 0u) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v = __ldg(w4 + i);
      wr[4 * i + 0] = v.x;
      wr[4 * i + 1] = v.y;
      wr[4 * i + 2] = v.z;
      wr[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int h = 0; h < 64; ++h) wr[h] = __ldg(w + h);
  }
}

__device__ __forceinline__ float relu_weighted_sum(const uint32_t (&lo)[32],
                                                   const uint32_t (&hi)[32],
                                                   const float (&wr)[64]) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int h = 0; h < 32; h += 4) {
    s0 = fmaf(wr[h + 0], fmaxf(__uint_as_float(lo[h + 0]), 0.f), s0);
    s1 = fmaf(wr[h + 1], fmaxf(__uint_as_float(lo[h + 1]), 0.f), s1);
    s2 = fmaf(wr[h + 2], fmaxf(__uint_as_float(lo[h + 2]), 0.f), s2);
    s3 = fmaf(wr[h + 3], fmaxf(__uint_as_float(lo[h + 3]), 0.f), s3);
  }
#pragma unroll
  for (int h = 0; h < 32; h += 4) {
    s0 = fmaf(wr[32 + h + 0], fmaxf(__uint_as_float(hi[h + 0]), 0.f), s0);
    s1 = fmaf(wr[32 + h + 1], fmaxf(__uint_as_float(hi[h + 1]), 0.f), s1);
    s2 = fmaf(wr[32 + h + 2], fmaxf(__uint_as_float(hi[h + 2]), 0.f), s2);
    s3 = fmaf(wr[32 + h + 3], fmaxf(__uint_as_float(hi[h + 3]), 0.f), s3);
  }
  return (s0 + s1) + (s2 + s3);
}

}  // namespace tdsa
