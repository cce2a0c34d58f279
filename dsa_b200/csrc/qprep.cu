// Decode-step tail of the sidecar query projection (reference sidecar.py:78-87), one launch:
//   q[b,h,:] = RoPE_noninterleaved(qraw[b, h*128 : h*128+128]) on the first rope_dim dims
//   w[b,h]   = scale * sum_k float(x[b,k]) * W_w[h,k]        (float32, as the reference's
//                                                              autocast-disabled weights_proj)
// qraw is the [B, 64*128] output of the W_q GEMM (cuBLAS, 16-bit).  Grid (B, 2): y = 0 CTAs
// rotate one row of q, y = 1 CTAs compute one row of w (a float32 GEMV over the hidden
// size; W_w streams from L2 as independent float4 loads).  RoPE angles are position * theta^(-j/half) in float32 as in
// the reference; the rotation is done in float32 and rounded once.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 512;

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half x) {
  return __half2float(x);
}
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half from_f<__half>(float x) {
  return __float2half_rn(x);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    qprep_kernel(const T* __restrict__ qraw, int64_t qraw_stride, const T* __restrict__ x,
                 int64_t x_stride, int hidden, const float* __restrict__ ww,
                 const int64_t* __restrict__ positions, T* __restrict__ q, int64_t q_stride,
                 float* __restrict__ w, int64_t w_stride, int rope_dim, float theta,
                 float scale) {
  extern __shared__ float xs[];  // GEMV partials [16][64]
  __shared__ float cs[64], sn[64];
  const int b = blockIdx.x;
  if (blockIdx.y == 0) {
    const int half = rope_dim >> 1;
    if (threadIdx.x < half) {
      const float inv_freq =
          powf(theta, -static_cast<float>(threadIdx.x) / static_cast<float>(half));
      const float angle = static_cast<float>(positions[b]) * inv_freq;
      sincosf(angle, &sn[threadIdx.x], &cs[threadIdx.x]);
    }
    __syncthreads();
    const T* src = qraw + static_cast<int64_t>(b) * qraw_stride;
    T* dst = q + static_cast<int64_t>(b) * q_stride;
    for (int i = threadIdx.x; i < kHeads * kHeadDim; i += kThreads) {
      const int h = i >> 7, d = i & 127;
      const T* row = src + h * kHeadDim;
      float out = to_f(row[d]);
      if (d < rope_dim) {
        const int j = d < half ? d : d - half;
        const float first = to_f(row[j]), second = to_f(row[j + half]);
        out = d < half ? first * cs[j] - second * sn[j] : second * cs[j] + first * sn[j];
      }
      dst[i] = from_f<T>(out);
    }
    return;
  }
  // w row b: the hidden axis is split over the 16 warps (128 dims per warp per round, 4 per
  // lane); every lane keeps 64 head partials, so each W_w load is an independent float4 and
  // the loads of all heads are in flight together.  Fixed-order reductions: lanes, then warps.
  float* red = xs;  // [16 warps][64 heads]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* xr = x + static_cast<int64_t>(b) * x_stride;
  float acc[kHeads];
#pragma unroll
  for (int h = 0; h < kHeads; ++h) acc[h] = 0.f;
  for (int k0 = warp * 128 + lane * 4; k0 < hidden; k0 += (kThreads / 32) * 128) {
    float xv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) xv[j] = k0 + j < hidden ? to_f(xr[k0 + j]) : 0.f;
    const bool full4 = k0 + 4 <= hidden && (hidden & 3) == 0;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      const float* wr = ww + static_cast<int64_t>(h) * hidden + k0;
      float4 v;
      if (full4) {
        v = __ldg(reinterpret_cast<const float4*>(wr));
      } else {
        v.x = k0 + 0 < hidden ? __ldg(wr + 0) : 0.f;
        v.y = k0 + 1 < hidden ? __ldg(wr + 1) : 0.f;
        v.z = k0 + 2 < hidden ? __ldg(wr + 2) : 0.f;
        v.w = k0 + 3 < hidden ? __ldg(wr + 3) : 0.f;
      }
      acc[h] = fmaf(xv[0], v.x, fmaf(xv[1], v.y, fmaf(xv[2], v.z, fmaf(xv[3], v.w, acc[h]))));
    }
  }
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    float v = acc[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * kHeads + h] = v;
  }
  __syncthreads();
  if (threadIdx.x < kHeads) {
    float s = 0.f;
    for (int wi = 0; wi < kThreads / 32; ++wi) s += red[wi * kHeads + threadIdx.x];
    w[static_cast<int64_t>(b) * w_stride + threadIdx.x] = s * scale;
  }
}

}  // namespace

int launch_qprep(const void* qraw, int64_t qraw_stride, const void* x, int64_t x_stride,
                 int hidden, const float* ww, const int64_t* positions, void* q,
                 int64_t q_stride, float* w, int64_t w_stride, int dtype, int batch,
                 int rope_dim, float theta, float scale, cudaStream_t stream) {
  const dim3 grid(batch, 2);
  const size_t smem = static_cast<size_t>(kThreads / 32) * kHeads * 4;
  if (dtype == TDSA_BF16) {
    auto kern = qprep_kernel<__nv_bfloat16>;
    TDSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    kern<<<grid, kThreads, smem, stream>>>(
        static_cast<const __nv_bfloat16*>(qraw), qraw_stride,
        static_cast<const __nv_bfloat16*>(x), x_stride, hidden, ww, positions,
        static_cast<__nv_bfloat16*>(q), q_stride, w, w_stride, rope_dim, theta, scale);
  } else {
    auto kern = qprep_kernel<__half>;
    TDSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    kern<<<grid, kThreads, smem, stream>>>(
        static_cast<const __half*>(qraw), qraw_stride, static_cast<const __half*>(x), x_stride,
        hidden, ww, positions, static_cast<__half*>(q), q_stride, w, w_stride, rope_dim, theta,
        scale);
  }
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
