// Query epilogue of the sidecar projection (reference sidecar.py:78-87), fused:
//   q[b,h,:]  = RoPE_noninterleaved(qraw[b, h*128 : h*128+128]) on the first rope_dim dims
//   w[b,h]    = wraw[b,h] * scale            (scale = (64*128)^-1/2 in the reference)
// qraw is the [B, 64*128] output of the W_q GEMM (cuBLAS), wraw the [B,64] float32 output
// of the W_w GEMM.  RoPE angles are position * theta^(-j/half) in float32, as the
// reference computes them; the rotation is done in float32 and rounded once.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

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
__global__ void qprep_kernel(const T* __restrict__ qraw, int64_t qraw_stride,
                             const float* __restrict__ wraw, int64_t wraw_stride,
                             const int64_t* __restrict__ positions, T* __restrict__ q,
                             int64_t q_stride, float* __restrict__ w, int64_t w_stride,
                             int rope_dim, float theta, float scale) {
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // element of the 64*128 row
  if (i < kHeads * kHeadDim) {
    const int h = i >> 7, d = i & 127;
    const T* src = qraw + static_cast<int64_t>(b) * qraw_stride + h * kHeadDim;
    float out = to_f(src[d]);
    if (d < rope_dim) {
      const int half = rope_dim >> 1;
      const int j = d < half ? d : d - half;
      const float inv_freq = powf(theta, -static_cast<float>(j) / static_cast<float>(half));
      const float angle = static_cast<float>(positions[b]) * inv_freq;
      float s, c;
      sincosf(angle, &s, &c);
      const float first = to_f(src[j]), second = to_f(src[j + half]);
      out = d < half ? first * c - second * s : second * c + first * s;
    }
    q[static_cast<int64_t>(b) * q_stride + i] = from_f<T>(out);
  }
  if (blockIdx.x == 0 && threadIdx.x < kHeads)
    w[static_cast<int64_t>(b) * w_stride + threadIdx.x] =
        wraw[static_cast<int64_t>(b) * wraw_stride + threadIdx.x] * scale;
}

}  // namespace

int launch_qprep(const void* qraw, int64_t qraw_stride, const float* wraw, int64_t wraw_stride,
                 const int64_t* positions, void* q, int64_t q_stride, float* w,
                 int64_t w_stride, int dtype, int batch, int rope_dim, float theta,
                 float scale, cudaStream_t stream) {
  const dim3 grid((kHeads * kHeadDim + 255) / 256, batch);
  if (dtype == TDSA_BF16)
    qprep_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(qraw), qraw_stride, wraw, wraw_stride, positions,
        static_cast<__nv_bfloat16*>(q), q_stride, w, w_stride, rope_dim, theta, scale);
  else
    qprep_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(qraw), qraw_stride, wraw, wraw_stride, positions,
        static_cast<__half*>(q), q_stride, w, w_stride, rope_dim, theta, scale);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
