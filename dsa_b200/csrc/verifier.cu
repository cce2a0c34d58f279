// Dimension-sparse verifier scorer on the device (reference verifier_scoring.py:9-139):
//   hadamard128_kernel      normalized_hadamard (:9-26) of 128-wide rows: one warp per row,
//                           four elements per lane, butterflies in the reference's order
//                           (stride 1 first; left + right, left - right), float32
//                           arithmetic, times the float32 of 128^-1/2
//   absmax_kernel           the tensor-wide max |x| of fake_symmetric_quantize (:29-41)
//   select_quant_kernel     the kept dimensions, optionally fake-quantized:
//                           clamp(rint(x / scale), -limit, limit) * scale; the others 0
// score_dim_sparse (:95-139) is then the dense scorer on these 128-wide rows: a dot
// product over the kept dimensions equals the reference's over the selected ones.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float ld<__half>(const __half* p) {
  return __half2float(*p);
}

template <typename T>
__device__ __forceinline__ void st(T* p, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, float v) {
  *p = v;
}
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void st<__half>(__half* p, float v) {
  *p = __float2half_rn(v);
}

template <typename T>
__global__ void hadamard128_kernel(const T* __restrict__ in, int64_t in_stride, int64_t rows,
                                   T* __restrict__ out, int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const T* src = in + r * in_stride + 4 * lane;
    float v[4] = {ld(src), ld(src + 1), ld(src + 2), ld(src + 3)};
    // stride 1 and 2: inside the lane's four elements
    float a = v[0] + v[1], b = v[0] - v[1], c = v[2] + v[3], d = v[2] - v[3];
    v[0] = a + c;
    v[1] = b + d;
    v[2] = a - c;
    v[3] = b - d;
    // strides 4 .. 64: element e pairs with e ^ stride, i.e. lane ^ (stride / 4)
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const bool left = (lane & m) == 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
        v[j] = left ? v[j] + o : o - v[j];
      }
    }
    constexpr float kScale = 0.08838834764831845f;  // 128^-1/2
    T* dst = out + r * out_stride + 4 * lane;
#pragma unroll
    for (int j = 0; j < 4; ++j) st(dst + j, v[j] * kScale);
  }
}

// max |x| over the kept entries, as the bits of a non-negative float (they order like
// unsigned integers), into *out (which starts at 0)
template <typename T>
__global__ void absmax_kernel(const T* __restrict__ in, int64_t stride, int64_t rows, int width,
                              const int8_t* __restrict__ keep, uint32_t* out) {
  float m = 0.f;
  const int64_t total = rows * width;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / width;
    const int c = static_cast<int>(e - r * width);
    if (!keep || keep[c]) m = fmaxf(m, fabsf(ld(in + r * stride + c)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

template <typename T>
__global__ void select_quant_kernel(const T* __restrict__ in, int64_t in_stride, int64_t rows,
                                    int width, const int8_t* __restrict__ keep, int bits,
                                    double scale_given, const uint32_t* __restrict__ absmax,
                                    T* __restrict__ out, int64_t out_stride) {
  const float limit = static_cast<float>((1 << (bits > 0 ? bits - 1 : 0)) - 1);
  float scale = 0.f;
  if (bits > 0) {
    // reference: float(max|x|) / max(limit, 1), then max(scale, 1e-12), in double; the
    // division and product below use that scale rounded to float32
    double s = scale_given > 0.0
                   ? scale_given
                   : static_cast<double>(__uint_as_float(*absmax)) / fmax(limit, 1.0);
    s = fmax(s, 1e-12);
    scale = static_cast<float>(s);
  }
  const int64_t total = rows * width;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / width;
    const int c = static_cast<int>(e - r * width);
    float v = 0.f;
    if (!keep || keep[c]) {
      v = ld(in + r * in_stride + c);
      if (bits > 0) v = fminf(fmaxf(rintf(v / scale), -limit), limit) * scale;
    }
    st(out + r * out_stride + c, v);
  }
}

template <typename T>
int launch_verifier_t(const void* in, int64_t in_stride, int64_t rows, int width,
                      const int8_t* keep, int bits, double scale, uint32_t* absmax, void* out,
                      int64_t out_stride, cudaStream_t stream) {
  const int64_t total = rows * width;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 8));
  if (bits > 0 && scale <= 0.0) {
    TDSA_CUDA_CHECK(cudaMemsetAsync(absmax, 0, sizeof(uint32_t), stream));
    absmax_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(in), in_stride, rows,
                                                  width, keep, absmax);
    TDSA_CUDA_CHECK(cudaGetLastError());
  }
  select_quant_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(in), in_stride, rows,
                                                     width, keep, bits, scale, absmax,
                                                     static_cast<T*>(out), out_stride);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace

int launch_hadamard128(const void* in, int64_t in_stride, int64_t rows, int dtype, void* out,
                       int64_t out_stride, cudaStream_t stream) {
  const int blocks = static_cast<int>(std::min<int64_t>((rows + 7) / 8, 148 * 16));
  if (dtype == TDSA_F32)
    hadamard128_kernel<float><<<blocks, 256, 0, stream>>>(
        static_cast<const float*>(in), in_stride, rows, static_cast<float*>(out), out_stride);
  else if (dtype == TDSA_BF16)
    hadamard128_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(in), in_stride, rows,
        static_cast<__nv_bfloat16*>(out), out_stride);
  else
    hadamard128_kernel<__half><<<blocks, 256, 0, stream>>>(
        static_cast<const __half*>(in), in_stride, rows, static_cast<__half*>(out), out_stride);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

int launch_select_quantize(const void* in, int64_t in_stride, int64_t rows, int width,
                           int dtype, const int8_t* keep, int bits, double scale,
                           uint32_t* absmax, void* out, int64_t out_stride,
                           cudaStream_t stream) {
  if (dtype == TDSA_F32)
    return launch_verifier_t<float>(in, in_stride, rows, width, keep, bits, scale, absmax, out,
                                    out_stride, stream);
  if (dtype == TDSA_BF16)
    return launch_verifier_t<__nv_bfloat16>(in, in_stride, rows, width, keep, bits, scale,
                                            absmax, out, out_stride, stream);
  return launch_verifier_t<__half>(in, in_stride, rows, width, keep, bits, scale, absmax, out,
                                   out_stride, stream);
}

}  // namespace tdsa
