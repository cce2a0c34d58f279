// Decode-step tail of the sidecar query projection (reference sidecar.py:78-87), one launch:
//   q[b,h,:] = RoPE_noninterleaved(qraw[b, h*128 : h*128+128]) on the first rope_dim dims
//   w[b,h]   = scale * sum_k float(x[b,k]) * W_w[h,k]     (float32, as the reference's
//                                                           autocast-disabled weights_proj)
// qraw is the [B, 64*128] output of the W_q GEMM (cuBLAS, 16-bit).
// CTAs [0, B) rotate one row of q each.  The other CTAs tile w by (head, group of 16 batch
// rows): the head's W_w row is read once into registers (8 dims per thread), each batch
// row's hidden state is one 16-byte load per thread, and every dot product reduces in a
// fixed order (lanes, then warps).  RoPE angles are position * theta^(-j/half) in float32
// as in the reference; the rotation is done in float32 and rounded once.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 256;
constexpr int kRows = 16;  // batch rows per GEMV CTA

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
                 float* __restrict__ w, int64_t w_stride, int batch, int rope_dim, float theta,
                 float scale) {
  __shared__ float cs[64], sn[64];
  __shared__ float red[kThreads / 32][kRows];
  if (static_cast<int>(blockIdx.x) < batch) {
    const int b = blockIdx.x;
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
  // GEMV tile: head h, batch rows [b0, b0 + kRows)
  const int tile = blockIdx.x - batch;
  const int h = tile % kHeads;
  const int b0 = (tile / kHeads) * kRows;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float part[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) part[r] = 0.f;
  for (int k0 = threadIdx.x * 8; k0 < hidden; k0 += kThreads * 8) {
    float wv[8];
    const float* wr = ww + static_cast<int64_t>(h) * hidden + k0;
    const bool full = k0 + 8 <= hidden;
    if (full && (reinterpret_cast<uintptr_t>(wr) & 15u) == 0u) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(wr));
      const float4 c = __ldg(reinterpret_cast<const float4*>(wr) + 1);
      wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
      wv[4] = c.x; wv[5] = c.y; wv[6] = c.z; wv[7] = c.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = k0 + j < hidden ? __ldg(wr + j) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (b0 + r < batch) {
        const T* xr = x + static_cast<int64_t>(b0 + r) * x_stride + k0;
        float xv[8];
        if (full && (reinterpret_cast<uintptr_t>(xr) & 15u) == 0u) {
          const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr));
          const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = to_f(e[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = k0 + j < hidden ? to_f(xr[j]) : 0.f;
        }
        float acc = part[r];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(xv[j], wv[j], acc);
        part[r] = acc;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    float v = part[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp][r] = v;
  }
  __syncthreads();
  if (threadIdx.x < kRows && b0 + static_cast<int>(threadIdx.x) < batch) {
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < kThreads / 32; ++wi) s += red[wi][threadIdx.x];
    w[static_cast<int64_t>(b0 + threadIdx.x) * w_stride + h] = s * scale;
  }
}

}  // namespace

int launch_qprep(const void* qraw, int64_t qraw_stride, const void* x, int64_t x_stride,
                 int hidden, const float* ww, const int64_t* positions, void* q,
                 int64_t q_stride, float* w, int64_t w_stride, int dtype, int batch,
                 int rope_dim, float theta, float scale, cudaStream_t stream) {
  const int gemv_ctas = kHeads * ((batch + kRows - 1) / kRows);
  const dim3 grid(batch + gemv_ctas);
  if (dtype == TDSA_BF16)
    qprep_kernel<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(qraw), qraw_stride,
        static_cast<const __nv_bfloat16*>(x), x_stride, hidden, ww, positions,
        static_cast<__nv_bfloat16*>(q), q_stride, w, w_stride, batch, rope_dim, theta, scale);
  else
    qprep_kernel<__half><<<grid, kThreads, 0, stream>>>(
        static_cast<const __half*>(qraw), qraw_stride, static_cast<const __half*>(x), x_stride,
        hidden, ww, positions, static_cast<__half*>(q), q_stride, w, w_stride, batch, rope_dim,
        theta, scale);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
