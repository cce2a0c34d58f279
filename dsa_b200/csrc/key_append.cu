// Decode-step key append (reference sidecar.py:74-76, encode_keys, one new token per
// sequence), fused into one launch that writes straight into the key cache:
//
//   k[b] = RoPE_{pos[b]}(LayerNorm(round16(h[b] @ W_k^T)))  ->  cache[b][slot[b]][0..128)
//
// A cluster of 8 CTAs serves 4 sequences.  CTA r takes the r-th eighth of the hidden
// dimension: it stages its W_k slice [128 features x chunk] in shared memory with coalesced
// 16-byte loads (rows padded by 16 bytes so the per-feature 16-byte reads of a warp land on
// distinct banks; cp.async, all in flight at once) and the 4 sequences' hidden slices as
// float32, and each thread forms two (sequence, feature) partial dot products in float32
// (two accumulator chains each).  After a cluster barrier CTA r < 4
// sums sequence r's eight partials over distributed shared memory, rounds the sum to the
// 16-bit type (the Linear's output type), applies LayerNorm (float32, biased variance,
// eps, affine) and RoPE on the first rope_dim features (float32, non-interleaved halves),
// and stores the row with one final rounding.  A second cluster barrier keeps every CTA's
// shared memory alive until the readers are done.  With programmatic dependent launch the
// first W_k chunk streams in before the wait on the previous kernel (W_k is a constant).
//
// Bytes per launch: W_k once from HBM (128 x hidden x 2; the clusters after the first read
// it from L2), hidden B x hidden x 2, and B x 256 bytes of cache rows.  The op is latency
// bound at decode sizes (one launch, two cluster barriers).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace tdsa {

namespace {

constexpr int kKaThreads = 256;
constexpr int kKaCluster = 8;    // CTAs per cluster: the hidden dimension splits 8 ways
constexpr int kKaSeqs = 4;       // sequences per cluster
constexpr int kKaChunk = 256;    // hidden elements staged per pass
constexpr int kKaRowPad = 8;     // 16-bit elements of padding per staged W_k row
constexpr int kKaRow = kKaChunk + kKaRowPad;
constexpr int kKaSmem =
    kHeadDim * kKaRow * 2 + kKaSeqs * kKaChunk * 4 + kKaSeqs * kHeadDim * 4 + kHeadDim * 4 + 64;

struct KeyAppendArgs {
  const uint16_t* hidden;
  int64_t hidden_stride;
  int hidden_size;
  const uint16_t* wk;
  int64_t wk_stride;
  const float* ln_w;
  const float* ln_b;
  float eps;
  const int64_t* positions;
  const int64_t* slots;
  uint16_t* cache;
  int64_t cache_bs;
  int64_t cache_rs;
  int64_t cache_rows;
  int batch;
  int rope_dim;
  float theta;
  int* status;
};

template <bool kBF16>
__device__ __forceinline__ float lo16(uint32_t p) {
  if (kBF16) return __uint_as_float(p << 16);
  return __half2float(__ushort_as_half(static_cast<uint16_t>(p & 0xFFFFu)));
}
template <bool kBF16>
__device__ __forceinline__ float hi16(uint32_t p) {
  if (kBF16) return __uint_as_float(p & 0xFFFF0000u);
  return __half2float(__ushort_as_half(static_cast<uint16_t>(p >> 16)));
}
template <bool kBF16>
__device__ __forceinline__ float to16(float x, uint16_t* bits) {
  if (kBF16) {
    const __nv_bfloat16 v = __float2bfloat16_rn(x);
    *bits = __bfloat16_as_ushort(v);
    return __bfloat162float(v);
  }
  const __half v = __float2half_rn(x);
  *bits = __half_as_ushort(v);
  return __half2float(v);
}

// sum of v over the 128 finishing threads (warps 0..3); red holds 4 floats
__device__ __forceinline__ float sum128(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  __syncwarp();
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const float s = (red[0] + red[1]) + (red[2] + red[3]);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  return s;
}

template <bool kBF16>
__global__ void __cluster_dims__(kKaCluster, 1, 1) __launch_bounds__(kKaThreads, 1)
    key_append_kernel(const KeyAppendArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* sw = reinterpret_cast<uint16_t*>(smem);                       // [128][kKaRow]
  float* sh = reinterpret_cast<float*>(smem + kHeadDim * kKaRow * 2);     // [4][kKaChunk]
  float* part = sh + kKaSeqs * kKaChunk;                                  // [4][128]
  float* yrow = part + kKaSeqs * kHeadDim;                                // [128]
  float* red = yrow + kHeadDim;                                           // [4]

  const uint32_t rank = cluster_ctarank();
  const int cluster = static_cast<int>(blockIdx.x) / kKaCluster;
  const int b0 = cluster * kKaSeqs;
  const int tid = threadIdx.x;
  const int H = a.hidden_size;
  // this CTA's hidden range [k0, k1): eighths rounded up to 8 elements (16 bytes)
  const int per = ((H + kKaCluster - 1) / kKaCluster + 7) & ~7;
  const int k0 = min(H, static_cast<int>(rank) * per);
  const int k1 = min(H, k0 + per);

  const int j = tid & (kHeadDim - 1);  // output feature
  const int sp = (tid >> 7) * 2;       // first of this thread's two sequences
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;  // seq sp: 0, 2; seq sp+1: 1, 3
  // W_k slice of a chunk: row f, vector v -> 16 bytes; consecutive threads take consecutive
  // vectors, all copies in flight at once (cp.async), waited for before the compute barrier
  auto stage_wk = [&](int c0, int vecs) {
    for (int i = tid; i < kHeadDim * vecs; i += kKaThreads) {
      const int f = i / vecs, v = i - f * vecs;
      cp_async16(sw + f * kKaRow + v * 8, a.wk + f * a.wk_stride + c0 + v * 8);
    }
  };
  // W_k is a constant input that no kernel of this library writes: its first chunk is
  // fetched while the previous kernel on the stream finishes; the hidden states (which
  // that kernel may produce) are read only after the dependency wait
  if (k0 < k1) stage_wk(k0, min(kKaChunk, k1 - k0) >> 3);
  pdl_wait();
  for (int c0 = k0; c0 < k1; c0 += kKaChunk) {
    const int n = min(kKaChunk, k1 - c0);  // a multiple of 8
    const int vecs = n >> 3;               // 16-byte vectors per row
    if (c0 != k0) stage_wk(c0, vecs);
    for (int i = tid; i < kKaSeqs * vecs; i += kKaThreads) {
      const int s = i / vecs, v = i - s * vecs;
      const int b = b0 + s;
      float* dst = sh + s * kKaChunk + v * 8;
      if (b < a.batch) {
        const uint4 x =
            *reinterpret_cast<const uint4*>(a.hidden + b * a.hidden_stride + c0 + v * 8);
        dst[0] = lo16<kBF16>(x.x), dst[1] = hi16<kBF16>(x.x);
        dst[2] = lo16<kBF16>(x.y), dst[3] = hi16<kBF16>(x.y);
        dst[4] = lo16<kBF16>(x.z), dst[5] = hi16<kBF16>(x.z);
        dst[6] = lo16<kBF16>(x.w), dst[7] = hi16<kBF16>(x.w);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e] = 0.f;
      }
    }
    cp_async_wait_all();
    __syncthreads();
    const uint16_t* wr = sw + j * kKaRow;
    const float* h0 = sh + sp * kKaChunk;
    const float* h1 = h0 + kKaChunk;
#pragma unroll 4
    for (int v = 0; v < vecs; ++v) {
      const uint4 x = *reinterpret_cast<const uint4*>(wr + v * 8);
      const float4 p0 = *reinterpret_cast<const float4*>(h0 + v * 8);
      const float4 p1 = *reinterpret_cast<const float4*>(h0 + v * 8 + 4);
      const float4 q0 = *reinterpret_cast<const float4*>(h1 + v * 8);
      const float4 q1 = *reinterpret_cast<const float4*>(h1 + v * 8 + 4);
      const float w0 = lo16<kBF16>(x.x), w1 = hi16<kBF16>(x.x), w2 = lo16<kBF16>(x.y),
                  w3 = hi16<kBF16>(x.y), w4 = lo16<kBF16>(x.z), w5 = hi16<kBF16>(x.z),
                  w6 = lo16<kBF16>(x.w), w7 = hi16<kBF16>(x.w);
      acc0 = fmaf(w0, p0.x, acc0), acc0 = fmaf(w1, p0.y, acc0);
      acc0 = fmaf(w2, p0.z, acc0), acc0 = fmaf(w3, p0.w, acc0);
      acc2 = fmaf(w4, p1.x, acc2), acc2 = fmaf(w5, p1.y, acc2);
      acc2 = fmaf(w6, p1.z, acc2), acc2 = fmaf(w7, p1.w, acc2);
      acc1 = fmaf(w0, q0.x, acc1), acc1 = fmaf(w1, q0.y, acc1);
      acc1 = fmaf(w2, q0.z, acc1), acc1 = fmaf(w3, q0.w, acc1);
      acc3 = fmaf(w4, q1.x, acc3), acc3 = fmaf(w5, q1.y, acc3);
      acc3 = fmaf(w6, q1.z, acc3), acc3 = fmaf(w7, q1.w, acc3);
    }
    __syncthreads();
  }
  part[sp * kHeadDim + j] = acc0 + acc2;
  part[(sp + 1) * kHeadDim + j] = acc1 + acc3;
  pdl_launch_dependents();
  cluster_sync_all();  // every CTA's partials are visible cluster-wide

  const int b = b0 + static_cast<int>(rank);
  if (rank < kKaSeqs && b < a.batch && tid < kHeadDim) {
    // the eight partials of feature j of sequence `rank`, in rank order
    const uint32_t local = smem_u32(part + rank * kHeadDim + j);
    float sum = 0.f;
#pragma unroll
    for (uint32_t c = 0; c < kKaCluster; ++c) {
      float v;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(mapa_shared(local, c)));
      sum += v;
    }
    uint16_t bits;
    const float x = to16<kBF16>(sum, &bits);  // the Linear's 16-bit output
    const float mean = sum128(x, red) * (1.f / kHeadDim);
    const float d = x - mean;
    const float var = sum128(d * d, red) * (1.f / kHeadDim);
    float y = d * rsqrtf(var + a.eps);
    y = y * (a.ln_w ? a.ln_w[j] : 1.f) + (a.ln_b ? a.ln_b[j] : 0.f);
    yrow[j] = y;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const int half = a.rope_dim >> 1;
    float out = y;
    if (j < a.rope_dim) {
      const int jj = j < half ? j : j - half;
      const float inv_freq = powf(a.theta, -static_cast<float>(jj) / static_cast<float>(half));
      const float ang = static_cast<float>(a.positions[b]) * inv_freq;
      // reduce the float32 angle by 2*pi in double precision, then the hardware cos/sin
      const double m = rint(static_cast<double>(ang) * 0.15915494309189535);
      const float r = static_cast<float>(fma(-m, 6.283185307179586, static_cast<double>(ang)));
      const float cs = __cosf(r), sn = __sinf(r);
      out = j < half ? y * cs - yrow[j + half] * sn : y * cs + yrow[j - half] * sn;
    }
    const int64_t slot = a.slots ? a.slots[b] : a.positions[b];
    if (slot >= 0 && slot < a.cache_rows) {
      to16<kBF16>(out, &bits);
      a.cache[b * a.cache_bs + slot * a.cache_rs + j] = bits;
    } else if (j == 0) {
      atomicOr(a.status, TDSA_STATUS_RANGE);
    }
  }
  cluster_sync_all();  // no CTA leaves while a peer may still read its partials
}

}  // namespace

int launch_key_append(const void* hidden, int64_t hidden_stride, int hidden_size,
                      const void* wk, int64_t wk_stride, const float* ln_w, const float* ln_b,
                      float eps, const int64_t* positions, const int64_t* slots, void* cache,
                      int64_t cache_bs, int64_t cache_rs, int64_t cache_rows, int dtype,
                      int batch, int rope_dim, float theta, int* status, cudaStream_t stream) {
  KeyAppendArgs a;
  a.hidden = static_cast<const uint16_t*>(hidden);
  a.hidden_stride = hidden_stride;
  a.hidden_size = hidden_size;
  a.wk = static_cast<const uint16_t*>(wk);
  a.wk_stride = wk_stride;
  a.ln_w = ln_w;
  a.ln_b = ln_b;
  a.eps = eps;
  a.positions = positions;
  a.slots = slots;
  a.cache = static_cast<uint16_t*>(cache);
  a.cache_bs = cache_bs;
  a.cache_rs = cache_rs;
  a.cache_rows = cache_rows;
  a.batch = batch;
  a.rope_dim = rope_dim;
  a.theta = theta;
  a.status = status;
  const int clusters = (batch + kKaSeqs - 1) / kKaSeqs;
  auto kern = dtype == TDSA_BF16 ? key_append_kernel<true> : key_append_kernel<false>;
  TDSA_CUDA_CHECK(
      ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kKaSmem));
  TDSA_CUDA_CHECK(launch_pdl(kern, dim3(static_cast<unsigned>(clusters * kKaCluster)),
                             dim3(kKaThreads), kKaSmem, stream, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
