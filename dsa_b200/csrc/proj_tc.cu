// Fused decode-step query projection of the indexer sidecar (reference sidecar.py:78-87)
// on the sm_100a tensor cores, one launch:
//
//   qraw[b, h*128 + d] = 16-bit( sum_k x[b,k] * W_q[h*128 + d, k] )      (nn.Linear output)
//   q[b, h, :]         = RoPE_noninterleaved(qraw[b, h*128 : h*128+128]) on the first
//                        rope_dim dims (float32 math, one rounding), others unchanged
//   w[b, h]            = scale * sum_k float(x[b,k]) * W_w[h,k]          (float32 GEMV)
//
// CTA (h, g) owns head h's 128 output features for the batch rows [g*N, g*N + N).  The
// W_q GEMM is D[128 features x N rows] = W_q[128 x K] . x[N x K]^T: UMMA M=128, N = 64/128/
// 256, K streamed in 64-element chunks (one 128-byte swizzle row) through a TMA ring; the
// accumulator lives in TMEM.  Every W_q byte is read once from HBM (the roofline: 16 MiB
// per 64 heads x 2048 hidden), x comes from L2.  Warp roles:
//   warp 0      TMA producer: W_q tile [128 x 64] and x tile [N x 64] per stage
//   warp 1      tcgen05 issuer: 4 x K16 UMMAs per stage, then one commit for the epilogue
//   warps 2..5  while the GEMM streams: the float32 head-weight GEMV for head h, reading
//               the same x tiles and the head's W_w slice (a third TMA box per stage) out of
//               shared memory (they release each stage with the MMA); afterwards: TMEM -> registers, 16-bit rounding, RoPE with the partner
//               dimension exchanged through shared memory, stores.
// Every wait is bounded (TDSA_ERR_TIMEOUT in the device status word on expiry).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "timeline.cuh"

namespace tdsa {

// (outside the unnamed namespace: the timeline readers keep external C linkage)
// timeline builds, per CTA: 0 entry, 1 past the dependency wait (thread 0); 2 first stage
// landed, 3 first refilled stage landed, 4 last MMA issued (MMA thread); 5 GEMM complete,
// 6 peer's partial sums received (first epilogue thread); 7 exit (thread 0)
TDSA_TL_DECL(proj, 128, 8)

namespace {

constexpr int kThreads = 192;
constexpr int kKChunk = 64;                        // hidden elements per stage
constexpr int kWTileBytes = 128 * kKChunk * 2;     // 16 KiB
constexpr int kRingBytes = 192 * 1024;             // stage ring budget
constexpr int kWwChunkBytes = kKChunk * 4;       // the head's W_w slice per stage (f32)
constexpr int kBarrierBytes = 2048;  // barriers, then positions [kN] and frequencies [64]

struct ProjArgs {
  const float* ww;          // [64][hidden] float32
  int hidden;
  const int64_t* positions; // [batch]
  void* q;                  // [batch][q_stride] 16-bit
  int64_t q_stride;
  float* w;                 // [batch][w_stride]
  int64_t w_stride;
  void* qraw;               // optional [batch][qraw_stride] 16-bit pre-RoPE output
  int64_t qraw_stride;
  int batch;
  int rope_dim;
  float theta;
  float scale;
  int packed;               // W_q in the packed tile layout (see pack_wq_kernel)
  int* status;
};

// Row coordinate of W_q tile (head h, K chunk kc) in the tensor map: natural layout
// [8192][hidden] (x coordinate kc * 64) or packed [64 heads][nk][128][64] (x = 0).
__device__ __forceinline__ void wq_coords(const ProjArgs& a, int h, int kc, int nk, int& x,
                                          int& y) {
  if (a.packed) {
    x = 0;
    y = (h * nk + kc) * 128;
  } else {
    x = kc * 64;
    y = h * 128;
  }
}

template <int kN>
constexpr int stage_bytes() {
  return kWTileBytes + kN * kKChunk * 2;
}

template <int kN>
constexpr int ring_stages() {
  return kRingBytes / stage_bytes<kN>() > 8 ? 8 : kRingBytes / stage_bytes<kN>();
}

template <int kN>
constexpr int smem_bytes() {
  return ring_stages<kN>() * (stage_bytes<kN>() + kWwChunkBytes) + kBarrierBytes + 1024;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <bool kBF16>
__device__ __forceinline__ float round16(float x) {
  if (kBF16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}

template <bool kBF16>
__device__ __forceinline__ void store16(void* base, int64_t off, float x) {
  if (kBF16)
    static_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(x);
  else
    static_cast<__half*>(base)[off] = __float2half_rn(x);
}

template <bool kBF16>
__device__ __forceinline__ float elem16(uint32_t packed, int hi) {
  const uint16_t bits = static_cast<uint16_t>(hi ? packed >> 16 : packed & 0xFFFFu);
  if (kBF16) return __uint_as_float(static_cast<uint32_t>(bits) << 16);
  return __half2float(__ushort_as_half(bits));
}

__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
}

// Barrier of the four epilogue warps that also ANDs a predicate over them.
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(out)
      : "r"(v ? 1u : 0u)
      : "memory");
  return out != 0u;
}

// Grid: blockIdx.x < 64 -- GEMM CTA of head blockIdx.x (W_q tiles + x tiles, tcgen05,
// RoPE epilogue); blockIdx.x >= 64 -- GEMV CTA of head blockIdx.x - 64 (x tiles + the
// head's W_w slice, float32 dot products on the four epilogue warps).  Both kinds stream
// the same x tiles through the same ring; the GEMV runs on otherwise idle SMs alongside.
template <bool kBF16, int kN>
__global__ void __launch_bounds__(kThreads, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                   const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap wwmap, const ProjArgs a) {
  constexpr int kStages = ring_stages<kN>();
  constexpr int kStage = stage_bytes<kN>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  float* ww_ring = reinterpret_cast<float*>(smem + kStages * kStage);  // [stages][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * (kStage + kWwChunkBytes));
  uint64_t* empty = full + kStages;
  uint64_t* accfull = empty + kStages;
  uint64_t* done = accfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* spos = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // [kN]
  float* sinv = spos + kN;                                                         // [64]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool gemm = blockIdx.x < kHeads;
  const int h = gemm ? blockIdx.x : blockIdx.x - kHeads;
  const int b0 = blockIdx.y * kN;
  const int nk = (a.hidden + kKChunk - 1) / kKChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], gemm ? 1 : 4);  // the MMA commit, or one arrival per GEMV warp
    }
    mbar_init(accfull, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(gemm ? &wmap : &wwmap);
    prefetch_tmap(&xmap);
  }
  if (gemm && warp == 1) {
    tmem_alloc(tmem_holder, kN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = gemm ? *tmem_holder : 0u;
  pdl_wait();  // hidden states and positions may come from the previous kernel
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const uint64_t pol_w = policy_evict_first();  // W_q: read once
      const uint64_t pol_x = policy_evict_last();   // x and W_w: read by many CTAs
      const uint32_t bytes = gemm ? kStage : kStage - kWTileBytes + kWwChunkBytes;
      int kc = 0;
      for (; kc < nk; ++kc) {
        const int s = kc % kStages;
        const uint32_t ph = (kc / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
        uint8_t* dst = smem + s * kStage;
        mbar_arrive_expect_tx(&full[s], bytes);
        if (gemm) {
          int wx, wy;
          wq_coords(a, h, kc, nk, wx, wy);
          tma_load_2d(dst, &wmap, &full[s], wx, wy, pol_w);
        } else {
          tma_load_2d(ww_ring + s * kKChunk, &wwmap, &full[s], kc * kKChunk, h, pol_x);
        }
        tma_load_2d(dst + kWTileBytes, &xmap, &full[s], kc * kKChunk, b0, pol_x);
      }
      // let every issued copy land before the CTA can exit (bounded, abort or not)
      volatile int no_abort = 0;
      for (int s = 0; s < kStages && s < kc; ++s) {
        const int n = (kc - s + kStages - 1) / kStages;
        mbar_wait(&full[s], (n - 1) & 1u, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (gemm && lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = umma_idesc_f16(kBF16, 128, kN);
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % kStages;
        if (!mbar_wait(&full[s], (kc / kStages) & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t w_addr = smem_u32(smem + s * kStage);
        const uint32_t x_addr = w_addr + kWTileBytes;
#pragma unroll
        for (int k = 0; k < kKChunk / 16; ++k) {
          umma_f16(tmem_base, sw128_kmajor_desc(w_addr + k * 32),
                   sw128_kmajor_desc(x_addr + k * 32), idesc, (kc | k) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accfull);
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort);
    }
  } else if (!gemm) {
    // ------------------------------------------------------ GEMV CTA: epilogue warps
    // w[b, h] = scale * sum_k float(x[b,k]) W_w[h,k].  Per stage the x tile holds kN rows x
    // 8 chunks of 8 elements; thread et takes chunks et + 128 i (i < kN / 16): row
    // (et + 128 i) / 8, chunk et % 8 -- eight consecutive threads read one 128-byte row.
    const int et = threadIdx.x - 64;  // 0..127
    constexpr int kPer = kN / 16;
    const int c = et & 7;
    float part[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) part[i] = 0.f;
    bool ok = true;
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % kStages;
      if (!mbar_wait(&full[s], (kc / kStages) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      // the head's W_w slice came with the stage (zero past the hidden size)
      const float4 wa = *reinterpret_cast<const float4*>(ww_ring + s * kKChunk + c * 8);
      const float4 wb = *reinterpret_cast<const float4*>(ww_ring + s * kKChunk + c * 8 + 4);
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint8_t* xt = smem + s * kStage + kWTileBytes;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int r = (et + 128 * i) >> 3;
        const uint4 v = *reinterpret_cast<const uint4*>(
            xt + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        float acc = part[i];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(elem16<kBF16>(u[j >> 1], j & 1), wv[j], acc);
        part[i] = acc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        float v = part[i];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        const int b = b0 + ((et + 128 * i) >> 3);
        if (c == 0 && b < a.batch) a.w[static_cast<int64_t>(b) * a.w_stride + h] = v * a.scale;
      }
    }
  } else {
    // ------------------------------------------------ GEMM CTA: epilogue warps (RoPE)
    const int et = threadIdx.x - 64;  // 0..127
    const int half = a.rope_dim >> 1;
    // while the GEMM streams: the tile's positions and the RoPE frequencies
    for (int i = et; i < kN; i += 128)
      spos[i] = static_cast<float>(a.positions[min(b0 + i, a.batch - 1)]);
    if (et < half) sinv[et] = powf(a.theta, -static_cast<float>(et) / static_cast<float>(half));
    const uint32_t quad = static_cast<uint32_t>(warp & 3);
    const int d = static_cast<int>(quad) * 32 + lane;  // this thread's feature (TMEM lane)
    const bool rot = d < a.rope_dim;
    const int j = d < half ? d : d - half;  // frequency index of this dim's rotation pair
    const int partner = d < half ? d + half : d - half;
    // The ring is idle once the GEMM is done: exchange rows [128][36], the cos/sin tables
    // [64 j][kN + 4] (row strides keep 16-byte reads on distinct banks), and the 16-bit
    // output staging [32 rows][128 dims].
    constexpr int kTabStride = kN + 4;
    float* ex = reinterpret_cast<float*>(smem);
    float* tcos = ex + 128 * 36;
    float* tsin = tcos + 64 * kTabStride;
    uint16_t* ostage = reinterpret_cast<uint16_t*>(tsin + 64 * kTabStride);
    const bool ok = mbar_wait(accfull, 0, abort_flag);
    // all epilogue threads agree (and have finished with the ring) before it is reused
    if (epi_all(ok && !*abort_flag)) {
      // angle = position * theta^(-j/half) rounded to float32, as the reference computes
      // it; cos/sin of that float: the angle (|angle| < 2^24) is reduced by 2*pi in double
      // precision (the product n * 2pi and the subtraction are exact to ~2^-53 relative),
      // then the hardware sin/cos approximations take the reduced |r| <= pi (absolute error
      // ~2^-21, far below the 16-bit rounding of q that follows).
      for (int i = et; i < kN * half; i += 128) {
        const int col = i / half, jj = i - col * half;
        const float ang = spos[col] * sinv[jj];
        const double n = rint(static_cast<double>(ang) * 0.15915494309189535);
        const float r = static_cast<float>(fma(-n, 6.283185307179586, static_cast<double>(ang)));
        tcos[jj * kTabStride + col] = __cosf(r);
        tsin[jj * kTabStride + col] = __sinf(r);
      }
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < kN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((quad * 32u) << 16) + c0, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int t = 0; t < 32; t += 4) {
          float4 f;
          f.x = v[t] = round16<kBF16>(__uint_as_float(r[t]));
          f.y = v[t + 1] = round16<kBF16>(__uint_as_float(r[t + 1]));
          f.z = v[t + 2] = round16<kBF16>(__uint_as_float(r[t + 2]));
          f.w = v[t + 3] = round16<kBF16>(__uint_as_float(r[t + 3]));
          *reinterpret_cast<float4*>(ex + d * 36 + t) = f;
        }
        epi_barrier();  // (the first one also publishes the cos/sin tables)
        for (int pass = 0; pass < (a.qraw ? 2 : 1); ++pass) {
#pragma unroll
          for (int t = 0; t < 32; t += 4) {
            float o[4] = {v[t], v[t + 1], v[t + 2], v[t + 3]};
            if (rot && pass == 0) {
              const float4 ot = *reinterpret_cast<const float4*>(ex + partner * 36 + t);
              const float4 cs = *reinterpret_cast<const float4*>(tcos + j * kTabStride + c0 + t);
              const float4 sn = *reinterpret_cast<const float4*>(tsin + j * kTabStride + c0 + t);
              const float oo[4] = {ot.x, ot.y, ot.z, ot.w};
              const float cc[4] = {cs.x, cs.y, cs.z, cs.w};
              const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
                o[u] = d < half ? o[u] * cc[u] - oo[u] * ss[u] : o[u] * cc[u] + oo[u] * ss[u];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float y = o[u];
              ostage[(t + u) * 128 + d] =
                  kBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(y))
                        : __half_as_ushort(__float2half_rn(y));
            }
          }
          epi_barrier();
          // 32 rows x 256 bytes, 16 bytes per thread per row group: coalesced stores
          void* dst = pass == 0 ? a.q : a.qraw;
          const int64_t stride = pass == 0 ? a.q_stride : a.qraw_stride;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int row = g * 8 + (et >> 4), ch = et & 15;
            const int b = b0 + c0 + row;
            if (b < a.batch) {
              const uint4 val = *reinterpret_cast<const uint4*>(ostage + row * 128 + ch * 8);
              *reinterpret_cast<uint4*>(static_cast<uint16_t*>(dst) + b * stride + h * 128 +
                                        ch * 8) = val;
            }
          }
          epi_barrier();
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (gemm && warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kN);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
}

// cos/sin of angle = position * theta^(-j/half), rounded to float32 as the reference computes
// it.  The angle (|angle| < 2^24) is reduced by 2*pi in double precision (the product
// n * 2pi and the subtraction are exact to ~2^-53 relative), then the hardware sin/cos
// approximations take the reduced |r| <= pi (absolute error ~2^-21, far below the 16-bit
// rounding of q that follows).  Table layout [j][col], row stride `stride`; run by the
// 128 epilogue threads.
__device__ __forceinline__ void build_rope_table(const float* spos, const float* sinv, int half,
                                                 int ncols, int stride, float* tcos,
                                                 float* tsin) {
  const int et = threadIdx.x - 64;
  for (int i = et; i < ncols * half; i += 128) {
    const int col = i / half, jj = i - col * half;
    const float ang = spos[col] * sinv[jj];
    const double n = rint(static_cast<double>(ang) * 0.15915494309189535);
    const float r = static_cast<float>(fma(-n, 6.283185307179586, static_cast<double>(ang)));
    tcos[jj * stride + col] = __cosf(r);
    tsin[jj * stride + col] = __sinf(r);
  }
}

// ---------------------------------------------------------------------------------
// Batches of at most 64 rows: split-K over a cluster of two CTAs per head, so 128 SMs
// stream W_q.  CTA rank r runs the GEMM and the W_w GEMV over its half of the hidden
// dimension, then the pair splits the epilogue by batch column: each rank ships the
// peer's 32 columns of its TMEM partial sums (and the peer's GEMV row sums) with one DSMEM
// bulk copy into the peer's receive region, adds what it received to its own half, and
// runs the RoPE epilogue and stores for that half.
constexpr int kSplitN = 64;
constexpr int kSplitStages = 7;
constexpr int kSplitStage = kWTileBytes + kSplitN * kKChunk * 2;  // 24 KiB
constexpr int kRecvStride = 36;  // floats per received row (16-byte reads on distinct banks)
constexpr int kEarlyTabBytes = 2 * 32 * (kSplitN + 4) * 4;  // cos/sin table, rope_dim <= 64
// the peer's partial sums for this rank's 32 columns [128][36] f32, then its 32 GEMV row
// sums of this rank's rows
constexpr int kRecvBytes = (128 * kRecvStride + kSplitN / 2) * 4;
constexpr int kSplitSmem = kSplitStages * (kSplitStage + kWwChunkBytes) + kBarrierBytes +
                           kEarlyTabBytes + kRecvBytes + 1024;

template <bool kBF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    proj_splitk_kernel(const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wwmap, const ProjArgs a) {
  constexpr int kN = kSplitN;
  constexpr int kStages = kSplitStages;
  constexpr int kStage = kSplitStage;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  float* ww_ring = reinterpret_cast<float*>(smem + kStages * kStage);  // [stages][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * (kStage + kWwChunkBytes));
  uint64_t* empty = full + kStages;
  uint64_t* accfull = empty + kStages;
  uint64_t* done = accfull + 1;
  uint64_t* recv = done + 1;  // the peer's partials have landed (bulk copy tx)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(recv + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* spos = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // [64]
  float* sinv = spos + kN;                                                         // [64]
  // the peer's partials for this rank's columns (its own region, so the peer ships them as
  // soon as its GEMM is done); each rank stages what it sends in its own ring
  float* recv_buf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + kBarrierBytes +
                                             kEarlyTabBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int h = blockIdx.x >> 1;
  const int nk = (a.hidden + kKChunk - 1) / kKChunk;
  const int split = (nk + 1) >> 1;
  const int kbeg = rank ? split : 0, kend = rank ? nk : split;
  const int nloc = kend - kbeg;
  __shared__ unsigned int tl_launch;

  if (threadIdx.x == 0) {
    tl_launch = TDSA_TL_TICKET(proj);
    TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 0);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);  // the MMA commit + one arrival per epilogue warp
    }
    mbar_init(accfull, 1);
    mbar_init(done, 1);
    mbar_init(recv, 1);
    mbar_arrive_expect_tx(recv, kRecvBytes);  // completes when the peer's copy has landed
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
    prefetch_tmap(&wwmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // W_q and W_w are constant inputs, so they need not wait for the previous kernel: the
  // first ring stages' weight tiles load now, and the rest of this CTA's W_q tiles -- plus,
  // for the CTAs of heads 0..31, those of head h + 32, whose CTAs start late when the
  // previous kernel still holds SMs -- are prefetched into L2 while that kernel finishes.
  const int pre = nloc < kStages ? nloc : kStages;
  if (warp == 0 && lane == 0) {
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    for (int it = 0; it < pre; ++it) {
      const int kc = kbeg + it;
      mbar_arrive_expect_tx(&full[it], kStage + kWwChunkBytes);
      int wx, wy;
      wq_coords(a, h, kc, nk, wx, wy);
      tma_load_2d(smem + it * kStage, &wmap, &full[it], wx, wy, pol_w);
      tma_load_2d(ww_ring + it * kKChunk, &wwmap, &full[it], kc * kKChunk, h, pol_x);
    }
    for (int kc = kbeg + pre; kc < kend; ++kc) {
      int wx, wy;
      wq_coords(a, h, kc, nk, wx, wy);
      tma_prefetch_l2_2d(&wmap, wx, wy);
    }
    if (h < kHeads / 2)
      for (int kc = kbeg; kc < kend; ++kc) {
        int wx, wy;
        wq_coords(a, h + kHeads / 2, kc, nk, wx, wy);
        tma_prefetch_l2_2d(&wmap, wx, wy);
      }
  }
  // the RoPE frequencies depend on the arguments only
  if (threadIdx.x >= 64 && threadIdx.x - 64 < (a.rope_dim >> 1)) {
    const int jj = threadIdx.x - 64, hf = a.rope_dim >> 1;
    sinv[jj] = powf(a.theta, -static_cast<float>(jj) / static_cast<float>(hf));
  }
  pdl_wait();  // hidden states and positions may come from the previous kernel
  if (threadIdx.x == 0) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 1);
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int it = 0;
      for (; it < nloc; ++it) {
        const int s = it % kStages;
        const int kc = kbeg + it;
        uint8_t* dst = smem + s * kStage;
        if (it < pre) {  // the weights of this stage are already on their way
          tma_load_2d(dst + kWTileBytes, &xmap, &full[s], kc * kKChunk, 0, pol_x);
          continue;
        }
        if (!mbar_wait(&empty[s], ((it / kStages) & 1u) ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], kStage + kWwChunkBytes);
        int wx, wy;
        wq_coords(a, h, kc, nk, wx, wy);
        tma_load_2d(dst, &wmap, &full[s], wx, wy, pol_w);
        tma_load_2d(dst + kWTileBytes, &xmap, &full[s], kc * kKChunk, 0, pol_x);
        tma_load_2d(ww_ring + s * kKChunk, &wwmap, &full[s], kc * kKChunk, h, pol_x);
      }
      volatile int no_abort = 0;
      for (int s = 0; s < kStages && s < it; ++s) {
        const int n = (it - s + kStages - 1) / kStages;
        mbar_wait(&full[s], (n - 1) & 1u, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = umma_idesc_f16(kBF16, 128, kN);
      for (int it = 0; it < nloc; ++it) {
        const int s = it % kStages;
        if (!mbar_wait(&full[s], (it / kStages) & 1u, abort_flag)) break;
        if (it == 0) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 2);
        if (it == pre) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 3);
        tc_fence_after();
        const uint32_t w_addr = smem_u32(smem + s * kStage);
        const uint32_t x_addr = w_addr + kWTileBytes;
#pragma unroll
        for (int k = 0; k < kKChunk / 16; ++k) {
          umma_f16(tmem_base, sw128_kmajor_desc(w_addr + k * 32),
                   sw128_kmajor_desc(x_addr + k * 32), idesc, (it | k) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 4);
      umma_commit(accfull);
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort);
    }
  } else {
    // -------------------------------------------------------------- epilogue warps
    const int et = threadIdx.x - 64;  // 0..127
    const int half = a.rope_dim >> 1;
    constexpr int kTabStride = kN + 4;
    // rope_dim <= 64: the cos/sin table has its own region and is built right after the
    // GEMV (while the last MMAs run); larger rope_dim builds it in the ring after the GEMM
    const bool early = half <= 32;
    float* etab = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + kBarrierBytes);
    // this thread's position (kN <= 128): the load is consumed after the GEMV, so its
    // latency hides behind it
    static_assert(kN <= 128, "one position per epilogue thread");
    const int64_t my_pos = et < kN ? a.positions[min(et, a.batch - 1)] : 0;
    // (1) the W_w GEMV over this CTA's half of the hidden dimension (layout as above), started
    // as soon as the first stage lands: the ring's stages are released by these warps too
    constexpr int kPer = kN / 16;
    const int c = et & 7;
    float part[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) part[i] = 0.f;
    bool ok = true;
    for (int it = 0; it < nloc; ++it) {
      const int s = it % kStages;
      if (!mbar_wait(&full[s], (it / kStages) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      const float4 wa = *reinterpret_cast<const float4*>(ww_ring + s * kKChunk + c * 8);
      const float4 wb = *reinterpret_cast<const float4*>(ww_ring + s * kKChunk + c * 8 + 4);
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint8_t* xt = smem + s * kStage + kWTileBytes;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int r = (et + 128 * i) >> 3;
        const uint4 v = *reinterpret_cast<const uint4*>(
            xt + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        float acc = part[i];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(elem16<kBF16>(u[j >> 1], j & 1), wv[j], acc);
        part[i] = acc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      float v = part[i];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      part[i] = v;  // the row sum (over this CTA's half) in the lanes with c == 0
    }
    // the positions, then (rope_dim <= 64) the cos/sin table in its own region, while the
    // last MMAs finish
    if (et < kN) spos[et] = static_cast<float>(my_pos);
    epi_barrier();
    if (early) build_rope_table(spos, sinv, half, kN, kTabStride, etab, etab + 32 * kTabStride);
    const uint32_t quad = static_cast<uint32_t>(warp & 3);
    const int d = static_cast<int>(quad) * 32 + lane;  // this thread's feature (TMEM lane)
    // (2) the pair shares the epilogue: rank r finishes batch columns [32r, 32r + 32).
    // Each rank stages the OTHER half of its partial sums (TMEM columns) and the GEMV row
    // sums of the other half's rows in its own ring (idle after its GEMM), and one bulk
    // copy moves them into the peer's receive region, completing on the peer's mbarrier.
    constexpr int kHalf = kN / 2;
    const int my0 = static_cast<int>(rank) * kHalf, peer0 = kHalf - my0;
    // every epilogue warp is past its last read of the ring (the GEMV) before the ring is
    // reused for staging; the MMA commit alone does not order those reads
    ok = epi_all(ok) && mbar_wait(accfull, 0, abort_flag);
    if (et == 0) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 5);
    float* stage = reinterpret_cast<float*>(smem);
    if (ok) {
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem_base + ((quad * 32u) << 16) + peer0, r);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 32; t += 4) {
        float4 f;
        f.x = __uint_as_float(r[t]);
        f.y = __uint_as_float(r[t + 1]);
        f.z = __uint_as_float(r[t + 2]);
        f.w = __uint_as_float(r[t + 3]);
        *reinterpret_cast<float4*>(stage + d * kRecvStride + t) = f;
      }
      tc_fence_before();
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int row = (et + 128 * i) >> 3;
        if (c == 0 && row >= peer0 && row < peer0 + kHalf)
          stage[128 * kRecvStride + row - peer0] = part[i];
      }
    }
    fence_proxy_async_smem();
    if (epi_all(ok && !*abort_flag) && et == 0)
      bulk_copy_to_peer(mapa_shared(smem_u32(recv_buf), rank ^ 1u), stage, kRecvBytes,
                        mapa_shared(smem_u32(recv), rank ^ 1u));
    {
      const bool rot = d < a.rope_dim;
      const int j = d < half ? d : d - half;
      const int partner = d < half ? d + half : d - half;
      // the ring past the outgoing stage: exchange rows, late cos/sin table, output staging
      float* ex = stage + 128 * kRecvStride + kHalf;
      float* tcos = early ? etab : ex + 128 * 36;
      float* tsin = early ? etab + 32 * kTabStride : tcos + 64 * kTabStride;
      uint16_t* ostage = reinterpret_cast<uint16_t*>(ex + 128 * 36 + 128 * kTabStride);
      const bool j_ok = epi_all(ok && !*abort_flag);
      if (j_ok && !early) build_rope_table(spos, sinv, half, kN, kTabStride, tcos, tsin);
      const bool got = j_ok && mbar_wait_cluster(recv, 0, abort_flag);
      if (et == 0) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 6);
      if (epi_all(got && !*abort_flag)) {
        const float* rbuf = recv_buf;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int row = (et + 128 * i) >> 3;
          if (c == 0 && row >= my0 && row < my0 + kHalf && row < a.batch)
            a.w[static_cast<int64_t>(row) * a.w_stride + h] =
                (part[i] + rbuf[128 * kRecvStride + row - my0]) * a.scale;
        }
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem_base + ((quad * 32u) << 16) + my0, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int t = 0; t < 32; t += 4) {
          const float4 o = *reinterpret_cast<const float4*>(rbuf + d * kRecvStride + t);
          float4 f;
          f.x = v[t] = round16<kBF16>(__uint_as_float(r[t]) + o.x);
          f.y = v[t + 1] = round16<kBF16>(__uint_as_float(r[t + 1]) + o.y);
          f.z = v[t + 2] = round16<kBF16>(__uint_as_float(r[t + 2]) + o.z);
          f.w = v[t + 3] = round16<kBF16>(__uint_as_float(r[t + 3]) + o.w);
          *reinterpret_cast<float4*>(ex + d * 36 + t) = f;
        }
        tc_fence_before();
        epi_barrier();
        for (int pass = 0; pass < (a.qraw ? 2 : 1); ++pass) {
#pragma unroll
          for (int t = 0; t < 32; t += 4) {
            float o[4] = {v[t], v[t + 1], v[t + 2], v[t + 3]};
            if (rot && pass == 0) {
              const float4 ot = *reinterpret_cast<const float4*>(ex + partner * 36 + t);
              const float4 cs = *reinterpret_cast<const float4*>(tcos + j * kTabStride + my0 + t);
              const float4 sn = *reinterpret_cast<const float4*>(tsin + j * kTabStride + my0 + t);
              const float oo[4] = {ot.x, ot.y, ot.z, ot.w};
              const float cc[4] = {cs.x, cs.y, cs.z, cs.w};
              const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
                o[u] = d < half ? o[u] * cc[u] - oo[u] * ss[u] : o[u] * cc[u] + oo[u] * ss[u];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
              ostage[(t + u) * 128 + d] = kBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(o[u]))
                                                : __half_as_ushort(__float2half_rn(o[u]));
          }
          epi_barrier();
          void* dst = pass == 0 ? a.q : a.qraw;
          const int64_t stride = pass == 0 ? a.q_stride : a.qraw_stride;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int row = g * 8 + (et >> 4), ch = et & 15;
            const int b = my0 + row;
            if (b < a.batch) {
              const uint4 val = *reinterpret_cast<const uint4*>(ostage + row * 128 + ch * 8);
              *reinterpret_cast<uint4*>(static_cast<uint16_t*>(dst) + b * stride + h * 128 +
                                        ch * 8) = val;
            }
          }
          epi_barrier();
        }
      }
    }
  }

  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its shared memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kN);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
  if (threadIdx.x == 0) TDSA_TL_REC(proj, 128, 8, tl_launch, blockIdx.x, 7);
}

template <bool kBF16>
int launch_proj_splitk(const CUtensorMap& wmap, const CUtensorMap& xmap,
                       const CUtensorMap& wwmap, const ProjArgs& a, cudaStream_t stream) {
  auto kern = proj_splitk_kernel<kBF16>;
  TDSA_CUDA_CHECK(
      ensure_dynamic_smem(reinterpret_cast<const void*>(kern), kSplitSmem));
  TDSA_CUDA_CHECK(launch_pdl(kern, dim3(2 * kHeads), dim3(kThreads), kSplitSmem, stream, wmap,
                             xmap, wwmap, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

template <bool kBF16, int kN>
int launch_proj_t(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& wwmap,
                  const ProjArgs& a, cudaStream_t stream) {
  auto kern = proj_tc_kernel<kBF16, kN>;
  constexpr int smem = smem_bytes<kN>();
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  const dim3 grid(2 * kHeads, (a.batch + kN - 1) / kN);
  TDSA_CUDA_CHECK(launch_pdl(kern, grid, dim3(kThreads), smem, stream, wmap, xmap, wwmap, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace

int launch_query_project(const void* x, int64_t x_stride, int hidden, const void* wq,
                         int64_t wq_stride, int packed, const float* ww,
                         const int64_t* positions, void* q,
                         int64_t q_stride, float* w, int64_t w_stride, int dtype, int batch,
                         int rope_dim, float theta, float scale, void* qraw,
                         int64_t qraw_stride, cudaStream_t stream, int* status) {
  const int n = batch <= 64 ? 64 : batch <= 128 ? 128 : 256;
  const CUtensorMapDataType dt =
      dtype == TDSA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap wmap, xmap, wwmap;
  const int nk = (hidden + kKChunk - 1) / kKChunk;
  {
    // packed: one contiguous 16 KiB block per (head, K chunk) -- whole DRAM pages per tile
    const uint64_t dims[2] = {static_cast<uint64_t>(packed ? kKChunk : hidden),
                              static_cast<uint64_t>(kHeads * 128) * (packed ? nk : 1)};
    const uint64_t strides[1] = {static_cast<uint64_t>(packed ? kKChunk : wq_stride) * 2};
    const uint32_t box[2] = {kKChunk, 128};
    int rc = encode_tmap(&wmap, dt, 2, wq, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(batch)};
    const uint64_t strides[1] = {static_cast<uint64_t>(batch > 1 ? x_stride : hidden) * 2};
    const uint32_t box[2] = {kKChunk, static_cast<uint32_t>(n)};
    int rc = encode_tmap(&xmap, dt, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(hidden), static_cast<uint64_t>(kHeads)};
    const uint64_t strides[1] = {static_cast<uint64_t>(hidden) * 4};
    const uint32_t box[2] = {kKChunk, 1};
    int rc = encode_tmap(&wwmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ww, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  ProjArgs a;
  a.ww = ww;
  a.hidden = hidden;
  a.positions = positions;
  a.q = q;
  a.q_stride = q_stride;
  a.w = w;
  a.w_stride = w_stride;
  a.qraw = qraw;
  a.qraw_stride = qraw_stride;
  a.batch = batch;
  a.rope_dim = rope_dim;
  a.theta = theta;
  a.scale = scale;
  a.packed = packed;
  a.status = status;
  const bool bf16 = dtype == TDSA_BF16;
  if (n == 64 && hidden > kKChunk)
    return bf16 ? launch_proj_splitk<true>(wmap, xmap, wwmap, a, stream)
                : launch_proj_splitk<false>(wmap, xmap, wwmap, a, stream);
  if (n == 64) return bf16 ? launch_proj_t<true, 64>(wmap, xmap, wwmap, a, stream)
                           : launch_proj_t<false, 64>(wmap, xmap, wwmap, a, stream);
  if (n == 128) return bf16 ? launch_proj_t<true, 128>(wmap, xmap, wwmap, a, stream)
                            : launch_proj_t<false, 128>(wmap, xmap, wwmap, a, stream);
  return bf16 ? launch_proj_t<true, 256>(wmap, xmap, wwmap, a, stream)
              : launch_proj_t<false, 256>(wmap, xmap, wwmap, a, stream);
}

namespace {

// W_q [8192][hidden] (row stride `stride`) -> packed [64 heads][nk][128 rows][64]: the
// (head, K chunk) tile the projection streams per stage becomes one contiguous 16 KiB
// block; K past the hidden size is zero.  One thread per 16-byte chunk.
__global__ void pack_wq_kernel(const uint16_t* __restrict__ wq, int64_t stride, int hidden,
                               int nk, uint16_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(kHeads) * 128 * nk * 8;  // 16-byte chunks
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ch = static_cast<int>(i & 7);       // chunk of 8 within the 64-wide row
    const int64_t rest = i >> 3;
    const int r = static_cast<int>(rest % 128);   // row within the head
    const int64_t tile = rest / 128;              // h * nk + kc
    const int kc = static_cast<int>(tile % nk);
    const int h = static_cast<int>(tile / nk);
    const int k0 = kc * 64 + ch * 8;
    const uint16_t* src = wq + static_cast<int64_t>(h * 128 + r) * stride + k0;
    uint16_t v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = k0 + j < hidden ? src[j] : uint16_t(0);
    uint4 o;
    o.x = v[0] | (static_cast<uint32_t>(v[1]) << 16);
    o.y = v[2] | (static_cast<uint32_t>(v[3]) << 16);
    o.z = v[4] | (static_cast<uint32_t>(v[5]) << 16);
    o.w = v[6] | (static_cast<uint32_t>(v[7]) << 16);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

}  // namespace

size_t packed_wq_bytes(int hidden) {
  const size_t nk = static_cast<size_t>((hidden + kKChunk - 1) / kKChunk);
  return static_cast<size_t>(kHeads) * 128 * nk * kKChunk * 2;
}

int launch_pack_wq(const void* wq, int64_t stride, int hidden, void* out, cudaStream_t stream) {
  const int nk = (hidden + kKChunk - 1) / kKChunk;
  const int64_t chunks = static_cast<int64_t>(kHeads) * 128 * nk * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148 * 16));
  pack_wq_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(wq), stride, hidden,
                                             nk, static_cast<uint16_t*>(out));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
