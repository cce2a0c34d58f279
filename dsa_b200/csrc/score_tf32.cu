// Dense indexer scoring for float32 queries and keys on the sm_100a tensor cores, with
// error-compensated TF32 (three products per term):
//
//   score[b][s] = sum_h w[b][h] * ReLU(q[b][h] . k[b][s]),   H = 64, D = 128
//   q . k ~= q_hi . k_hi + q_lo . k_hi + q_hi . k_lo
//
// kind::tf32 reads a float32 operand as TF32 by dropping its 13 low mantissa bits, so the
// raw float32 words are the high parts as they stand; the low parts are the exact float32
// differences x_lo = x - (x with those bits cleared).  The dropped q_lo . k_lo term and the
// truncation of the low parts leave a relative error of about 2^-21 per product, far
// inside the 1e-5 float32 tolerance the TF32 product alone (2^-11) misses.
//
// One persistent CTA per SM walks a contiguous range of 128-key tiles; a tile streams as
// four 32-dimension slices (one 128-byte swizzle row per key).  Warp roles:
//   warp 0      TMA producer: key slices [128 keys x 32 dims] f32 into an 8-stage ring;
//               the sequence's q [64 x 128] into rows 0..63 of the B operand.
//   warp 1      tcgen05 issuer, per 8-dimension step of a slice: M=128 keys x N=128 with
//               B = [q_hi; q_lo] (TMEM columns 0..63: q_hi . k, 64..127: q_lo . k), then
//               M=128 x N=64 with A = k_lo, B = q_hi into columns 64..127.
//   warps 2..5  residual writers: k_lo of each landed slice into a 2-slot ring, q_lo of
//               each new sequence into rows 64..127 of the B operand (elementwise in the
//               128-byte swizzled layout, which leaves every element's position unchanged).
//   warps 6..9  epilogue: each thread owns one key (one TMEM lane), adds the two column
//               halves per head, applies ReLU * w_h and sums the heads in the fixed order of
//               the 16-bit kernels, one float per key.
// HBM traffic per key = its 512 bytes, read once; q/w per sequence come from L2.
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace tdsa {

namespace {

constexpr int kTileKeys = 128;
constexpr int kSliceDims = 32;                          // one 128-byte row of f32
constexpr int kSlices = kHeadDim / kSliceDims;          // 4 per tile
constexpr int kStageBytes = kTileKeys * kSliceDims * 4; // 16 KiB
constexpr int kStages = 8;
constexpr int kLoSlots = 2;
constexpr int kQBoxBytes = 2 * kHeads * kSliceDims * 4; // 128 rows (q_hi, q_lo) x 32 dims
constexpr int kQRawBytes = kHeads * kSliceDims * 4;     // the 64 loaded rows of a box
constexpr int kQBytes = kSlices * kQBoxBytes;           // 64 KiB
constexpr int kAccBufs = 2;
constexpr int kAccCols = 2 * kHeads;                    // 128 f32 columns per tile
constexpr int kTmemCols = kAccBufs * kAccCols;
constexpr int kThreads = 320;
constexpr int kBarrierBytes = 1024;
constexpr int kSmemBytes =
    (kStages + kLoSlots) * kStageBytes + kQBytes + kBarrierBytes + 1024;

struct Tf32Args {
  const float* w;
  int64_t w_stride;
  float* out;
  int64_t out_stride;
  int length;
  int tiles_per_seq;
  int64_t total_tiles;
  int* status;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Instruction descriptor for kind::tf32 with f32 accumulation, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// x - (x with its 13 low mantissa bits cleared): exact in float32.
__device__ __forceinline__ float tf32_residual(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// n floats at src (16-byte aligned) -> their residuals at dst, 128 threads, float4 steps.
__device__ __forceinline__ void write_residuals(const float* src, float* dst, int n, int tid) {
  for (int i = tid * 4; i < n; i += 128 * 4) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    float4 r;
    r.x = tf32_residual(v.x);
    r.y = tf32_residual(v.y);
    r.z = tf32_residual(v.z);
    r.w = tf32_residual(v.w);
    *reinterpret_cast<float4*>(dst + i) = r;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    score_dense_tf32_kernel(const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap qmap, const Tf32Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* ring = smem;                                   // [kStages][16 KiB] raw k slices
  uint8_t* lo_ring = smem + kStages * kStageBytes;        // [kLoSlots][16 KiB] k_lo
  uint8_t* q_base = lo_ring + kLoSlots * kStageBytes;     // [4 slices][128 rows][32] f32
  uint64_t* full = reinterpret_cast<uint64_t*>(q_base + kQBytes);
  uint64_t* empty = full + kStages;
  uint64_t* lofull = empty + kStages;
  uint64_t* loempty = lofull + kLoSlots;
  uint64_t* qfull = loempty + kLoSlots;   // raw q landed
  uint64_t* qready = qfull + 1;           // q_lo written
  uint64_t* qempty = qready + 1;          // the MMA is done with this sequence's q
  uint64_t* accfull = qempty + 1;
  uint64_t* accempty = accfull + kAccBufs;
  uint64_t* done = accempty + kAccBufs;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t t0 = a.total_tiles * blockIdx.x / gridDim.x;
  const int64_t t1 = a.total_tiles * (blockIdx.x + 1) / gridDim.x;
  const int tps = a.tiles_per_seq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kLoSlots; ++s) {
      mbar_init(&lofull[s], 4);  // one arrival per residual warp
      mbar_init(&loempty[s], 1);
    }
    mbar_init(qfull, 1);
    mbar_init(qready, 4);
    mbar_init(qempty, 1);
    for (int s = 0; s < kAccBufs; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&qmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();  // q, w and the keys may come from the previous kernel
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const uint64_t pol_k = policy_evict_first();
      const uint64_t pol_q = policy_evict_last();
      int prev_b = -1;
      uint32_t qcount = 0, it = 0;
      bool ok = true;
      for (int64_t t = t0; t < t1 && ok; ++t) {
        const int b = static_cast<int>(t / tps);
        const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tps);
        if (b != prev_b) {
          if (!mbar_wait(qempty, (qcount & 1u) ^ 1u, abort_flag)) break;
          mbar_arrive_expect_tx(qfull, kSlices * kQRawBytes);
          for (int j = 0; j < kSlices; ++j)
            tma_load_3d(q_base + j * kQBoxBytes, &qmap, qfull, j * kSliceDims, 0, b, pol_q);
          ++qcount;
          prev_b = b;
        }
        for (int j = 0; j < kSlices; ++j, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_3d(ring + s * kStageBytes, &kmap, &full[s], j * kSliceDims, tt * kTileKeys,
                      b, pol_k);
        }
      }
      // Let every issued copy land before the CTA can exit (bounded, abort or not).
      volatile int no_abort = 0;
      for (uint32_t s = 0; s < kStages && s < it; ++s) {
        const uint32_t n = (it - s + kStages - 1) / kStages;
        mbar_wait(&full[s], (n - 1) & 1u, &no_abort);
      }
      if (qcount) mbar_wait(qfull, (qcount - 1) & 1u, &no_abort);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc_wide = umma_idesc_tf32(128, 2 * kHeads);
      constexpr uint32_t idesc_half = umma_idesc_tf32(128, kHeads);
      int prev_b = -1;
      uint32_t qcount = 0, it = 0, acc_it = 0;
      bool ok = true;
      for (int64_t t = t0; t < t1 && ok; ++t, ++acc_it) {
        const int b = static_cast<int>(t / tps);
        if (b != prev_b) {
          if (prev_b >= 0) umma_commit(qempty);
          if (!mbar_wait(qready, qcount & 1u, abort_flag)) break;
          ++qcount;
          prev_b = b;
        }
        const uint32_t acc = acc_it % kAccBufs, aph = (acc_it / kAccBufs) & 1u;
        if (!mbar_wait(&accempty[acc], aph ^ 1u, abort_flag)) break;
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int j = 0; j < kSlices; ++j, ++it) {
          const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
          const uint32_t l = it % kLoSlots, lph = (it / kLoSlots) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag) || !mbar_wait(&lofull[l], lph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(ring + s * kStageBytes);
          const uint32_t a_lo = smem_u32(lo_ring + l * kStageBytes);
          const uint32_t bq = smem_u32(q_base + j * kQBoxBytes);
#pragma unroll
          for (int k = 0; k < kSliceDims / 8; ++k) {
            const uint64_t bd = sw128_kmajor_desc(bq + k * 32);
            umma_tf32(d_tmem, sw128_kmajor_desc(a_hi + k * 32), bd, idesc_wide,
                      (j | k) ? 1u : 0u);
            umma_tf32(d_tmem + kHeads, sw128_kmajor_desc(a_lo + k * 32), bd, idesc_half, 1u);
          }
          umma_commit(&empty[s]);
          umma_commit(&loempty[l]);
        }
        if (ok) umma_commit(&accfull[acc]);
      }
      // All MMAs must be complete before TMEM is released.
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ residual writers
    const int rt = threadIdx.x - 64;  // 0..127
    int prev_b = -1;
    uint32_t qcount = 0, it = 0;
    bool ok = true;
    for (int64_t t = t0; t < t1 && ok; ++t) {
      const int b = static_cast<int>(t / tps);
      if (b != prev_b) {
        if (!mbar_wait(qfull, qcount & 1u, abort_flag)) break;
        for (int j = 0; j < kSlices; ++j) {
          const float* src = reinterpret_cast<const float*>(q_base + j * kQBoxBytes);
          write_residuals(src, const_cast<float*>(src) + kQRawBytes / 4, kQRawBytes / 4, rt);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(qready);
        ++qcount;
        prev_b = b;
      }
      for (int j = 0; j < kSlices; ++j, ++it) {
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        const uint32_t l = it % kLoSlots, lph = (it / kLoSlots) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag) ||
            !mbar_wait(&loempty[l], lph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        write_residuals(reinterpret_cast<const float*>(ring + s * kStageBytes),
                        reinterpret_cast<float*>(lo_ring + l * kStageBytes), kStageBytes / 4,
                        rt);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&lofull[l]);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const uint32_t quad = static_cast<uint32_t>(warp & 3);
    int prev_b = -1;
    uint32_t acc_it = 0;
    float wr[kHeads];
    for (int64_t t = t0; t < t1; ++t, ++acc_it) {
      const int b = static_cast<int>(t / tps);
      const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tps);
      if (b != prev_b) {
        const float* wb = a.w + static_cast<int64_t>(b) * a.w_stride;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) wr[h] = __ldg(wb + h);
        prev_b = b;
      }
      const uint32_t acc = acc_it % kAccBufs, aph = (acc_it / kAccBufs) & 1u;
      if (!mbar_wait(&accfull[acc], aph, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + acc * kAccCols;
      // the 16-bit kernels' fixed order: four interleaved sums over h mod 4, heads 0..31
      // then 32..63, combined as (s0 + s1) + (s2 + s3)
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hi[32], lo[32];
        tmem_ld32(taddr + half * 32, hi);            // q_hi . k for heads 32 half + i
        tmem_ld32(taddr + kHeads + half * 32, lo);   // q_lo . k_hi + q_hi . k_lo
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 32; h += 4) {
          const float* wh = wr + half * 32 + h;
          s0 = fmaf(wh[0], fmaxf(__uint_as_float(hi[h + 0]) + __uint_as_float(lo[h + 0]), 0.f), s0);
          s1 = fmaf(wh[1], fmaxf(__uint_as_float(hi[h + 1]) + __uint_as_float(lo[h + 1]), 0.f), s1);
          s2 = fmaf(wh[2], fmaxf(__uint_as_float(hi[h + 2]) + __uint_as_float(lo[h + 2]), 0.f), s2);
          s3 = fmaf(wh[3], fmaxf(__uint_as_float(hi[h + 3]) + __uint_as_float(lo[h + 3]), 0.f), s3);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[acc]);
      const int row = tt * kTileKeys + static_cast<int>(quad) * 32 + lane;
      if (row < a.length)
        a.out[static_cast<int64_t>(b) * a.out_stride + row] = (s0 + s1) + (s2 + s3);
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
}

}  // namespace

bool score_dense_tf32_supported(const float* q, int64_t q_bs, const float* k, int64_t k_bs,
                                int64_t k_rs, int batch) {
  const auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return aligned(q) && aligned(k) && k_rs % 4 == 0 && k_rs >= kHeadDim &&
         (batch == 1 || (k_bs % 4 == 0 && q_bs % 4 == 0));
}

int launch_score_dense_tf32(const float* q, int64_t q_bs, const float* w, int64_t w_bs,
                            const float* k, int64_t k_bs, int64_t k_rs, int batch, int length,
                            float* out, int64_t o_bs, cudaStream_t stream, int* status) {
  CUtensorMap kmap, qmap;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(length),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(k_bs) * 4
                                       : static_cast<uint64_t>(k_rs) * 4 * length;
    const uint64_t strides[2] = {static_cast<uint64_t>(k_rs) * 4, bstride};
    const uint32_t box[3] = {kSliceDims, kTileKeys, 1};
    int rc = encode_tmap(&kmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, k, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(kHeads),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(q_bs) * 4
                                       : static_cast<uint64_t>(kHeads * kHeadDim * 4);
    const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim) * 4, bstride};
    const uint32_t box[3] = {kSliceDims, kHeads, 1};
    int rc = encode_tmap(&qmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, q, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Tf32Args a;
  a.w = w;
  a.w_stride = w_bs;
  a.out = out;
  a.out_stride = o_bs;
  a.length = length;
  a.tiles_per_seq = (length + kTileKeys - 1) / kTileKeys;
  a.total_tiles = static_cast<int64_t>(a.tiles_per_seq) * batch;
  a.status = status;
  const int sms = device_sm_count(current_device());
  const int64_t grid = a.total_tiles < sms ? a.total_tiles : sms;
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(score_dense_tf32_kernel),
                                      kSmemBytes));
  TDSA_CUDA_CHECK(launch_pdl(score_dense_tf32_kernel, dim3(static_cast<unsigned>(grid)),
                             dim3(kThreads), kSmemBytes, stream, kmap, qmap, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
