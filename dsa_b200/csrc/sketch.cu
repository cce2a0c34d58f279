// Certified INT8 key sketch: an exact top-k that reads a key's full 256 bytes only where a
// 136-byte sketch of it cannot rule the key out.
//
// Sketch of key k (tdsa_sketch_keys): per-key symmetric INT8 values k^ = rint(k / s_k),
// s_k = max|k_i| / 127, and two norms rounded up to float16: r_k >= ||k - s_k k^|| (the
// quantization residual) and n_k >= ||s_k k^||.  128 + 4 + 4 = 136 bytes per key.
//
// Query of one step (sketch_query_kernel): per head h INT8 values q^_h = rint(q_h / s_h),
// s_h = max|q_h| / 127, q~_h = s_h q^_h and the exact residual d_h = q_h - q~_h; per sequence
// G = sum_h |w_h| ||q_h|| and D = sum_h |w_h| ||d_h||.
//
// Bound: with the head dots q_h . k and their sketch q~_h . s_k k^ (an int8 MMA, exact in
// int32), |q_h.k - q~_h.s_k k^| <= ||q_h|| r_k + ||d_h|| n_k, and ReLU is 1-Lipschitz, so the
// score S = sum_h w_h ReLU(q_h . k) (reference progressive_kernel.py:45-55) lies within
// gap_k = G r_k + D n_k of the sketch score S~ (plus a 2^-14 relative allowance for the
// float32 arithmetic of S~, folded into D).  Every key gets an upper bound U_k = S~ + gap_k
// and a lower bound L_k = S~ - gap_k.
//
// Selection: the k-th largest true score is at least the k-th largest L_k (each score is
// at least its own lower bound), so tau = the lower edge of the histogram sub-bin holding
// the k-th largest L_k never exceeds it.  A key whose U_k < tau is below the k-th score and
// is never read; the 16-key blocks holding a key with U_k >= tau are scored exactly
// (score_blocks.cu, the dense kernel's arithmetic), the rest score -inf, and the top-k of
// that row is dense scoring's top-k, ties included.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "tiles.cuh"

namespace tdsa {

namespace {

constexpr int kTileKeys = 128;
constexpr int kStages = 8;
constexpr int kStageBytes = kTileKeys * kHeadDim;  // 16 KiB of int8 sketch rows
constexpr int kQRows = kHeads;                     // one int8 row per head
constexpr int kQBytes = kQRows * kHeadDim;         // 8 KiB
constexpr int kQSlots = 2;
constexpr int kAccBufs = 2;
constexpr int kAccCols = kHeads;                // one s32 accumulator column per head
constexpr int kTmemCols = kAccBufs * kAccCols;  // 128
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, taking alternate tiles
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kBarrierBytes = 1024;
constexpr int kHistBytes = kKeyHistBins * 4;
constexpr int kSmemBytes =
    kStages * kStageBytes + kQSlots * kQBytes + kBarrierBytes + kHistBytes + 1024;
constexpr int kSelThreads = kTileListThreads;  // the selection kernel emits tile lists
constexpr int kHistCopies = 8;
constexpr int kHistCopyBytes = kHistCopies * kKeyHistBins * 4;
constexpr uint32_t kNegInfBin = 0x007FFFFFu >> 20;  // histogram bin of the -inf key

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ void decode4(uint2 raw, int dtype, float (&v)[4]) {
  const uint16_t e[4] = {static_cast<uint16_t>(raw.x & 0xFFFFu), static_cast<uint16_t>(raw.x >> 16),
                         static_cast<uint16_t>(raw.y & 0xFFFFu), static_cast<uint16_t>(raw.y >> 16)};
#pragma unroll
  for (int j = 0; j < 4; ++j)
    v[j] = dtype == TDSA_BF16 ? __uint_as_float(static_cast<uint32_t>(e[j]) << 16)
                              : __half2float(__ushort_as_half(e[j]));
}

// int32 -> float32, exact for |x| < 2^22, with one integer and one float add (full rate;
// the conversion unit runs at a quarter of that): the bits of x + 1.5 * 2^23 read as a float
// are 1.5 * 2^23 + x (a float ulp of 1 there).  Written in PTX so that the pair stays two
// adds.
__device__ __forceinline__ float small_int_to_float(uint32_t x) {
  float r;
  asm("{\n\t.reg .b32 t;\n\t"
      "add.s32 t, %1, 0x4B400000;\n\t"
      "sub.rn.f32 %0, t, 0f4B400000;\n\t}"
      : "=f"(r)
      : "r"(x));
  return r;
}

__device__ __forceinline__ int q8(float x) {
  return static_cast<int>(fminf(fmaxf(rintf(x), -127.f), 127.f));
}

__device__ __forceinline__ uint32_t pack4(const int (&q)[4]) {
  return (static_cast<uint32_t>(q[0]) & 0xFFu) | ((static_cast<uint32_t>(q[1]) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(q[2]) & 0xFFu) << 16) |
         ((static_cast<uint32_t>(q[3]) & 0xFFu) << 24);
}

__device__ __forceinline__ double warp_sum(double x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// sqrt(x) rounded up to float16 (x >= 0; a relative 2^-40 covers the float64 sum's rounding).
__device__ __forceinline__ __half norm_up(double x) {
  return __float2half_ru(__double2float_ru(sqrt(x * (1.0 + 0x1p-40))));
}

// ---------------------------------------------------------------- key sketch
// One warp per key, 4 dimensions per lane.  A key holding a non-finite value gets scale 0
// and infinite bounds: it is always read in full.
__global__ void sketch_keys_kernel(const void* keys, int64_t k_bs, int64_t k_rs, int dtype,
                                   int first, int length, int8_t* sketch, int64_t sk_bs,
                                   float* scale, __half2* bounds, int64_t sc_bs) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warps = (blockDim.x >> 5) * gridDim.x;
  for (int key = first + blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); key < length;
       key += warps) {
    const uint2 raw = *reinterpret_cast<const uint2*>(
        static_cast<const uint16_t*>(keys) + static_cast<int64_t>(b) * k_bs +
        static_cast<int64_t>(key) * k_rs + lane * 4);
    float v[4];
    decode4(raw, dtype, v);
    float m = 0.f;
    bool finite = true;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      finite = finite && isfinite(v[j]);
      m = fmaxf(m, fabsf(v[j]));
    }
    finite = __all_sync(0xffffffffu, finite);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = (finite && m > 0.f) ? m / 127.f : 0.f;
    int qk[4] = {0, 0, 0, 0};
    double e2 = 0.0, n2 = 0.0;
    if (s > 0.f) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qk[j] = q8(v[j] / s);
        const double e = static_cast<double>(v[j]) - static_cast<double>(s) * qk[j];
        e2 += e * e;
        n2 += static_cast<double>(qk[j]) * qk[j];
      }
    }
    e2 = warp_sum(e2);
    n2 = warp_sum(n2);
    const int64_t at = static_cast<int64_t>(b) * sk_bs + static_cast<int64_t>(key) * kHeadDim;
    reinterpret_cast<uint32_t*>(sketch + at)[lane] = pack4(qk);
    if (lane == 0) {
      const int64_t i = static_cast<int64_t>(b) * sc_bs + key;
      scale[i] = s;
      const double sd = static_cast<double>(s);
      bounds[i] = finite ? __halves2half2(norm_up(e2), norm_up(n2 * sd * sd))
                         : __halves2half2(__float2half(INFINITY), __float2half(INFINITY));
    }
  }
}

// ---------------------------------------------------------------- query of one step
struct QueryArgs {
  const void* q;
  int64_t q_bs;
  const float* w;
  int64_t w_bs;
  int dtype;
  int8_t* qhl;       // [B][64][128]: the int8 query rows
  float* wq;         // [B][64]: w_h * s_h
  float* gd;         // [B][2]: G, D (rounded up; D with the float32 allowance)
  uint32_t* hist_l;  // [B][4096]: cleared for the bound kernel
  int32_t* counter;  // tile counter: cleared for the selection kernel
};

constexpr int kQueryThreads = 1024;  // 32 warps: two heads each

// One CTA per sequence, one warp per head at a time (4 dims per lane).
__global__ void __launch_bounds__(kQueryThreads) sketch_query_kernel(const QueryArgs a) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  constexpr int kWarps = kQueryThreads / 32;
  __shared__ double sg[kWarps], sdd[kWarps];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* hrow = a.hist_l + static_cast<int64_t>(b) * kKeyHistBins;
  for (int i = threadIdx.x; i < kKeyHistBins; i += kQueryThreads) hrow[i] = 0u;
  if (b == 0 && threadIdx.x == 0) *a.counter = 0;
  double g = 0.0, d = 0.0;
  for (int h = warp; h < kHeads; h += kWarps) {
    const uint2 raw = *reinterpret_cast<const uint2*>(
        static_cast<const uint16_t*>(a.q) + static_cast<int64_t>(b) * a.q_bs + h * kHeadDim +
        lane * 4);
    float v[4];
    decode4(raw, a.dtype, v);
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m > 0.f ? m / 127.f : 0.f;
    int qq[4] = {0, 0, 0, 0};
    double dq2 = 0.0, qq2 = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s > 0.f) qq[j] = q8(v[j] / s);
      const double dl = static_cast<double>(v[j]) - static_cast<double>(s) * qq[j];
      dq2 += dl * dl;
      qq2 += static_cast<double>(v[j]) * v[j];
    }
    dq2 = warp_sum(dq2);
    qq2 = warp_sum(qq2);
    int8_t* row = a.qhl + static_cast<int64_t>(b) * kQBytes;
    reinterpret_cast<uint32_t*>(row + h * kHeadDim)[lane] = pack4(qq);
    if (lane == 0) {
      const float wh = a.w[static_cast<int64_t>(b) * a.w_bs + h];
      a.wq[static_cast<int64_t>(b) * kHeads + h] = wh * s;
      g += fabs(static_cast<double>(wh)) * sqrt(qq2);
      d += fabs(static_cast<double>(wh)) * sqrt(dq2);
    }
  }
  if (lane == 0) {
    sg[warp] = g;
    sdd[warp] = d;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double gt = 0.0, dt = 0.0;
    for (int i = 0; i < kWarps; ++i) {
      gt += sg[i];
      dt += sdd[i];
    }
    gt *= 1.0 + 0x1p-40;
    dt = (dt + 0x1p-14 * (gt + dt)) * (1.0 + 0x1p-40);
    a.gd[2 * b] = __double2float_ru(gt);
    a.gd[2 * b + 1] = __double2float_ru(dt);
  }
}

// ---------------------------------------------------------------- sketch bounds
struct BoundArgs {
  const float* wq;
  const float* gd;
  const float* scale;
  const __half2* bounds;
  int64_t sc_bs;
  float* upper;      // [B][ub_bs]: per 16-key block, the largest upper bound of its keys
  int64_t ub_bs;
  float* lower;      // [B][o_bs]: per key
  int64_t o_bs;
  uint32_t* hist_l;  // [B][4096]: bins of the lower bounds (added)
  int length;
  int tiles_per_seq;
  int64_t total_tiles;
  int* status;
};

// The dense kernel's pipeline (score_tc.cu) on the INT8 sketch: warp 0 loads 16 KiB sketch
// tiles (128 keys x 128 bytes) and each sequence's 8 KiB int8 query by TMA; warp 1 issues
// per tile one K=128 int8 MMA (4 x K32, s32 accumulators in TMEM); warps 2..5 own one key
// each: S~ = s_k sum_h (w_h s_h) ReLU(acc_h), then the
// bounds, and the lower bound's key bin into the row histogram.
__global__ void __launch_bounds__(kThreads, 1)
    sketch_bounds_kernel(const __grid_constant__ CUtensorMap smap,
                         const __grid_constant__ CUtensorMap qmap, const BoundArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* stage_base = smem;
  uint8_t* q_base = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(q_base + kQSlots * kQBytes);
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + kQSlots;
  uint64_t* accfull = qempty + kQSlots;
  uint64_t* accempty = accfull + kAccBufs;
  uint64_t* done = accempty + kAccBufs;
  uint64_t* hbar = done + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(hbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint32_t* shist = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + kBarrierBytes);

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
    for (int s = 0; s < kQSlots; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], 1);
    }
    for (int s = 0; s < kAccBufs; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);  // the four warps of the buffer's half
    }
    mbar_init(done, 1);
    mbar_init(hbar, kEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < kKeyHistBins; i += kThreads) shist[i] = 0u;
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&smap);
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
  pdl_wait();  // the query tiles, weights and the histogram come from the previous kernel
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const uint64_t pol_k = policy_evict_first();
      const uint64_t pol_q = policy_evict_last();
      int prev_b = -1;
      uint32_t qcount = 0, it = 0;
      for (int64_t t = t0; t < t1; ++t) {
        const int b = static_cast<int>(t / tps);
        const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tps);
        if (b != prev_b) {
          const uint32_t slot = qcount % kQSlots, ph = (qcount / kQSlots) & 1u;
          if (!mbar_wait(&qempty[slot], ph ^ 1u, abort_flag)) break;
          mbar_arrive_expect_tx(&qfull[slot], kQBytes);
          tma_load_3d(q_base + slot * kQBytes, &qmap, &qfull[slot], 0, 0, b, pol_q);
          ++qcount;
          prev_b = b;
        }
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_3d(stage_base + s * kStageBytes, &smap, &full[s], 0, tt * kTileKeys, b, pol_k);
        ++it;
      }
      volatile int no_abort = 0;
      for (uint32_t s = 0; s < kStages && s < it; ++s) {
        const uint32_t n = (it - s + kStages - 1) / kStages;
        mbar_wait(&full[s], (n - 1) & 1u, &no_abort);
      }
      for (uint32_t s = 0; s < kQSlots && s < qcount; ++s) {
        const uint32_t n = (qcount - s + kQSlots - 1) / kQSlots;
        mbar_wait(&qfull[s], (n - 1) & 1u, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = umma_idesc_s8(128, kHeads);
      int prev_b = -1;
      uint32_t qcount = 0, it = 0, acc_it = 0, slot = 0;
      for (int64_t t = t0; t < t1; ++t) {
        const int b = static_cast<int>(t / tps);
        if (b != prev_b) {
          if (prev_b >= 0) umma_commit(&qempty[slot]);
          slot = qcount % kQSlots;
          if (!mbar_wait(&qfull[slot], (qcount / kQSlots) & 1u, abort_flag)) break;
          ++qcount;
          prev_b = b;
        }
        const uint32_t acc = acc_it & 1u, aph = (acc_it >> 1) & 1u;
        if (!mbar_wait(&accempty[acc], aph ^ 1u, abort_flag)) break;
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(stage_base + s * kStageBytes);
        const uint32_t b_addr = smem_u32(q_base + slot * kQBytes);
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
#pragma unroll
        for (int k = 0; k < kHeadDim / 32; ++k)
          umma_i8(d_tmem, sw128_kmajor_desc(a_addr + k * 32),
                  sw128_kmajor_desc(b_addr + k * 32), idesc, k > 0 ? 1u : 0u);
        umma_commit(&empty[s]);
        umma_commit(&accfull[acc]);
        ++it;
        ++acc_it;
      }
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    // warp w reads TMEM lanes 32 * (w % 4); warps 2..5 take the CTA's even tiles
    // (accumulator buffer 0), warps 6..9 the odd ones (buffer 1)
    const uint32_t quad = static_cast<uint32_t>(warp & 3);
    const uint32_t half = static_cast<uint32_t>(warp - 2) >> 2;
    const int etid = (warp - 2) * 32 + lane;
    int prev_b = -1;
    uint32_t mine = 0, hph = 0;
    float wr[kHeads];
    float G = 0.f, D = 0.f;
    auto hist_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(hbar);
      const bool ok = mbar_wait(hbar, hph & 1u, abort_flag);
      ++hph;
      return ok;
    };
    auto hist_flush = [&](int b) -> bool {
      if (!hist_sync()) return false;
      uint32_t* dst = a.hist_l + static_cast<int64_t>(b) * kKeyHistBins;
      for (int i = etid; i < kKeyHistBins; i += 32 * kEpiWarps) {
        const uint32_t c = shist[i];
        if (c) {
          atomicAdd(dst + i, c);
          shist[i] = 0u;
        }
      }
      return hist_sync();
    };
    bool ok = true;
    for (int64_t t = t0; t < t1; ++t) {
      const int b = static_cast<int>(t / tps);
      const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tps);
      if (b != prev_b) {
        if (prev_b >= 0 && !hist_flush(prev_b)) {
          ok = false;
          break;
        }
        const float* wqb = a.wq + static_cast<int64_t>(b) * kHeads;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) wr[h] = __ldg(wqb + h);
        G = __ldg(a.gd + 2 * b);
        D = __ldg(a.gd + 2 * b + 1);
        prev_b = b;
      }
      if (static_cast<uint32_t>((t - t0) & 1) != half) continue;
      const int row = tt * kTileKeys + static_cast<int>(quad) * 32 + lane;
      const bool valid = row < a.length;
      float sk = 0.f, r = 0.f, n = 0.f;
      if (valid) {
        const int64_t i = static_cast<int64_t>(b) * a.sc_bs + row;
        sk = __ldg(a.scale + i);
        const __half2 bb = a.bounds[i];
        r = __low2float(bb);
        n = __high2float(bb);
      }
      const uint32_t aph = mine & 1u;
      if (!mbar_wait(&accfull[half], aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + half * kAccCols;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      {
        uint32_t h0[32], h1[32];
        tmem_ld32(taddr, h0);
        tmem_ld32(taddr + 32, h1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[half]);
        // |acc| <= 128 * 127 * 127 < 2^22: exact conversions
#pragma unroll
        for (int h = 0; h < 32; h += 4) {
          s0 = fmaf(wr[h + 0], fmaxf(small_int_to_float(h0[h + 0]), 0.f), s0);
          s1 = fmaf(wr[h + 1], fmaxf(small_int_to_float(h0[h + 1]), 0.f), s1);
          s2 = fmaf(wr[h + 2], fmaxf(small_int_to_float(h0[h + 2]), 0.f), s2);
          s3 = fmaf(wr[h + 3], fmaxf(small_int_to_float(h0[h + 3]), 0.f), s3);
        }
#pragma unroll
        for (int h = 0; h < 32; h += 4) {
          s0 = fmaf(wr[32 + h + 0], fmaxf(small_int_to_float(h1[h + 0]), 0.f), s0);
          s1 = fmaf(wr[32 + h + 1], fmaxf(small_int_to_float(h1[h + 1]), 0.f), s1);
          s2 = fmaf(wr[32 + h + 2], fmaxf(small_int_to_float(h1[h + 2]), 0.f), s2);
          s3 = fmaf(wr[32 + h + 3], fmaxf(small_int_to_float(h1[h + 3]), 0.f), s3);
        }
      }
      const float sketch_score = sk * ((s0 + s1) + (s2 + s3));
      const float gap = __fmaf_ru(G, r, __fmul_ru(D, n));
      const float up = __fadd_ru(sketch_score, gap);
      const float lo = __fsub_rd(sketch_score, gap);
      if (valid) a.lower[static_cast<int64_t>(b) * a.o_bs + row] = lo;
      // the block's largest upper bound: 16 lanes hold one 16-key block
      float ub = valid ? up : -INFINITY;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ub = fmaxf(ub, __shfl_xor_sync(0xffffffffu, ub, o));
      if ((lane & 15) == 0 && row < a.length)
        a.upper[static_cast<int64_t>(b) * a.ub_bs + (row >> 4)] = ub;
      add_to_bin(shist, valid, float_to_key(lo) >> 20);
      ++mine;
    }
    if (ok && prev_b >= 0) hist_flush(prev_b);
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
}

// ---------------------------------------------------------------- selection
struct SelectArgs {
  const float* upper;  // [B][nb_stride] block maxima of the upper bounds
  const float* lower;  // [B][o_bs]
  int64_t o_bs;
  uint32_t* hist_l;  // [B][4096] lower-bound bins: read, then cleared
  uint32_t* hist;    // [B][4096] the exact pass's key histogram: cleared, -inf keys counted
  int hist_for_topk;
  float* scores;  // [B][o_bs]: -inf for the keys of blocks that are not read
  int8_t* flag;   // [B][nb_stride]: 1 = the 16-key block is read
  int64_t nb_stride;
  int32_t* tile_seq;
  int32_t* tile_blk;
  int32_t* counter;
  float* tau;
  unsigned long long* stats;  // [B][2]: keys read, blocks read (added); or null
  int length, k;
};

// One 1024-thread CTA per sequence: tau from the lower bounds' histogram (12 bits, then 12
// more inside that bin), the blocks holding a key with U >= tau, their tile list, -inf for
// the keys of the other blocks.
__global__ void __launch_bounds__(kSelThreads) sketch_select_kernel(const SelectArgs a) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  extern __shared__ uint32_t hcopies[];  // kHistCopies x 4096 words
  __shared__ uint32_t h[kKeyHistBins];
  __shared__ uint32_t wtot[32];
  __shared__ uint32_t sbase[4];
  __shared__ unsigned long long acc[2];
  __shared__ float s_tau;
  __shared__ uint32_t s_bin, s_rank;
  const int seq = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = (a.length + 15) / 16;
  uint32_t* lrow = a.hist_l + static_cast<int64_t>(seq) * kKeyHistBins;
  uint32_t* frow = a.hist + static_cast<int64_t>(seq) * kKeyHistBins;
  const float* up = a.upper + static_cast<int64_t>(seq) * a.nb_stride;
  const float* lo = a.lower + static_cast<int64_t>(seq) * a.o_bs;
  int8_t* fl = a.flag + static_cast<int64_t>(seq) * a.nb_stride;
  if (threadIdx.x < 2) acc[threadIdx.x] = 0ull;
  for (int i = threadIdx.x; i < kKeyHistBins; i += kSelThreads) {
    h[i] = lrow[i];
    lrow[i] = 0u;
    frow[i] = 0u;
  }
  __syncthreads();
  // level 1: the bin of the k-th largest lower bound (thread t: bins 4095-4t .. 4092-4t)
  uint32_t c[4], tot = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    c[i] = h[kKeyHistBins - 1 - (4 * threadIdx.x + i)];
    tot += c[i];
  }
  uint32_t x = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  if (threadIdx.x == 0) {
    s_tau = -INFINITY;
    s_bin = 0xFFFFFFFFu;
  }
  __syncthreads();
  uint32_t above = x - tot;
  for (int i = 0; i < warp; ++i) above += wtot[i];
  const uint32_t kk = static_cast<uint32_t>(a.k);
  if (above < kk && kk <= above + tot) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (above < kk && kk <= above + c[i]) {
        s_bin = kKeyHistBins - 1 - (4 * threadIdx.x + i);
        s_rank = kk - above;
      }
      above += c[i];
    }
  }
  __syncthreads();
  const uint32_t bin1 = s_bin;
  if (bin1 != 0xFFFFFFFFu && bin1 != 0u) {
    // level 2: the next 12 key bits of the lower bounds in that bin
    for (int i = threadIdx.x; i < kHistCopies * kKeyHistBins; i += kSelThreads) hcopies[i] = 0u;
    __syncthreads();
    uint32_t* mine = hcopies + (warp & (kHistCopies - 1)) * kKeyHistBins;
    constexpr int kUnroll = 8;
    for (int base = 0; base < a.length; base += kSelThreads * kUnroll) {
      float v[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int i = base + j * kSelThreads + static_cast<int>(threadIdx.x);
        v[j] = i < a.length ? lo[i] : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int i = base + j * kSelThreads + static_cast<int>(threadIdx.x);
        const uint32_t key = float_to_key(v[j]);
        add_to_bin(mine, i < a.length && (key >> 20) == bin1, (key >> 8) & 0xFFFu);
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kKeyHistBins; i += kSelThreads) {
      uint32_t t = 0;
#pragma unroll
      for (int cc = 0; cc < kHistCopies; ++cc) t += hcopies[cc * kKeyHistBins + i];
      h[i] = t;
    }
    __syncthreads();
    const uint32_t r = s_rank;
    uint32_t d[4], dt = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      d[i] = h[kKeyHistBins - 1 - (4 * threadIdx.x + i)];
      dt += d[i];
    }
    uint32_t y = dt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t z = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) y += z;
    }
    if (lane == 31) wtot[warp] = y;
    __syncthreads();
    uint32_t ab = y - dt;
    for (int i = 0; i < warp; ++i) ab += wtot[i];
    if (ab < r && r <= ab + dt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (ab < r && r <= ab + d[i]) {
          const uint32_t lok = (bin1 << 20) | ((kKeyHistBins - 1 - (4 * threadIdx.x + i)) << 8);
          s_tau = lok > 0xFF800000u ? INFINITY : key_to_float(lok);
        }
        ab += d[i];
      }
    }
    __syncthreads();
  }
  const float tau = s_tau;
  if (threadIdx.x == 0) a.tau[seq] = tau;
  // block flags: read a block when its largest upper bound reaches tau
  unsigned long long read = 0, nread = 0;
  for (int blk = threadIdx.x; blk < nb; blk += kSelThreads) {
    const bool take = up[blk] >= tau;
    fl[blk] = take ? 1 : 0;
    if (take) {
      read += static_cast<unsigned long long>(min(16, a.length - blk * 16));
      ++nread;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    read += __shfl_xor_sync(0xffffffffu, read, o);
    nread += __shfl_xor_sync(0xffffffffu, nread, o);
  }
  if (lane == 0) {
    atomicAdd(&acc[0], read);
    atomicAdd(&acc[1], nread);
  }
  __syncthreads();
  const unsigned long long keys_read = acc[0];
  // keys of blocks that are not read score -inf (the top-k reads the whole row): one 16-key
  // block is four 16-byte stores (rows are 16-byte aligned and padded to whole blocks)
  if (keys_read < static_cast<unsigned long long>(a.length)) {
    float4* srow = reinterpret_cast<float4*>(a.scores + static_cast<int64_t>(seq) * a.o_bs);
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    for (int i = threadIdx.x; i < nb * 4; i += kSelThreads)
      if (fl[i >> 2] == 0) srow[i] = ninf;
  }
  if (threadIdx.x == 0) {
    if (a.hist_for_topk)
      frow[kNegInfBin] = static_cast<uint32_t>(static_cast<unsigned long long>(a.length) - keys_read);
    if (a.stats) {
      a.stats[2 * seq] += keys_read;
      a.stats[2 * seq + 1] += acc[1];
    }
  }
  emit_tiles(fl, nb, 1, 8, seq, a.tile_seq, a.tile_blk, a.counter, wtot, sbase);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct SketchLayout {
  size_t qhl = 0, wq = 0, gd = 0, upper = 0, lower = 0, scores = 0, hist_l = 0, hist = 0;
  size_t flag = 0, bmax = 0, tau = 0, tile_seq = 0, tile_blk = 0, counter = 0, topk_ws = 0;
  size_t topk_ws_bytes = 0, total = 0;
  int64_t nb_stride = 0, tcap = 0, ld = 0;
};

SketchLayout sketch_layout(int batch, int max_length, int k) {
  SketchLayout L;
  L.nb_stride = (max_length + 15) / 16;
  L.tcap = static_cast<int64_t>(batch) * ((L.nb_stride + 7) / 8);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  L.ld = L.nb_stride * 16;  // rows padded to whole 16-key blocks (16-byte aligned)
  const size_t rowf = static_cast<size_t>(batch) * L.ld * 4;
  L.qhl = take(static_cast<size_t>(batch) * kQBytes);
  L.wq = take(static_cast<size_t>(batch) * kHeads * 4);
  L.gd = take(static_cast<size_t>(batch) * 8);
  L.upper = take(static_cast<size_t>(batch) * L.nb_stride * 4);
  L.lower = take(rowf);
  L.scores = take(rowf);
  L.hist_l = take(static_cast<size_t>(batch) * kKeyHistBins * 4);
  L.hist = take(static_cast<size_t>(batch) * kKeyHistBins * 4);
  L.flag = take(static_cast<size_t>(batch) * L.nb_stride);
  L.bmax = take(static_cast<size_t>(batch) * L.nb_stride * 4);
  L.tau = take(static_cast<size_t>(batch) * 4);
  L.tile_seq = take(static_cast<size_t>(L.tcap) * 4);
  L.tile_blk = take(static_cast<size_t>(L.tcap) * 8 * 4);
  L.counter = take(16);
  L.topk_ws_bytes = topk_workspace_bytes(batch, max_length, k);
  L.topk_ws = take(L.topk_ws_bytes);
  L.total = off;
  return L;
}

}  // namespace

size_t sketch_workspace_bytes(int batch, int max_length, int k) {
  return sketch_layout(batch, max_length, k).total;
}

void sketch_workspace_offsets(int batch, int max_length, int k, int64_t* out) {
  const SketchLayout L = sketch_layout(batch, max_length, k);
  out[0] = static_cast<int64_t>(L.upper);
  out[1] = static_cast<int64_t>(L.lower);
  out[2] = static_cast<int64_t>(L.scores);
  out[3] = static_cast<int64_t>(L.tau);
  out[4] = L.nb_stride;
  out[5] = L.ld;
}

int launch_sketch_keys(const void* keys, int64_t k_bs, int64_t k_rs, int dtype, int batch,
                       int first, int length, int8_t* sketch, int64_t sk_bs, float* scale,
                       void* bounds, int64_t sc_bs, cudaStream_t stream) {
  const int nkeys = length - first;
  if (nkeys <= 0) return TDSA_OK;
  const int blocks_x = std::min(device_sm_count(current_device()) * 4, (nkeys + 7) / 8);
  TDSA_CUDA_CHECK(launch_pdl(sketch_keys_kernel, dim3(blocks_x, batch), dim3(256), 0, stream,
                             keys, k_bs, k_rs, dtype, first, length, sketch, sk_bs, scale,
                             static_cast<__half2*>(bounds), sc_bs));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

int run_sketch_topk(const void* q, int64_t q_bs, const float* w, int64_t w_bs, const void* keys,
                    int64_t k_bs, int64_t k_rs, int dtype, const int8_t* sketch, int64_t sk_bs,
                    const float* scale, const void* bounds, int64_t sc_bs, int batch,
                    int length, int max_length, int k, int sorted, void* out_idx,
                    int idx_bytes, int64_t idx_bs, float* out_val, int64_t val_bs,
                    unsigned long long* stats, void* ws, cudaStream_t stream) {
  const SketchLayout L = sketch_layout(batch, max_length, k);
  uint8_t* base = static_cast<uint8_t*>(ws);
  auto at = [&](size_t off) { return base + off; };
  int8_t* qhl = reinterpret_cast<int8_t*>(at(L.qhl));
  float* wq = reinterpret_cast<float*>(at(L.wq));
  float* gd = reinterpret_cast<float*>(at(L.gd));
  float* upper = reinterpret_cast<float*>(at(L.upper));
  float* lower = reinterpret_cast<float*>(at(L.lower));
  float* scores = reinterpret_cast<float*>(at(L.scores));
  uint32_t* hist_l = reinterpret_cast<uint32_t*>(at(L.hist_l));
  uint32_t* hist = reinterpret_cast<uint32_t*>(at(L.hist));
  int8_t* flag = reinterpret_cast<int8_t*>(at(L.flag));
  float* bmax = reinterpret_cast<float*>(at(L.bmax));
  float* tau = reinterpret_cast<float*>(at(L.tau));
  int32_t* tile_seq = reinterpret_cast<int32_t*>(at(L.tile_seq));
  int32_t* tile_blk = reinterpret_cast<int32_t*>(at(L.tile_blk));
  int32_t* counter = reinterpret_cast<int32_t*>(at(L.counter));
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  const bool hist_for_topk = length <= kTopkSegment;

  // 1. the step's int8 query, G and D; the histogram and tile counter cleared
  QueryArgs qa;
  qa.q = q;
  qa.q_bs = q_bs;
  qa.w = w;
  qa.w_bs = w_bs;
  qa.dtype = dtype;
  qa.qhl = qhl;
  qa.wq = wq;
  qa.gd = gd;
  qa.hist_l = hist_l;
  qa.counter = counter;
  TDSA_CUDA_CHECK(launch_pdl(sketch_query_kernel, dim3(batch), dim3(kQueryThreads), 0, stream,
                             qa));
  TDSA_CUDA_CHECK(cudaGetLastError());

  // 2. sketch bounds of every key (int8 MMAs), lower bounds into the row histograms
  CUtensorMap smap, qmap;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(length),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(sk_bs)
                                       : static_cast<uint64_t>(kHeadDim) * length;
    const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim), bstride};
    const uint32_t box[3] = {kHeadDim, kTileKeys, 1};
    int rc = encode_tmap(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, sketch, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(kQRows),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim),
                                 static_cast<uint64_t>(kQBytes)};
    const uint32_t box[3] = {kHeadDim, kQRows, 1};
    int rc = encode_tmap(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, qhl, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  BoundArgs ba;
  ba.wq = wq;
  ba.gd = gd;
  ba.scale = scale;
  ba.bounds = static_cast<const __half2*>(bounds);
  ba.sc_bs = sc_bs;
  ba.upper = upper;
  ba.ub_bs = L.nb_stride;
  ba.lower = lower;
  ba.o_bs = L.ld;
  ba.hist_l = hist_l;
  ba.length = length;
  ba.tiles_per_seq = (length + kTileKeys - 1) / kTileKeys;
  ba.total_tiles = static_cast<int64_t>(ba.tiles_per_seq) * batch;
  ba.status = status;
  const int sms = device_sm_count(current_device());
  const int grid = static_cast<int>(std::min<int64_t>(ba.total_tiles, sms));
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(sketch_bounds_kernel),
                                      kSmemBytes));
  TDSA_CUDA_CHECK(launch_pdl(sketch_bounds_kernel, dim3(grid), dim3(kThreads), kSmemBytes,
                             stream, smap, qmap, ba));
  TDSA_CUDA_CHECK(cudaGetLastError());

  // 3. tau, the blocks to read, their tile list
  SelectArgs sa;
  sa.upper = upper;
  sa.lower = lower;
  sa.o_bs = L.ld;
  sa.hist_l = hist_l;
  sa.hist = hist;
  sa.hist_for_topk = hist_for_topk ? 1 : 0;
  sa.scores = scores;
  sa.flag = flag;
  sa.nb_stride = L.nb_stride;
  sa.tile_seq = tile_seq;
  sa.tile_blk = tile_blk;
  sa.counter = counter;
  sa.tau = tau;
  sa.stats = stats;
  sa.length = length;
  sa.k = k;
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(sketch_select_kernel),
                                      kHistCopyBytes));
  TDSA_CUDA_CHECK(launch_pdl(sketch_select_kernel, dim3(batch), dim3(kSelThreads),
                             kHistCopyBytes, stream, sa));
  TDSA_CUDA_CHECK(cudaGetLastError());

  // 4. exact scores of the listed blocks (the dense kernel's arithmetic)
  BlockArgs xa;
  xa.bs = 16;
  xa.bpt = 8;
  xa.length = length;
  xa.nblocks = (length + 15) / 16;
  xa.tile_seq = tile_seq;
  xa.tile_blocks = tile_blk;
  xa.tile_count = counter;
  xa.w = w;
  xa.w_stride = w_bs;
  xa.out = scores;
  xa.out_stride = L.ld;
  xa.block_max = bmax;
  xa.bm_stride = L.nb_stride;
  xa.hist = hist_for_topk ? hist : nullptr;
  xa.status = status;
  int rc = launch_score_blocks(kModeExact, q, q_bs, keys, k_bs, k_rs, dtype, batch, xa, sms,
                               stream);
  if (rc) return rc;

  // 5. top-k of the row (from its histogram when it is one segment)
  return launch_topk(scores, L.ld, nullptr, 0, batch, length, k, sorted, out_idx,
                     idx_bytes, idx_bs, out_val, val_bs, at(L.topk_ws), L.topk_ws_bytes, stream,
                     nullptr, hist_for_topk ? hist : nullptr);
}

}  // namespace tdsa
