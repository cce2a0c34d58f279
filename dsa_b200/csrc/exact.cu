// Exact (certified) progressive top-k: the host schedule and its small device kernels.
//
// One decode step per sequence (all sequences of the batch advance together), five
// launches chained by programmatic dependent launch:
//   1. prepare (one CTA per sequence): the previous step's state update (U_b <- exact block
//      max of a scored block, its bound when pruned), the norms of the keys appended since
//      (max ||k|| per block), the certified coefficient
//      c = sum_h |w_t-w_p| ||q_p,h|| + |w_t| ||q_t,h-q_p,h|| (reference certified.py:18-48,
//      one key vector shared by the heads) plus a rounding slack, q/w kept for the next
//      step, per-block bounds U_b + maxnorm_b * c (blocks with new keys: +inf, as
//      replay.py:263-266), and wave 1 = the blocks holding a previous top-k key or new keys
//      (hot first, replay.py:153-169) -- every block when those leave at most 1/16 out;
//   2. wave 1 scored on the tensor cores; the epilogue adds every score to the row's key
//      histogram and writes the exact block maxima;
//   3. wave2 (one CTA per sequence): tau = the lower edge of the key bin holding the k-th
//      largest wave-1 score (>= the seed threshold min(current[prev_topk])), wave 2 = the
//      other blocks whose bound reaches tau; the rest are pruned unread, their keys set to
//      -inf and counted in the histogram; statistics;
//   4. wave 2 scored (histogram as in 2);
//   5. top-k over the row from its histogram, the indices also kept as the next step's seeds.
// Every pruned key has a score strictly below tau <= the k-th largest, so the top-k equals
// dense scoring's; the scores are bit-identical to the dense kernel's (same MMA tile, same
// epilogue summation order).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "tiles.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 1024;
constexpr double kGamma = 0x1p-12;  // relative rounding slack of a computed score
constexpr int kFoldKeys = 1024;     // appends up to this many keys are normed in prepare
constexpr uint32_t kNegInfBin = 0x007FFFFFu >> 20;  // histogram bin of the -inf key

// Squared norm of key `key`, rounded up, folded into its block's max (float bits of
// non-negative floats order like unsigned integers).  Called by one whole warp.
__device__ __forceinline__ void fold_key_norm(const void* keys, int64_t base, int64_t k_rs,
                                              int dtype, int key, int bs, uint32_t* maxsq_row) {
  const int lane = threadIdx.x & 31;
  // 4 dims per lane in one 8-byte load (rows are 16-byte aligned: TMA layout rules)
  const uint2 raw = *reinterpret_cast<const uint2*>(
      static_cast<const uint16_t*>(keys) + base + static_cast<int64_t>(key) * k_rs + lane * 4);
  const uint16_t e[4] = {static_cast<uint16_t>(raw.x & 0xFFFFu), static_cast<uint16_t>(raw.x >> 16),
                         static_cast<uint16_t>(raw.y & 0xFFFFu), static_cast<uint16_t>(raw.y >> 16)};
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float v = dtype == TDSA_BF16 ? __uint_as_float(static_cast<uint32_t>(e[j]) << 16)
                                       : __half2float(__ushort_as_half(e[j]));
    s = __fadd_ru(s, __fmul_ru(v, v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_ru(s, __shfl_xor_sync(0xffffffffu, s, o));
  if (lane == 0) atomicMax(&maxsq_row[key / bs], __float_as_uint(s));
}

// Norms of many appended keys (the first step, or a large append): one warp per key.
__global__ void new_key_norms_kernel(const void* keys, int64_t k_bs, int64_t k_rs, int dtype,
                                     int first_key, int length, int bs, uint32_t* maxsq,
                                     int64_t nb_stride) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int warps = (blockDim.x >> 5) * gridDim.x;
  for (int key = first_key + blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); key < length;
       key += warps)
    fold_key_norm(keys, static_cast<int64_t>(b) * k_bs, k_rs, dtype, key, bs,
                  maxsq + static_cast<int64_t>(b) * nb_stride);
}

struct PrepArgs {
  const void* q;
  int64_t q_bs;
  const float* w;
  int64_t w_bs;
  void* qprev;   // [B][8192] 16-bit
  float* wprev;  // [B][64]
  const void* keys;
  int64_t k_bs, k_rs;
  int dtype;
  int prev_length, length, bs, bpt, k;
  int fold_norms;  // 1: the keys [prev_length, length) are normed here
  int64_t nb_stride;
  float* upper;
  uint32_t* maxsq;
  const float* bmax;
  const int32_t* prev_topk;
  float* bound;
  int8_t* flag;
  int32_t* tile_seq;
  int32_t* tile_blk;
  int32_t* counters;  // [0]: wave-1 tiles (zero on entry), [1]: wave-2 tiles (zeroed here)
  unsigned long long* stats;
  int init;  // 1: every block is scored (first step)
};

// Blocks (and previous top-k entries) whose loads a thread issues before any barrier: the
// whole state of a sequence of up to 2048 blocks arrives in one round trip.
constexpr int kPrepUnroll = 2;
// When wave 1 already covers all but at most 1/kAllHotFraction of a sequence's blocks, the
// rest join wave 1 too: the few blocks left could not pay for tau and a second wave (on
// i.i.d. caches the previous top-2048 touch nearly every block and nothing is pruned), and
// scoring a block never changes the top-k.
constexpr int kAllHotFraction = 16;

__global__ void __launch_bounds__(kThreads) exact_prepare_kernel(const PrepArgs a) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  extern __shared__ int8_t hot[];  // [nb]: this step's wave-1 flags
  __shared__ double wsum[32];
  __shared__ int s_cold;  // blocks outside wave 1
  static_assert(kThreads == 8192 / 8, "one thread per 8 query elements");
  __shared__ uint32_t wtot[32];
  __shared__ uint32_t sbase[4];
  const int seq = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (a.length + a.bs - 1) / a.bs;
  // blocks holding keys appended since the last step are never pruned (replay.py:263-266)
  const int first_new = a.init ? 0 : (a.length > a.prev_length ? a.prev_length / a.bs : nb);
  const int64_t brow = static_cast<int64_t>(seq) * a.nb_stride;
  if (seq == 0 && tid == 0) a.counters[1] = 0;  // wave 2's list (used after this)
  if (tid == 0) s_cold = 0;

  // ---- every load of the step's state, issued before the first barrier.  Thread t owns q
  // elements [8t, 8t + 8) (one 16-byte load; rows are 16-byte aligned: the scoring kernels'
  // TMA rules), 16 threads per head, blocks t + 1024 j and previous top-k entries t + 1024 j.
  const int h = tid >> 4;
  const uint4 qv = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.q) +
                                                  static_cast<int64_t>(seq) * a.q_bs)[tid];
  uint4* qp4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.qprev) +
                                        static_cast<int64_t>(seq) * 8192) + tid;
  const float wn = a.w[static_cast<int64_t>(seq) * a.w_bs + h];
  float* wp_row = a.wprev + static_cast<int64_t>(seq) * 64;
  uint4 pv = make_uint4(0u, 0u, 0u, 0u);
  float wp = 0.f;
  int8_t pflag[kPrepUnroll] = {};
  float pmax[kPrepUnroll] = {}, pbound[kPrepUnroll] = {};
  uint32_t pnsq[kPrepUnroll] = {};
  int32_t ptop[kPrepUnroll] = {-1, -1};
  if (!a.init) {
    pv = *qp4;
    wp = wp_row[h];
#pragma unroll
    for (int j = 0; j < kPrepUnroll; ++j) {
      const int b = tid + j * kThreads;
      if (b < first_new) {
        pflag[j] = a.flag[brow + b];
        pmax[j] = a.bmax[brow + b];
        pbound[j] = a.bound[brow + b];
        pnsq[j] = a.maxsq[brow + b];
      }
      const int i = tid + j * kThreads;
      ptop[j] = i < a.k ? a.prev_topk[static_cast<int64_t>(seq) * a.k + i] : -1;
    }
  }
  if (a.fold_norms) {  // few appended keys: one warp per key, into blocks >= first_new
    for (int key = a.prev_length + warp; key < a.length; key += kThreads / 32)
      fold_key_norm(a.keys, static_cast<int64_t>(seq) * a.k_bs, a.k_rs, a.dtype, key, a.bs,
                    a.maxsq + brow);
  }

  // ---- certified coefficient c = sum_h |w_t-w_p| ||q_p,h|| + |w_t| ||q_t,h-q_p,h|| plus
  // the rounding slack, in float64; the 64 head terms are summed in a fixed order (pairs
  // of heads per warp, then the 32 warp sums)
  if (!a.init) {
    const uint32_t nw[4] = {qv.x, qv.y, qv.z, qv.w}, pw[4] = {pv.x, pv.y, pv.z, pv.w};
    double dd = 0.0, pp = 0.0, nn = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint16_t nb16 = static_cast<uint16_t>(nw[j >> 1] >> (16 * (j & 1)));
      const uint16_t pb16 = static_cast<uint16_t>(pw[j >> 1] >> (16 * (j & 1)));
      const double qn = a.dtype == TDSA_BF16 ? __uint_as_float(static_cast<uint32_t>(nb16) << 16)
                                             : __half2float(__ushort_as_half(nb16));
      const double qpv = a.dtype == TDSA_BF16 ? __uint_as_float(static_cast<uint32_t>(pb16) << 16)
                                              : __half2float(__ushort_as_half(pb16));
      dd += (qn - qpv) * (qn - qpv);
      pp += qpv * qpv;
      nn += qn * qn;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      dd += __shfl_xor_sync(0xffffffffu, dd, o);
      pp += __shfl_xor_sync(0xffffffffu, pp, o);
      nn += __shfl_xor_sync(0xffffffffu, nn, o);
    }
    double term = 0.0;
    if ((tid & 15) == 0) {
      const double wpd = wp;
      const double nqp = sqrt(pp), nqn = sqrt(nn), ndq = sqrt(dd);
      term = fabs(wn - wpd) * nqp + fabs(wn) * ndq + kGamma * (fabs(wn) * nqn + fabs(wpd) * nqp);
    }
    term += __shfl_xor_sync(0xffffffffu, term, 16);  // heads 2 warp and 2 warp + 1
    if (lane == 0) wsum[warp] = term;
  }
  *qp4 = qv;  // kept for the next step (this thread read the old copy above)
  // wave 1 starts as the blocks with new keys (every block at the first step)
  for (int b = tid; b < nb; b += kThreads) hot[b] = (a.init || b >= first_new) ? 1 : 0;
  __syncthreads();  // every read of wprev; the warp sums; hot[] prefilled
  if ((tid & 15) == 0) wp_row[h] = wn;
  if (!a.init) {
    // the 32 warp sums reduced by a butterfly in a fixed order (every warp alike)
    double c = wsum[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    const double c_total = c * (1.0 + 0x1p-40);
    // the blocks holding a previous top-k key join wave 1 (hot first, replay.py:153-169)
#pragma unroll
    for (int j = 0; j < kPrepUnroll; ++j) {
      const int blk = ptop[j] >= 0 ? ptop[j] / a.bs : -1;
      if (blk >= 0 && blk < nb) hot[blk] = 1;
    }
    for (int i = tid + kPrepUnroll * kThreads; i < a.k; i += kThreads) {
      const int32_t t = a.prev_topk[static_cast<int64_t>(seq) * a.k + i];
      const int blk = t >= 0 ? t / a.bs : -1;
      if (blk >= 0 && blk < nb) hot[blk] = 1;
    }
    // the previous step's state update (U_b <- exact block max of a scored block, its
    // bound when pruned), then this step's bound U_b + maxnorm_b * c; a block below
    // first_new (<= the previous step's block count) existed at the previous step
    auto update = [&](int b, int8_t f, float bm, float bo, uint32_t nsq) {
      float bnd = INFINITY;
      if (b < first_new) {
        const float u = f ? bm : bo;
        a.upper[brow + b] = u;
        const double nrm = static_cast<double>(__fsqrt_ru(__uint_as_float(nsq)));
        bnd = __double2float_ru(static_cast<double>(u) + nrm * c_total);
      }
      a.bound[brow + b] = bnd;
    };
#pragma unroll
    for (int j = 0; j < kPrepUnroll; ++j) {
      const int b = tid + j * kThreads;
      if (b < nb) update(b, pflag[j], pmax[j], pbound[j], pnsq[j]);
    }
    for (int b = tid + kPrepUnroll * kThreads; b < nb; b += kThreads) {
      if (b < first_new)
        update(b, a.flag[brow + b], a.bmax[brow + b], a.bound[brow + b], a.maxsq[brow + b]);
      else
        update(b, 0, 0.f, 0.f, 0u);
    }
  } else {
    for (int b = tid; b < nb; b += kThreads) a.bound[brow + b] = INFINITY;
    if (tid == 0) {  // the first step scores every block (adds that return nothing)
      unsigned long long* st = a.stats + static_cast<int64_t>(seq) * 8;
      atomicAdd(&st[0], 1ull);
      atomicAdd(&st[1], static_cast<unsigned long long>(nb));
      atomicAdd(&st[2], static_cast<unsigned long long>(nb));
      atomicAdd(&st[4], static_cast<unsigned long long>(a.length));
      atomicAdd(&st[5], static_cast<unsigned long long>(a.length));
      atomicAdd(&st[6], static_cast<unsigned long long>(nb));
    }
  }
  __syncthreads();  // hot[] complete
  if (!a.init) {
    int cold = 0;
    for (int b = tid; b < nb; b += kThreads) cold += hot[b] == 0;
    cold = __reduce_add_sync(0xffffffffu, cold);
    if ((tid & 31) == 0 && cold) atomicAdd(&s_cold, cold);
    __syncthreads();
    if (s_cold > 0 && s_cold * kAllHotFraction <= nb) {  // (the same for the whole CTA)
      for (int b = tid; b < nb; b += kThreads) hot[b] = 1;
      __syncthreads();
    }
  }
  for (int b = tid; b < nb; b += kThreads) a.flag[brow + b] = hot[b];
  emit_tiles(hot, nb, 1, a.bpt, seq, a.tile_seq, a.tile_blk, a.counters, wtot, sbase);
}

constexpr int kHistCopies = 8;  // private copies of the row histogram (one per 4 warps)
constexpr int kHistCopyBytes = kHistCopies * kKeyHistBins * 4;
// largest dynamic shared memory of the prepare and wave-2 kernels (one flag byte per block,
// after wave 2's 16 KB of sub-bin counts)
constexpr int kWave2MaxSmem = 200 * 1024;
constexpr int kMaxHistSegs = 64;  // 32768-key histogram segments per sequence (2^21 keys)
static_assert(kTopkSegment == 1 << 15, "a key's histogram segment is its index >> 15");

// Counts the 4096-bin key histogram (top 12 bits of the order-preserving key) of one score
// row into h[0, 4096) (shared memory).  Finite scores go to eight private copies in `hc`
// (kHistCopies x 4096 words, one per 4 warps) that are summed at the end, so clustered
// scores do not serialise on a few words; -inf (unscored keys) is counted apart.  Loads
// are coalesced (thread t reads t, t + 1024, ...).  Returns the -inf count.
__device__ uint32_t row_histogram(const float* srow, int length, uint32_t* h, uint32_t* hc) {
  __shared__ uint32_t s_inf;
  for (int i = threadIdx.x; i < kHistCopies * kKeyHistBins; i += kThreads) hc[i] = 0u;
  if (threadIdx.x == 0) s_inf = 0u;
  __syncthreads();
  uint32_t* mine = hc + ((threadIdx.x >> 5) & (kHistCopies - 1)) * kKeyHistBins;
  uint32_t inf = 0;
  const int span = (length + 31) & ~31;  // whole warps iterate together
  for (int i = threadIdx.x; i < span; i += kThreads) {
    const float v = i < length ? srow[i] : -INFINITY;
    if (i < length && v == -INFINITY) ++inf;
    add_to_bin(mine, v != -INFINITY, v != -INFINITY ? float_to_key(v) >> 20 : 0u);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) inf += __shfl_xor_sync(0xffffffffu, inf, o);
  if ((threadIdx.x & 31) == 0 && inf) atomicAdd(&s_inf, inf);
  __syncthreads();
  for (int i = threadIdx.x; i < kKeyHistBins; i += kThreads) {
    uint32_t t = 0;
#pragma unroll
    for (int c = 0; c < kHistCopies; ++c) t += hc[c * kKeyHistBins + i];
    h[i] = t;
  }
  __syncthreads();
  return s_inf;
}

// Wave 2: blocks not scored yet whose bound reaches tau.  tau is the lower edge of the key
// bin (top 12 bits from the wave-1 histogram, then the next 12 bits inside that bin) that
// holds the k-th largest wave-1 score: at most that score, so every block pruned against it
// holds no top-k key.  Pruned keys are set to -inf in the score row and counted in the -inf
// bin of their segment's histogram, which the top-k then consumes (and clears).
struct Wave2Args {
  int length, bs, bpt, k;
  int64_t nb_stride, l_stride;
  const float* bound;
  float* scores;
  float* tau;
  int8_t* flag;
  int32_t* tile_seq;
  int32_t* tile_blk;
  int32_t* counters;  // [1]: wave-2 tiles; [0] is cleared for the next step's wave 1
  uint32_t* hist;     // [B][hist_segs][4096]: the wave-1 scores' key histograms, one per
                      // 32768-key segment of the row
  int hist_segs;
  unsigned long long* stats;
};

constexpr int kW2Vec = 8;  // 16-byte score pieces per thread per pass (32768 keys per CTA)

// One step of a CTA-wide selection from the top of a 4096-bin histogram: thread t holds bins
// 4095-4t .. 4092-4t in c[0..3].  Returns true in the one thread whose bins hold the kk-th
// largest key, with that bin and the key's rank inside it (from the top); no thread does
// when fewer than kk keys are counted.  `wtot` (32 words) is free on entry; the caller
// passes a barrier before it is reused.
__device__ __forceinline__ bool select_bin(const uint32_t (&c)[4], uint32_t kk, uint32_t* wtot,
                                           uint32_t& bin, uint32_t& rank) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t tot = c[0] + c[1] + c[2] + c[3];
  uint32_t x = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  // keys in the earlier warps: an inclusive scan of the 32 warp totals, read at warp - 1
  uint32_t wt = wtot[lane];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, wt, o);
    if (lane >= o) wt += y;
  }
  const uint32_t earlier = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
  uint32_t above = x - tot + (warp ? earlier : 0u);
  bool found = false;
  if (above < kk && kk <= above + tot) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (!found && kk <= above + c[i]) {
        bin = kKeyHistBins - 1 - (4 * threadIdx.x + i);
        rank = kk - above;
        found = true;
      }
      above += c[i];
    }
  }
  return found;
}

// Adds the scored keys of bin `bin1` among four scores to the sub-bin histogram (the next 12
// key bits).  The keys of one bin are few (a few percent of the row) and spread over 4096
// sub-bins, so every lane adds alone.  With kFloat the bin test compares the floats with the
// bin's smallest and largest float [f_lo, f_hi] (two compares per key; the key is formed
// only for the keys inside), which is exact for bins of finite nonzero floats: the key map is
// monotone there.  The pass runs on one SM per sequence and is bound by its integer pipe.
template <bool kFloat>
__device__ __forceinline__ void add_sub_bins(uint32_t* h2, float4 v, bool scored, uint32_t bin1,
                                             float f_lo, float f_hi) {
  const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const bool in = kFloat ? scored && e[u] >= f_lo && e[u] <= f_hi
                           : scored && (float_to_key(e[u]) >> 20) == bin1;
    if (in) atomicAdd(&h2[(float_to_key(e[u]) >> 8) & 0xFFFu], 1u);
  }
}

// Level 2 of tau over a row held partly in registers (v: pieces tid + 1024 j of the first
// 32768 keys) and the rest read here.
template <bool kFloat>
__device__ __forceinline__ void sub_bin_pass(uint32_t* h2, const float4 (&v)[8], const float* srow,
                                             int nvec, const int8_t* sflag, int bshift,
                                             uint32_t bin1, float f_lo, float f_hi) {
  const int tid = threadIdx.x;
  const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j * 1024 < nvec) {  // uniform: rows shorter than 32768 keys skip the empty pieces
      const int i = tid + j * 1024;
      add_sub_bins<kFloat>(h2, v[j], i < nvec && sflag[(4 * i) >> bshift] == 1, bin1, f_lo, f_hi);
    }
  }
  for (int base = 8 * 1024; base < nvec; base += 8 * 1024) {
    float4 w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + tid + j * 1024;
      w[j] = i < nvec ? reinterpret_cast<const float4*>(srow)[i] : ninf;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + tid + j * 1024;
      add_sub_bins<kFloat>(h2, w[j], i < nvec && sflag[(4 * i) >> bshift] == 1, bin1, f_lo, f_hi);
    }
  }
}

__global__ void __launch_bounds__(kThreads) exact_wave2_kernel(const Wave2Args a) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  extern __shared__ uint32_t dyn[];  // the 4096 sub-bin counts, then the row's block flags
  uint32_t* h2 = dyn;
  int8_t* sflag = reinterpret_cast<int8_t*>(dyn + kKeyHistBins);  // [nb]
  __shared__ uint32_t wtot[32];
  __shared__ uint32_t sbase[4];
  __shared__ uint32_t acc[5];
  __shared__ float s_tau;
  __shared__ uint32_t s_bin, s_rank;
  __shared__ uint32_t seg_pruned[kMaxHistSegs];  // pruned keys per segment
  const int seq = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int nb = (a.length + a.bs - 1) / a.bs;
  const int64_t brow = static_cast<int64_t>(seq) * a.nb_stride;
  float* srow = a.scores + static_cast<int64_t>(seq) * a.l_stride;
  uint32_t* grow = a.hist + static_cast<int64_t>(seq) * a.hist_segs * kKeyHistBins;
  // the row in 16-byte pieces when its base allows (bs is a multiple of 4, so a piece lies
  // in one block)
  const bool vec = (reinterpret_cast<uintptr_t>(srow) & 15u) == 0u;
  const int nvec = vec ? a.length >> 2 : 0;
  const int bshift = __ffs(a.bs) - 1;  // block sizes are powers of two
  const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);

  // ---- loads issued together: this thread's 4 bins of every segment histogram, the
  // bounds of blocks tid and tid + 1024, the row's flags and its first 32768 scores
  // (pieces tid + 1024 j, read whatever their block: unscored ones are masked later)
  uint32_t c[4] = {0u, 0u, 0u, 0u};
  for (int g = 0; g < a.hist_segs; ++g) {
    const uint4 t = reinterpret_cast<const uint4*>(grow + g * kKeyHistBins)[kThreads - 1 - tid];
    c[0] += t.w;
    c[1] += t.z;
    c[2] += t.y;
    c[3] += t.x;
  }
  float pb[2];
  int8_t pf[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int b = tid + j * kThreads;
    pb[j] = b < nb ? a.bound[brow + b] : 0.f;
    pf[j] = b < nb ? a.flag[brow + b] : 0;
  }
  float4 v[kW2Vec];
#pragma unroll
  for (int j = 0; j < kW2Vec; ++j) {
    const int i = tid + j * kThreads;
    v[j] = i < nvec ? reinterpret_cast<const float4*>(srow)[i] : ninf;
  }
#pragma unroll
  for (int j = 0; j < 2; ++j)
    if (tid + j * kThreads < nb) sflag[tid + j * kThreads] = pf[j];
  for (int b = tid + 2 * kThreads; b < nb; b += kThreads) sflag[b] = a.flag[brow + b];
  for (int i = tid; i < kKeyHistBins; i += kThreads) h2[i] = 0u;
  if (seq == 0 && tid == 0) a.counters[0] = 0;  // wave 1 of this step is done
  if (tid < 5) acc[tid] = 0u;
  if (tid < kMaxHistSegs) seg_pruned[tid] = 0u;
  if (tid == 0) {
    s_bin = 0xFFFFFFFFu;
    s_tau = -INFINITY;  // fewer than k wave-1 scores: prune nothing
  }
  // a row whose blocks were all scored in wave 1 has nothing to prune: no tau
  bool unscored = false;
#pragma unroll
  for (int j = 0; j < 2; ++j) unscored |= tid + j * kThreads < nb && pf[j] == 0;
  for (int b = tid + 2 * kThreads; b < nb; b += kThreads) unscored |= sflag[b] == 0;
  const bool any_unscored = __syncthreads_or(unscored) != 0;

  // ---- level 1: the bin holding the k-th largest wave-1 score
  uint32_t bin, rank;
  if (any_unscored && select_bin(c, static_cast<uint32_t>(a.k), wtot, bin, rank)) {
    s_bin = bin;
    s_rank = rank;
  }
  __syncthreads();
  const uint32_t bin1 = s_bin;
  if (bin1 != 0xFFFFFFFFu && bin1 != 0u) {
    // level 2: the next 12 key bits of the wave-1 keys in that bin (the row holds stale
    // scores outside the wave-1 blocks) narrow tau to 2^8 keys.  Bins of finite nonzero
    // floats (8 .. 0xFF7 but not the two holding zero) test the floats themselves.
    static_assert(kW2Vec == 8 && kThreads == 1024, "sub_bin_pass layout");
    const float f_lo = key_to_float(bin1 << 20), f_hi = key_to_float((bin1 << 20) | 0xFFFFFu);
    if (bin1 >= 8u && bin1 <= 0xFF7u && bin1 != 0x7FFu && bin1 != 0x800u)
      sub_bin_pass<true>(h2, v, srow, nvec, sflag, bshift, bin1, f_lo, f_hi);
    else
      sub_bin_pass<false>(h2, v, srow, nvec, sflag, bshift, bin1, f_lo, f_hi);
    // the keys past the 16-byte pieces (all of them when the row is not 16-byte aligned)
    for (int base = 4 * nvec; base < a.length; base += kThreads) {
      const int i = base + tid;
      const bool scored = i < a.length && sflag[i >> bshift] == 1;
      const uint32_t key = float_to_key(scored ? srow[i] : -INFINITY);
      if (scored && (key >> 20) == bin1) atomicAdd(&h2[(key >> 8) & 0xFFFu], 1u);
    }
    __syncthreads();
    const uint4 t = reinterpret_cast<const uint4*>(h2)[kThreads - 1 - tid];
    const uint32_t d[4] = {t.w, t.z, t.y, t.x};
    if (select_bin(d, s_rank, wtot, bin, rank)) {
      const uint32_t lo = (bin1 << 20) | (bin << 8);
      // the smallest key of the sub-bin as a float (past +inf only NaN: +inf)
      s_tau = lo > 0xFF800000u ? INFINITY : key_to_float(lo);
    }
    __syncthreads();
  }
  const float tau = s_tau;
  if (tid == 0) a.tau[seq] = tau;

  // ---- wave 2: unscored blocks whose bound reaches tau; the rest are pruned
  uint32_t scored = 0, keys = 0, hot = 0, second = 0, pruned_keys = 0;
  auto decide = [&](int b, float bound) -> uint32_t {
    int8_t f = sflag[b];
    if (f == 0 && bound >= tau) {
      f = 2;
      sflag[b] = 2;
      a.flag[brow + b] = 2;
    }
    const uint32_t n = static_cast<uint32_t>(min(a.bs, a.length - b * a.bs));
    if (f) {
      ++scored;
      keys += n;
      hot += f == 1;
      second += f == 2;
    } else {
      pruned_keys += n;
    }
    return f ? 0u : n;
  };
  // pruned keys per histogram segment: a warp's 32 consecutive blocks span at most two
  auto seg_add = [&](int b, uint32_t n) {
    const int seg = b < nb ? (b * a.bs) >> 15 : -1;
    const int seg0 = __shfl_sync(0xffffffffu, seg, 0);
    const uint32_t lo = __reduce_add_sync(0xffffffffu, seg == seg0 ? n : 0u);
    const uint32_t hi = __reduce_add_sync(0xffffffffu, seg != seg0 ? n : 0u);
    const int seg31 = __shfl_sync(0xffffffffu, seg, 31);
    if (lane == 0) {
      if (lo && seg0 >= 0) atomicAdd(&seg_pruned[seg0], lo);
      if (hi) atomicAdd(&seg_pruned[seg31 >= 0 ? seg31 : seg0 + 1], hi);
    }
  };
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int b = tid + j * kThreads;
    if (j * kThreads < nb) seg_add(b, b < nb ? decide(b, pb[j]) : 0u);
  }
  for (int b0 = 2 * kThreads; b0 < nb; b0 += kThreads) {
    const int b = b0 + tid;
    seg_add(b, b < nb ? decide(b, a.bound[brow + b]) : 0u);
  }
  // warp sums first (a row's counts fit 32 bits), then one shared add per warp and count
  scored = __reduce_add_sync(0xffffffffu, scored);
  keys = __reduce_add_sync(0xffffffffu, keys);
  hot = __reduce_add_sync(0xffffffffu, hot);
  second = __reduce_add_sync(0xffffffffu, second);
  pruned_keys = __reduce_add_sync(0xffffffffu, pruned_keys);
  if (lane == 0) {
    atomicAdd(&acc[0], scored);
    atomicAdd(&acc[1], keys);
    atomicAdd(&acc[2], hot);
    atomicAdd(&acc[3], second);
    atomicAdd(&acc[4], pruned_keys);
  }
  __syncthreads();
  // the wave-2 list's place: the atomic is in flight while the pruned keys are filled
  if (tid == 0) {
    const uint32_t ntiles = (acc[3] + a.bpt - 1) / a.bpt;
    if (gridDim.x == 1) {
      sbase[3] = 0u;
      a.counters[1] = static_cast<int32_t>(ntiles);  // zeroed by this step's prepare
    } else {
      sbase[3] = ntiles ? static_cast<uint32_t>(atomicAdd(&a.counters[1], static_cast<int>(ntiles)))
                        : 0u;
    }
  }
  // pruned keys score -inf (the top-k reads the whole row)
  if (acc[4]) {
    for (int i = tid; i < nvec; i += kThreads)
      if (sflag[(4 * i) >> bshift] == 0) reinterpret_cast<float4*>(srow)[i] = ninf;
    for (int i = 4 * nvec + tid; i < a.length; i += kThreads)
      if (sflag[i >> bshift] == 0) srow[i] = -INFINITY;
  }
  if (tid < a.hist_segs && seg_pruned[tid])
    atomicAdd(&grow[tid * kKeyHistBins + kNegInfBin], seg_pruned[tid]);
  if (tid == 0) {  // adds that return nothing: no thread waits on a read
    unsigned long long* st = a.stats + static_cast<int64_t>(seq) * 8;
    using ull = unsigned long long;
    atomicAdd(&st[0], 1ull);                                // steps
    atomicAdd(&st[1], static_cast<ull>(nb));                // blocks visited
    atomicAdd(&st[2], static_cast<ull>(acc[0]));            // blocks scored
    atomicAdd(&st[3], static_cast<ull>(nb - acc[0]));       // blocks pruned
    atomicAdd(&st[4], static_cast<ull>(acc[1]));            // keys scored (read)
    atomicAdd(&st[5], static_cast<ull>(a.length));          // keys in the cache
    atomicAdd(&st[6], static_cast<ull>(acc[2]));            // first-wave (hot) blocks
    atomicAdd(&st[7], static_cast<ull>(acc[3]));            // second-wave blocks
  }
  emit_tiles(sflag, nb, 2, a.bpt, seq, a.tile_seq, a.tile_blk, a.counters + 1, wtot, sbase,
             &sbase[3]);
}

// Part of a row's key histogram, added to hist[seq] (zero before the launch): CTA
// blockIdx.x of gridDim.x takes one contiguous chunk of the row, so a small batch still
// spreads over many SMs.  Finite scores by bin; the unscored (-inf) keys are counted in
// the bin of the -inf key itself (0x007FFFFF >> 20 = 7), as the cluster top-k expects.
__global__ void __launch_bounds__(kThreads)
    row_hist_part_kernel(const float* scores, int64_t l_stride, int length, uint32_t* hist) {
  pdl_wait();  // every global access follows the previous kernel
  pdl_launch_dependents();
  extern __shared__ uint32_t hcopies[];  // kHistCopies x 4096 words
  __shared__ uint32_t h[kKeyHistBins];
  const int seq = blockIdx.y;
  const int chunk = ((length + gridDim.x - 1) / gridDim.x + 31) & ~31;
  const int lo = min(length, static_cast<int>(blockIdx.x) * chunk);
  const int n = min(chunk, length - lo);
  const uint32_t inf =
      row_histogram(scores + static_cast<int64_t>(seq) * l_stride + lo, n, h, hcopies);
  uint32_t* dst = hist + static_cast<int64_t>(seq) * kKeyHistBins;
  for (int i = threadIdx.x; i < kKeyHistBins; i += kThreads) {
    const uint32_t c = h[i] + (i == (0x007FFFFFu >> 20) ? inf : 0u);
    if (c) atomicAdd(dst + i, c);
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

int launch_row_hist_parts(const float* scores, int64_t l_stride, int batch, int length,
                          uint32_t* hist, cudaStream_t stream) {
  const int parts = std::max(1, std::min({16, device_sm_count(current_device()) / batch, (length + 2047) / 2048}));
  TDSA_CUDA_CHECK(cudaMemsetAsync(hist, 0, static_cast<size_t>(batch) * kKeyHistBins * 4,
                                  stream));
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(row_hist_part_kernel),
                                      kHistCopyBytes));
  TDSA_CUDA_CHECK(launch_pdl(row_hist_part_kernel, dim3(parts, batch), dim3(kThreads),
                             kHistCopyBytes, stream, scores, l_stride, length, hist));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

ExactLayout exact_layout(int batch, int max_length, int k, int block_size) {
  ExactLayout L;
  L.nb_stride = (max_length + block_size - 1) / block_size;
  L.bpt = 128 / block_size;
  L.tcap = static_cast<int64_t>(batch) * ((L.nb_stride + L.bpt - 1) / L.bpt);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t nbt = static_cast<size_t>(batch) * L.nb_stride;
  L.upper = take(nbt * 4);
  L.maxsq = take(nbt * 4);
  L.bound = take(nbt * 4);
  L.bmax = take(nbt * 4);
  L.flag = take(nbt);
  L.topk = take(static_cast<size_t>(batch) * k * 4);
  L.qprev = take(static_cast<size_t>(batch) * 8192 * 2);
  L.wprev = take(static_cast<size_t>(batch) * 64 * 4);
  L.scores = take(static_cast<size_t>(batch) * max_length * 4);
  L.tau = take(static_cast<size_t>(batch) * 4);
  L.stats = take(static_cast<size_t>(batch) * 8 * 8);
  L.tile_seq = take(static_cast<size_t>(L.tcap) * 4);
  L.tile_blk = take(static_cast<size_t>(L.tcap) * L.bpt * 4);
  L.counters = take(16);
  const size_t segs = (static_cast<size_t>(max_length) + kTopkSegment - 1) / kTopkSegment;
  L.hist = take(static_cast<size_t>(batch) * segs * kKeyHistBins * 4);
  L.topk_ws_bytes = topk_workspace_bytes(batch, max_length, k);
  L.topk_ws = take(L.topk_ws_bytes);
  L.total = off;
  return L;
}

int run_exact(int init, uint8_t* state, const ExactLayout& L, const void* q, int64_t q_bs,
              const float* w, int64_t w_bs, const void* keys, int64_t k_bs, int64_t k_rs,
              int dtype, int batch, int prev_length, int length, int max_length, int k,
              int block_size, int sorted, void* out_idx, int idx_bytes, int64_t idx_bs,
              float* out_val, int64_t val_bs, cudaStream_t stream) {
  const int bpt = 128 / block_size;
  float* upper = reinterpret_cast<float*>(state + L.upper);
  uint32_t* maxsq = reinterpret_cast<uint32_t*>(state + L.maxsq);
  float* bound = reinterpret_cast<float*>(state + L.bound);
  float* bmax = reinterpret_cast<float*>(state + L.bmax);
  int8_t* flag = reinterpret_cast<int8_t*>(state + L.flag);
  int32_t* topk = reinterpret_cast<int32_t*>(state + L.topk);
  void* qprev = state + L.qprev;
  float* wprev = reinterpret_cast<float*>(state + L.wprev);
  float* scores = reinterpret_cast<float*>(state + L.scores);
  float* tau = reinterpret_cast<float*>(state + L.tau);
  auto* stats = reinterpret_cast<unsigned long long*>(state + L.stats);
  int32_t* tile_seq = reinterpret_cast<int32_t*>(state + L.tile_seq);
  int32_t* tile_blk = reinterpret_cast<int32_t*>(state + L.tile_blk);
  int32_t* counters = reinterpret_cast<int32_t*>(state + L.counters);
  uint32_t* hist = reinterpret_cast<uint32_t*>(state + L.hist);
  void* tws = state + L.topk_ws;
  // the score waves build one key histogram per 32768-key segment of a row, which the
  // top-k's first level starts from (and clears)
  const int hsegs = (length + kTopkSegment - 1) / kTopkSegment;
  const int max_segs = (max_length + kTopkSegment - 1) / kTopkSegment;
  if (hsegs > kMaxHistSegs)
    return fail(TDSA_ERR_UNSUPPORTED, "exact progressive: at most 2^21 keys per sequence");

  if (init) {
    TDSA_CUDA_CHECK(cudaMemsetAsync(maxsq, 0, static_cast<size_t>(batch) * L.nb_stride * 4,
                                    stream));
    TDSA_CUDA_CHECK(cudaMemsetAsync(stats, 0, static_cast<size_t>(batch) * 64, stream));
    TDSA_CUDA_CHECK(cudaMemsetAsync(counters, 0, 16, stream));
    TDSA_CUDA_CHECK(cudaMemsetAsync(
        hist, 0, static_cast<size_t>(batch) * max_segs * kKeyHistBins * 4, stream));
  }
  // 1. norms of the appended keys: many (the first step) in a kernel of their own, a few
  // inside prepare
  const int first_key = init ? 0 : prev_length;
  const int nkeys = length - first_key;
  const bool fold = !init && nkeys <= kFoldKeys;
  if (nkeys > 0 && !fold) {
    const int blocks_x = std::min(device_sm_count(current_device()), (nkeys + 7) / 8);
    TDSA_CUDA_CHECK(launch_pdl(new_key_norms_kernel, dim3(blocks_x, batch), dim3(256), 0, stream,
                               keys, k_bs, k_rs, dtype, first_key, length, block_size, maxsq,
                               L.nb_stride));
    TDSA_CUDA_CHECK(cudaGetLastError());
  }
  // 2. state update, bounds, flags, wave-1 tiles
  PrepArgs pa;
  pa.q = q;
  pa.q_bs = q_bs;
  pa.w = w;
  pa.w_bs = w_bs;
  pa.qprev = qprev;
  pa.wprev = wprev;
  pa.keys = keys;
  pa.k_bs = k_bs;
  pa.k_rs = k_rs;
  pa.dtype = dtype;
  pa.prev_length = init ? 0 : prev_length;
  pa.length = length;
  pa.bs = block_size;
  pa.bpt = bpt;
  pa.k = k;
  pa.fold_norms = fold ? 1 : 0;
  pa.nb_stride = L.nb_stride;
  pa.upper = upper;
  pa.maxsq = maxsq;
  pa.bmax = bmax;
  pa.prev_topk = topk;
  pa.bound = bound;
  pa.flag = flag;
  pa.tile_seq = tile_seq;
  pa.tile_blk = tile_blk;
  pa.counters = counters;
  pa.stats = stats;
  pa.init = init;
  // dynamic shared memory: one wave-1 flag byte per block
  const int prep_smem = ((length + block_size - 1) / block_size + 15) & ~15;
  if (prep_smem > kWave2MaxSmem)
    return fail(TDSA_ERR_UNSUPPORTED, "exact progressive: too many blocks per sequence");
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(exact_prepare_kernel),
                                      prep_smem));
  TDSA_CUDA_CHECK(launch_pdl(exact_prepare_kernel, dim3(batch), dim3(kThreads), prep_smem,
                             stream, pa));
  TDSA_CUDA_CHECK(cudaGetLastError());

  BlockArgs ba;
  ba.bs = block_size;
  ba.bpt = bpt;
  ba.length = length;
  ba.nblocks = (length + block_size - 1) / block_size;
  ba.tile_seq = tile_seq;
  ba.tile_blocks = tile_blk;
  ba.w = w;
  ba.w_stride = w_bs;
  ba.out = scores;
  ba.out_stride = max_length;
  ba.block_max = bmax;
  ba.bm_stride = L.nb_stride;
  ba.status = device_status_ptr();
  if (!ba.status) return fail(TDSA_ERR_CUDA, "device status word not available");
  const int grid = device_sm_count(current_device());
  // 3. wave 1 (every block at the first step), its scores into the row's segment
  // histograms
  ba.tile_count = counters;
  ba.hist = hist;
  ba.hist_segs = hsegs;
  int rc = launch_score_blocks(kModeExact, q, q_bs, keys, k_bs, k_rs, dtype, batch, ba, grid,
                               stream);
  if (rc) return rc;
  if (init) {
    // the next step's prepare appends its tiles from zero (a step's wave2 kernel clears it)
    TDSA_CUDA_CHECK(cudaMemsetAsync(counters, 0, 4, stream));
  } else {
    // 4. tau, wave-2 list, pruned keys, statistics; 5. wave 2
    Wave2Args wa;
    wa.length = length;
    wa.bs = block_size;
    wa.bpt = bpt;
    wa.k = k;
    wa.nb_stride = L.nb_stride;
    wa.l_stride = max_length;
    wa.bound = bound;
    wa.scores = scores;
    wa.tau = tau;
    wa.flag = flag;
    wa.tile_seq = tile_seq;
    wa.tile_blk = tile_blk;
    wa.counters = counters;
    wa.hist = hist;
    wa.hist_segs = hsegs;
    wa.stats = stats;
    // the sub-bin counts, then the row's block flags
    const int w2_smem = kKeyHistBins * 4 + ((ba.nblocks + 15) & ~15);
    if (w2_smem > kWave2MaxSmem)
      return fail(TDSA_ERR_UNSUPPORTED, "exact progressive: too many blocks per sequence");
    TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(exact_wave2_kernel),
                                        w2_smem));
    TDSA_CUDA_CHECK(launch_pdl(exact_wave2_kernel, dim3(batch), dim3(kThreads), w2_smem,
                               stream, wa));
    TDSA_CUDA_CHECK(cudaGetLastError());
    ba.tile_count = counters + 1;
    rc = launch_score_blocks(kModeExact, q, q_bs, keys, k_bs, k_rs, dtype, batch, ba, grid,
                             stream);
    if (rc) return rc;
  }
  // 6. top-k over the row, each first-level segment from its histogram; the indices are
  // also kept as the next step's seeds
  void* oi = out_idx ? out_idx : topk;
  return launch_topk(scores, max_length, nullptr, 0, batch, length, k, sorted, oi,
                     out_idx ? idx_bytes : 4, out_idx ? idx_bs : k, out_val, val_bs, tws,
                     L.topk_ws_bytes, stream, nullptr, hist,
                     out_idx ? topk : nullptr, k);
}

}  // namespace tdsa
