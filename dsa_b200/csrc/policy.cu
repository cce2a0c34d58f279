// Temporal policy state machine on the device (reference approx.py:112-364 and
// verifier.py:103-375): one CTA per sequence, the state arrays stay in HBM between steps.
//
//   policy_init_kernel      initialize_state (approx.py:112-126) from the step-0 top-k
//   policy_decide_kernel    one step's decisions: the seed (previous top-k) and tau_seed,
//                           per-block maxima and risk, the visiting order, which blocks are
//                           read, and for the verifier the rescued cold blocks; writes the
//                           score row masked to the keys read (-inf elsewhere)
//   (top-k kernel)          the stable top-k of that masked row = the policy's selection
//   policy_finalize_kernel  the next state (metadata of read blocks, ages, cold streaks,
//                           top-k lists) and the step's statistics
//
// The dynamic threshold (the running k-th best score of everything read so far, which
// decides the next block) is sequential over the visiting order.  The CTA walks the order
// in windows of up to 32 positions, holding the running top-k as two ascending lists of
// 64-bit items (a main list of k items and a short pending list of insertions).  Per
// window: one warp per candidate block (a block not already below the threshold) collects
// its unseen items above the threshold; the CTA sorts them (bitonic), merges them into the
// pending list (merge path) and one warp finds the items that drop out (32-way search).
// If every candidate still passes against the threshold after all of them, that is the
// exact outcome (each saw a threshold no higher); otherwise the window is retried one block
// at a time.  The window doubles after each success.  Items are (order-preserving score key << 32) |
// (0xFFFFFFFF - index): larger item = higher score, then lower index, the reference heap's
// order (approx.py:214-236).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace tdsa {

namespace {

constexpr int kPolThreads = 1024;
constexpr int kPendCap = 2048;   // pending list capacity (>= the window capacity)
constexpr int kWindowCap = 1024; // items one window may insert at once (>= a block, 128)
static_assert(kWindowCap <= kPendCap, "a window must fit the pending list");
constexpr int kMaxWindow = 128;  // positions of the visiting order one window may span
static_assert(kMaxWindow % 32 == 0, "whole warps of candidates");

__device__ __forceinline__ uint64_t item_of(float s, int idx) {
  return (static_cast<uint64_t>(float_to_key(s)) << 32) |
         static_cast<uint64_t>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ float item_score(uint64_t it) {
  return key_to_float(static_cast<uint32_t>(it >> 32));
}

// descending order of a double as an ascending 64-bit key (NaN sorts as -inf, -0 as +0)
__device__ __forceinline__ uint64_t desc_key64(double v) {
  if (isnan(v)) v = -INFINITY;
  uint64_t b = static_cast<uint64_t>(__double_as_longlong(v));
  if ((b << 1) == 0) b = 0;
  const uint64_t asc = (b >> 63) ? ~b : (b | 0x8000000000000000ull);
  return ~asc;
}

// numpy's max: any NaN makes the result NaN
__device__ __forceinline__ float nan_max(float a, float b) {
  return (isnan(a) || a > b || isnan(b)) ? (isnan(b) ? b : a) : b;
}

// ascending bitonic sort of (key, idx) pairs, n a power of two, whole CTA
__device__ void cta_sort_pairs(uint64_t* key, uint32_t* idx, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t kl = key[lo], kh = key[hi];
        const bool gt = kl > kh || (kl == kh && idx[lo] > idx[hi]);
        if (gt == up) {
          key[lo] = kh;
          key[hi] = kl;
          const uint32_t t = idx[lo];
          idx[lo] = idx[hi];
          idx[hi] = t;
        }
      }
    }
  }
  __syncthreads();
}

// ascending bitonic sort of keys, n a power of two, whole CTA
__device__ void cta_sort_keys(uint64_t* key, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t kl = key[lo], kh = key[hi];
        if ((kl > kh) == up) {
          key[lo] = kh;
          key[hi] = kl;
        }
      }
    }
  }
  __syncthreads();
}

// number of elements the first d outputs of merge(x, y) take from x (distinct items)
__device__ __forceinline__ int merge_split(const uint64_t* x, int n1, const uint64_t* y, int n2,
                                           int d) {
  int lo = d > n2 ? d - n2 : 0, hi = d < n1 ? d : n1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (x[mid] < y[d - 1 - mid])
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// merge_split by a whole warp: a 32-way search (every lane probes one split point per
// round), the same answer on every lane
__device__ __forceinline__ int warp_split(const uint64_t* x, int n1, const uint64_t* y, int n2,
                                          int d, int lane) {
  int lo = d > n2 ? d - n2 : 0, hi = d < n1 ? d : n1;
  while (lo < hi) {
    const int step = (hi - lo + 31) >> 5;
    const int a = lo + lane * step;
    const bool pred = a < hi && x[a] < y[d - 1 - a];  // true on a prefix of the lanes
    const int cnt = __popc(__ballot_sync(0xffffffffu, pred));
    const int nlo = cnt ? lo + (cnt - 1) * step + 1 : lo;
    const int nhi = (cnt < 32 && lo + cnt * step < hi) ? lo + cnt * step : hi;
    lo = nlo;
    hi = nhi;
  }
  return lo;
}

// out = merge(x[0..n1), y[0..n2)), ascending, by the whole CTA (merge path); ends with a
// barrier
__device__ void cta_merge(const uint64_t* x, int n1, const uint64_t* y, int n2, uint64_t* out) {
  const int n = n1 + n2;
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int d0 = min(n, static_cast<int>(threadIdx.x) * per), d1 = min(n, d0 + per);
  if (d0 < d1) {
    int i = merge_split(x, n1, y, n2, d0), j = d0 - i;
    for (int o = d0; o < d1; ++o) {
      if (j >= n2 || (i < n1 && x[i] < y[j]))
        out[o] = x[i++];
      else
        out[o] = y[j++];
    }
  }
  __syncthreads();
}

__device__ __forceinline__ float block_reduce_min(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

template <typename T>
__device__ __forceinline__ T block_reduce_sum(T v, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : T(0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// sums of N per-thread counters over the CTA in one pass (red: >= 32 * N ints); every
// thread gets the totals
template <int N>
__device__ __forceinline__ void block_reduce_sum_n(int (&v)[N], int* red) {
#pragma unroll
  for (int q = 0; q < N; ++q)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[q] += __shfl_xor_sync(0xffffffffu, v[q], o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int q = 0; q < N; ++q) red[q * 32 + (threadIdx.x >> 5)] = v[q];
  __syncthreads();
  if (threadIdx.x < 32) {
#pragma unroll
    for (int q = 0; q < N; ++q) {
      int x = threadIdx.x < (blockDim.x >> 5) ? red[q * 32 + threadIdx.x] : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (threadIdx.x == 0) red[q * 32] = x;
    }
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < N; ++q) v[q] = red[q * 32];
  __syncthreads();
}

// ascending bitonic sort of up to 64 keys held two per lane (lane l: elements 2l, 2l+1),
// by shuffles; every lane returns its two sorted elements
__device__ __forceinline__ void warp_sort64(uint64_t& x0, uint64_t& x1, int lane) {
  for (int size = 2; size <= 64; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride == 1) {
        const bool up = ((2 * lane) & size) == 0;
        if ((x0 > x1) == up) {
          const uint64_t t = x0;
          x0 = x1;
          x1 = t;
        }
      } else {
        const int ls = stride >> 1;  // partner lane distance
        const uint64_t y0 = __shfl_xor_sync(0xffffffffu, x0, ls);
        const uint64_t y1 = __shfl_xor_sync(0xffffffffu, x1, ls);
        const bool lower = (lane & ls) == 0;
        const bool up = ((2 * lane) & size) == 0;
        // the lower element of each pair keeps min when ascending
        const bool keep_min = lower == up;
        x0 = keep_min ? (x0 < y0 ? x0 : y0) : (x0 > y0 ? x0 : y0);
        x1 = keep_min ? (x1 < y1 ? x1 : y1) : (x1 > y1 ? x1 : y1);
      }
    }
  }
}

// ascending bitonic sort of n keys (a power of two, 64 <= n <= 2 * blockDim.x), two per
// thread (thread t: elements 2t, 2t+1): partners within a warp by shuffles, farther ones
// through shared memory
__device__ void cta_sort_keys_reg(uint64_t* key, int n) {
  __syncthreads();  // the keys were written by other threads
  const int t = threadIdx.x, lane = t & 31;
  // whole warps are active or not (n >= 64); idle warps only meet the barriers
  const bool act = 2 * t < n;
  uint64_t x0 = act ? key[2 * t] : 0ull, x1 = act ? key[2 * t + 1] : 0ull;
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const bool up = ((2 * t) & size) == 0;
      if (stride > 32) {  // partner in another warp: through shared memory
        __syncthreads();
        if (act) {
          key[2 * t] = x0;
          key[2 * t + 1] = x1;
        }
        __syncthreads();
        const int ts2 = stride >> 1;  // partner thread distance
        if (act) {
          const int pt = t ^ ts2;
          const uint64_t y0 = key[2 * pt], y1 = key[2 * pt + 1];
          const bool keep_min = ((t & ts2) == 0) == up;
          x0 = keep_min ? (x0 < y0 ? x0 : y0) : (x0 > y0 ? x0 : y0);
          x1 = keep_min ? (x1 < y1 ? x1 : y1) : (x1 > y1 ? x1 : y1);
        }
      } else if (act) {
        if (stride == 1) {
          if ((x0 > x1) == up) {
            const uint64_t tmp = x0;
            x0 = x1;
            x1 = tmp;
          }
        } else {
          const int ls = stride >> 1;
          const uint64_t y0 = __shfl_xor_sync(0xffffffffu, x0, ls);
          const uint64_t y1 = __shfl_xor_sync(0xffffffffu, x1, ls);
          const bool keep_min = ((lane & ls) == 0) == up;
          x0 = keep_min ? (x0 < y0 ? x0 : y0) : (x0 > y0 ? x0 : y0);
          x1 = keep_min ? (x1 < y1 ? x1 : y1) : (x1 > y1 ? x1 : y1);
        }
      }
    }
  }
  __syncthreads();
  if (act) {
    key[2 * t] = x0;
    key[2 * t + 1] = x1;
  }
  __syncthreads();
}

__device__ __forceinline__ int block_reduce_min_int(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0x7FFFFFFF;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// control state of the dynamic-threshold walk (shared by the CTA)
struct WalkCtl {
  uint64_t T;   // the running minimum item (the threshold)
  double ts;    // its score
  int a_sel, p_sel, ha, na, hp, np;  // main list mains[a_sel][ha..na), pending [hp..np)
  int pos, w, ncand, tot;
  int cand[kMaxWindow], cnt[kMaxWindow], off[kMaxWindow];
};

// shared-memory carve of the decide kernel
struct DecideSmem {
  int words, nb, nbp, kp;
  size_t bits, risk, cmax, fl, skey, sidx, A, A2, P, P2, C, ctl, red, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline int pow2_at_least(int n, int floor_value) {
  int p = floor_value;
  while (p < n) p <<= 1;
  return p;
}

__host__ __device__ inline DecideSmem decide_smem(int length, int bs, int k) {
  DecideSmem d;
  d.words = (length + 31) / 32;
  d.nb = (length + bs - 1) / bs;
  d.nbp = pow2_at_least(d.nb, 32);
  d.kp = pow2_at_least(k, 32);
  size_t o = 0;
  d.risk = o;  o = align_up(o + sizeof(double) * d.nb, 16);
  d.skey = o;  o = align_up(o + sizeof(uint64_t) * d.nbp, 16);
  d.A = o;     o = align_up(o + sizeof(uint64_t) * d.kp, 16);
  d.A2 = o;    o = align_up(o + sizeof(uint64_t) * d.kp, 16);
  d.P = o;     o = align_up(o + sizeof(uint64_t) * kPendCap, 16);
  d.P2 = o;    o = align_up(o + sizeof(uint64_t) * kPendCap, 16);
  d.C = o;     o = align_up(o + sizeof(uint64_t) * kWindowCap, 16);
  d.ctl = o;   o = align_up(o + sizeof(WalkCtl), 16);
  d.bits = o;  o = align_up(o + sizeof(uint32_t) * d.words, 16);
  d.cmax = o;  o = align_up(o + sizeof(float) * d.nb, 16);
  d.sidx = o;  o = align_up(o + sizeof(uint32_t) * d.nbp, 16);
  d.red = o;   o = align_up(o + 32 * 12 * sizeof(int), 16);
  d.fl = o;    o = align_up(o + d.nb, 16);
  d.total = o;
  return d;
}

struct PolicyArgs {
  // state, [batch][k] and [batch][nbc]
  int32_t* topk;
  int32_t* baseline;
  float* last_max;
  float* ema;
  float* vol;
  int16_t* age;
  int16_t* cold;
  int32_t* nblocks;
  int k;
  int nbc;
  // inputs
  const float* scores;
  int64_t s_stride;
  const float* vscores;  // verifier scores (rescue step) or null
  int64_t v_stride;
  int length;
  int prev_length;
  int bs;
  // policy (approx.py:15-39)
  double gamma, ema_alpha, vol_lambda, age_slope;
  int cold_streak, dynamic, order, buckets, age_cap, recent_window, risk_ema;
  int teacher, full_refresh;
  // rescue (verifier.py:173-233)
  int rescue, use_threshold;
  double rescue_fraction, promotion_threshold;
  // workspace and outputs
  float* masked;  // [batch][length] scores of the keys read, -inf elsewhere
  float* cmax;    // [batch][nbc] block maxima of the current scores
  uint8_t* flags;  // [batch][nbc] bit0 forced, bit1 read (refreshed), bit2 rescued
  int32_t* ranking;  // [batch][nbc] rescue ranking (cold blocks first) or null
  uint32_t* ebits;   // [batch][words] keys read (after any rescue)
  int64_t e_stride;
  const int32_t* approx;    // [batch][k] the selection (finalize)
  const int32_t* base_new;  // [batch][k] dense top-k of the current scores (finalize)
  double* stats;            // [batch][TDSA_POLICY_NSTATS]
  int* status;
};

// ---------------------------------------------------------------------------- init
__global__ void __launch_bounds__(kPolThreads) policy_init_kernel(const PolicyArgs a,
                                                                  const int32_t* top) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const float* s = a.scores + b * a.s_stride;
  const int nb = (a.length + a.bs - 1) / a.bs;
  const int64_t so = static_cast<int64_t>(b) * a.nbc;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int blk = warp; blk < nb; blk += kPolThreads / 32) {
    const int lo = blk * a.bs, n = min(a.bs, a.length - lo);
    float m = -INFINITY;
    for (int e = lane; e < n; e += 32) m = nan_max(m, s[lo + e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
      a.last_max[so + blk] = m;
      a.ema[so + blk] = m;
      a.vol[so + blk] = 0.f;
      a.age[so + blk] = 0;
      a.cold[so + blk] = 1;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.k; i += kPolThreads) {
    const int32_t key = top[static_cast<int64_t>(b) * a.k + i];
    a.topk[static_cast<int64_t>(b) * a.k + i] = key;
    a.baseline[static_cast<int64_t>(b) * a.k + i] = key;
    a.cold[so + key / a.bs] = 0;
  }
  if (threadIdx.x == 0) a.nblocks[b] = nb;
}

// ---------------------------------------------------------------------------- decide
__global__ void __launch_bounds__(kPolThreads, 1) policy_decide_kernel(const PolicyArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const DecideSmem d = decide_smem(a.length, a.bs, a.k);
  uint32_t* bits = reinterpret_cast<uint32_t*>(sm + d.bits);
  double* risk = reinterpret_cast<double*>(sm + d.risk);
  float* cmax = reinterpret_cast<float*>(sm + d.cmax);
  uint8_t* fl = sm + d.fl;
  uint64_t* skey = reinterpret_cast<uint64_t*>(sm + d.skey);
  uint32_t* sidx = reinterpret_cast<uint32_t*>(sm + d.sidx);
  uint64_t* A = reinterpret_cast<uint64_t*>(sm + d.A);
  uint64_t* A2 = reinterpret_cast<uint64_t*>(sm + d.A2);
  uint64_t* P = reinterpret_cast<uint64_t*>(sm + d.P);
  uint64_t* P2 = reinterpret_cast<uint64_t*>(sm + d.P2);
  uint64_t* C = reinterpret_cast<uint64_t*>(sm + d.C);
  WalkCtl* ctl = reinterpret_cast<WalkCtl*>(sm + d.ctl);
  double* red = reinterpret_cast<double*>(sm + d.red);
  int* ired = reinterpret_cast<int*>(sm + d.red);

  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = a.length, bs = a.bs, nb = d.nb, k = a.k;
  const int lbs = __ffs(bs) - 1;  // block sizes are powers of two
  const float* s = a.scores + b * a.s_stride;
  const int64_t so = static_cast<int64_t>(b) * a.nbc;
  const int nb_prev = a.nblocks[b];
  double* st = a.stats + static_cast<int64_t>(b) * TDSA_POLICY_NSTATS;

  for (int w = tid; w < d.words; w += kPolThreads) bits[w] = 0u;
  // extend the state to nb blocks (approx.py:152-156): new blocks start unseen and cold
  for (int blk = nb_prev + tid; blk < nb; blk += kPolThreads) {
    a.last_max[so + blk] = -INFINITY;
    a.ema[so + blk] = -INFINITY;
    a.vol[so + blk] = 0.f;
    a.age[so + blk] = 0;
    a.cold[so + blk] = 1;
  }
  __syncthreads();

  // the seed: the previous selection (own) or dense top-k (teacher), keys < length
  const int32_t* seed = (a.teacher ? a.baseline : a.topk) + static_cast<int64_t>(b) * k;
  float smin = INFINITY;
  for (int i = tid; i < k; i += kPolThreads) {
    const int32_t key = seed[i];
    if (key >= 0 && key < L) {
      atomicOr(&bits[key >> 5], 1u << (key & 31));
      smin = fminf(smin, s[key]);
    }
  }
  const float tau_seed = block_reduce_min(smin, reinterpret_cast<float*>(red));
  int cnt = 0;
  for (int w = tid; w < d.words; w += kPolThreads) cnt += __popc(bits[w]);
  const int seeded = block_reduce_sum<int>(cnt, reinterpret_cast<int*>(red));
  if (seeded != k) {  // approx.py:160-162: the seed must be k unique keys inside the row
    if (tid == 0) {
      st[TDSA_PST_ERROR] = 1.0;
      atomicOr(a.status, TDSA_STATUS_RANGE);
    }
    return;
  }

  // risk (approx.py:186-198) and forced reads (:241-248): one thread per block, the state
  // arrays read coalesced; whether the block holds a seed key comes from the bitmap
  for (int blk = tid; blk < nb; blk += kPolThreads) {
    const int16_t ag = a.age[so + blk];
    const double slope = a.age_slope * static_cast<double>(ag);
    double r;
    if (a.risk_ema) {
      const float spread = __fmul_rn(static_cast<float>(a.vol_lambda), a.vol[so + blk]);
      r = __dadd_rn(__dadd_rn(__dadd_rn(static_cast<double>(a.ema[so + blk]),
                                        static_cast<double>(spread)),
                              a.gamma),
                    slope);
    } else {
      r = __dadd_rn(__dadd_rn(static_cast<double>(a.last_max[so + blk]), a.gamma), slope);
    }
    risk[blk] = r;
    bool forced = a.full_refresh != 0;
    forced |= a.prev_length < L && blk >= a.prev_length / bs;
    forced |= a.recent_window > 0 && blk >= max(0, L - a.recent_window) / bs;
    forced |= a.age_cap >= 0 && ag >= a.age_cap;
    forced |= a.cold[so + blk] < a.cold_streak;
    bool has_seed = false;
    const int lo = blk * bs, hi = min(L, lo + bs);
    for (int w = lo >> 5; w <= (hi - 1) >> 5; ++w) {
      uint32_t word = bits[w];
      const int w0 = w * 32;
      if (lo > w0) word &= ~0u << (lo - w0);
      if (hi < w0 + 32) word &= (1u << (hi - w0)) - 1u;
      has_seed |= word != 0;
    }
    fl[blk] = (forced ? 1u : 0u) | (has_seed ? 8u : 0u);
  }
  // per-block maxima (numpy's NaN-propagating max): a warp takes four blocks at a time so
  // their loads are in flight together
  for (int blk0 = warp; blk0 < nb; blk0 += 4 * (kPolThreads / 32)) {
    float m[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int blk = blk0 + u * (kPolThreads / 32);
      m[u] = -INFINITY;
      if (blk < nb) {
        const int lo = blk * bs, n = min(bs, L - lo);
        for (int e = lane; e < n; e += 32) m[u] = nan_max(m[u], s[lo + e]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int blk = blk0 + u * (kPolThreads / 32);
      float mu = m[u];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mu = nan_max(mu, __shfl_xor_sync(0xffffffffu, mu, o));
      if (lane == 0 && blk < nb) {
        cmax[blk] = mu;
        a.cmax[so + blk] = mu;
      }
    }
  }
  __syncthreads();

  // the visiting order (approx.py:92-109, :200-204)
  if (a.order != TDSA_ORDER_ADDRESS && a.dynamic) {
    for (int i = tid; i < d.nbp; i += kPolThreads) {
      if (i < nb) {
        skey[i] = desc_key64(a.order == TDSA_ORDER_ORACLE_CURRENT ? static_cast<double>(cmax[i])
                                                                  : risk[i]);
        sidx[i] = static_cast<uint32_t>(i);
      } else {
        skey[i] = ~0ull;
        sidx[i] = 0xFFFFFFFFu;
      }
    }
    cta_sort_pairs(skey, sidx, d.nbp);
    if (a.order == TDSA_ORDER_BUCKET) {
      // rank r -> bucket min(B-1, r*B // nb); then by (bucket, address)
      for (int r = tid; r < d.nbp; r += kPolThreads) {
        if (r < nb) {
          const uint32_t blk = sidx[r];
          const int64_t bucket =
              min(static_cast<int64_t>(a.buckets) - 1,
                  static_cast<int64_t>(r) * a.buckets / max(1, nb));
          skey[r] = static_cast<uint64_t>(bucket);
          sidx[r] = blk;
        }
      }
      __syncthreads();
      cta_sort_pairs(skey, sidx, d.nbp);
    }
  } else {
    for (int i = tid; i < nb; i += kPolThreads) sidx[i] = static_cast<uint32_t>(i);
  }
  __syncthreads();

  // which blocks are read (approx.py:206-238)
  if (!a.dynamic) {
    for (int blk = tid; blk < nb; blk += kPolThreads)
      if ((fl[blk] & 1u) || !(risk[blk] < static_cast<double>(tau_seed))) fl[blk] |= 2u;
  } else {
    // the running top-k starts as the seed items, ascending
    for (int i = tid; i < d.kp; i += kPolThreads)
      A[i] = i < k ? item_of(s[seed[i]], seed[i]) : ~0ull;
    if (d.kp >= 64 && d.kp <= 2 * kPolThreads)
      cta_sort_keys_reg(A, d.kp);
    else
      cta_sort_keys(A, d.kp);
    auto mains = [&](int sel) { return sel ? A2 : A; };
    auto pends = [&](int sel) { return sel ? P2 : P; };
    if (tid == 0) {
      ctl->a_sel = ctl->p_sel = 0;
      ctl->ha = 0;
      ctl->na = k;
      ctl->hp = ctl->np = 0;
      ctl->T = A[0];
      ctl->ts = static_cast<double>(item_score(A[0]));
      ctl->pos = 0;
      ctl->w = 1;
    }
    __syncthreads();
    const unsigned below = (1u << lane) - 1u;
    while (ctl->pos < nb) {
      const int pos = ctl->pos, w = ctl->w;
      const double ts = ctl->ts;
      const uint64_t T = ctl->T;
      // (a) the window's candidates: blocks not already below the threshold (a block that
      // is not a candidate now is skipped for good: the threshold only rises)
      if (warp == 0) {
        int base = 0;
        for (int q = 0; q < w; q += 32) {
          const int p = pos + q + lane;
          int blk = 0;
          bool cand = false;
          if (q + lane < w && p < nb) {
            blk = static_cast<int>(sidx[p]);
            cand = (fl[blk] & 1u) || !(risk[blk] < ts);
          }
          const unsigned cm = __ballot_sync(0xffffffffu, cand);
          if (cand) ctl->cand[base + __popc(cm & below)] = blk;
          base += __popc(cm);
        }
        if (lane == 0) ctl->ncand = base;
      }
      __syncthreads();
      const int ncand = ctl->ncand;
      if (ncand == 0) {
        __syncthreads();
        if (tid == 0) {
          ctl->pos = pos + w;
          ctl->w = min(kMaxWindow, 2 * w);
        }
        __syncthreads();
        continue;
      }
      // (b) each warp loads its candidates' scores (up to kMaxWindow / 32 blocks, the loads
      // in flight together), keeps them in registers and counts the items above T
      constexpr int kPer = kMaxWindow / (kPolThreads / 32);  // candidates per warp (4)
      float sv[kPer][4];
      uint32_t take_mask[kPer];
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int c = warp + r * (kPolThreads / 32);
        const int blk = c < ncand ? ctl->cand[c] : 0;
        const int lo = blk * bs, n = c < ncand ? min(bs, L - lo) : 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int e = q * 32 + lane;
          sv[r][q] = e < n ? s[lo + e] : 0.f;
        }
      }
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int c = warp + r * (kPolThreads / 32);
        take_mask[r] = 0u;
        if (c < ncand) {  // warp-uniform
          const int lo = ctl->cand[c] * bs, n = min(bs, L - lo);
          int m = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int e = q * 32 + lane;
            bool take = false;
            if (e < n) {
              const int j = lo + e;
              take = !((bits[j >> 5] >> (j & 31)) & 1u) && item_of(sv[r][q], j) > T;
            }
            take_mask[r] |= take ? (1u << q) : 0u;
            m += __popc(__ballot_sync(0xffffffffu, take));
          }
          if (lane == 0) ctl->cnt[c] = m;
        }
      }
      __syncthreads();
      // (c) offsets of the candidates' items (warp 0, four candidates per lane)
      if (warp == 0) {
        int loc[kMaxWindow / 32], sum = 0;
#pragma unroll
        for (int r = 0; r < kMaxWindow / 32; ++r) {
          const int c = lane * (kMaxWindow / 32) + r;
          loc[r] = c < ncand ? ctl->cnt[c] : 0;
          sum += loc[r];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        int run = incl - sum;
#pragma unroll
        for (int r = 0; r < kMaxWindow / 32; ++r) {
          const int c = lane * (kMaxWindow / 32) + r;
          if (c < ncand) ctl->off[c] = run;
          run += loc[r];
        }
        if (lane == 31) ctl->tot = incl;
      }
      __syncthreads();
      const int tot = ctl->tot;
      if (tot == 0 || tot > kWindowCap) {
        // nothing enters: the threshold stays and every candidate is read; too many items
        // for one window (never with one block): a quarter of the window
        if (tot == 0)
          for (int c = tid; c < ncand; c += kPolThreads) fl[ctl->cand[c]] |= 2u;
        __syncthreads();
        if (tid == 0) {
          if (tot == 0) {
            ctl->pos = pos + w;
            ctl->w = min(kMaxWindow, 2 * w);
          } else {
            ctl->w = max(1, w / 4);
          }
        }
        __syncthreads();
        continue;
      }
      // (d) write the items at their offsets (each candidate's warp) and sort them
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int c = warp + r * (kPolThreads / 32);
        if (c < ncand) {  // warp-uniform
          const int lo = ctl->cand[c] * bs;
          int m = ctl->off[c];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const bool take = (take_mask[r] >> q) & 1u;
            const unsigned bal = __ballot_sync(0xffffffffu, take);
            if (take) C[m + __popc(bal & below)] = item_of(sv[r][q], lo + q * 32 + lane);
            m += __popc(bal);
          }
        }
      }
      const int mp = pow2_at_least(tot, 2);
      for (int i = tot + tid; i < mp; i += kPolThreads) C[i] = ~0ull;
      __syncthreads();
      if (mp <= 64) {
        if (warp == 0) {
          uint64_t x0 = 2 * lane < mp ? C[2 * lane] : ~0ull;
          uint64_t x1 = 2 * lane + 1 < mp ? C[2 * lane + 1] : ~0ull;
          warp_sort64(x0, x1, lane);
          if (2 * lane < mp) {
            C[2 * lane] = x0;
            C[2 * lane + 1] = x1;
          }
        }
        __syncthreads();
      } else if (mp <= 2 * kPolThreads) {
        cta_sort_keys_reg(C, mp);
      } else {
        cta_sort_keys(C, mp);
      }
      // (e) fold the pending list into the main list when it outgrows the insertions or
      // its capacity (same set, one sorted list); merge the items into the pending list
      {
        const int live = ctl->np - ctl->hp;
        if (live + tot > kPendCap || live > 4 * max(tot, 64)) {
          cta_merge(mains(ctl->a_sel) + ctl->ha, ctl->na - ctl->ha,
                    pends(ctl->p_sel) + ctl->hp, live, mains(ctl->a_sel ^ 1));
          if (tid == 0) {
            ctl->a_sel ^= 1;
            ctl->na = ctl->na - ctl->ha + live;
            ctl->ha = 0;
            ctl->hp = ctl->np = 0;
          }
          __syncthreads();
        }
      }
      const uint64_t* Am = mains(ctl->a_sel);
      uint64_t* Pn = pends(ctl->p_sel ^ 1);
      const int ha = ctl->ha, na = ctl->na;
      const int npn = ctl->np - ctl->hp + tot;
      cta_merge(pends(ctl->p_sel) + ctl->hp, ctl->np - ctl->hp, C, tot, Pn);
      // (f) drop the tot smallest of main + merged pending; the speculation holds if every
      // candidate still passes against the resulting threshold (each saw one no higher)
      if (warp == 0) {
        const int take = warp_split(Am + ha, na - ha, Pn, npn, tot, lane);
        uint64_t te = ha + take < na ? Am[ha + take] : ~0ull;
        if (tot - take < npn && Pn[tot - take] < te) te = Pn[tot - take];
        const double tes = static_cast<double>(item_score(te));
        bool ok = true;
        for (int c = lane; c < ncand; c += 32) {
          const int blk = ctl->cand[c];
          ok &= (fl[blk] & 1u) || !(risk[blk] < tes);
        }
        const bool commit = w == 1 || __all_sync(0xffffffffu, ok);
        if (commit) {
          for (int c = lane; c < ncand; c += 32) fl[ctl->cand[c]] |= 2u;
          if (lane == 0) {
            ctl->p_sel ^= 1;
            ctl->np = npn;
            ctl->hp = tot - take;
            ctl->ha = ha + take;
            ctl->T = te;
            ctl->ts = tes;
            ctl->pos = pos + w;
            ctl->w = min(kMaxWindow, 2 * w);
          }
        } else if (lane == 0) {
          ctl->w = max(1, w / 4);  // retry from the same position with a smaller window
        }
      }
      __syncthreads();
    }
  }

  // the verifier's rescue (verifier.py:186-233): the cold keys' verifier maxima per block,
  // cold blocks ranked by (maximum desc, address asc), a budget or a threshold
  if (a.rescue) {
    const float* v = a.vscores + b * a.v_stride;
    for (int blk = warp; blk < nb; blk += kPolThreads / 32) {
      const int lo = blk * bs, n = (fl[blk] & 2u) ? 0 : min(bs, L - lo);
      float m = -INFINITY;
      bool any = false;
      for (int e = lane; e < n; e += 32) {
        const int j = lo + e;
        if (!((bits[j >> 5] >> (j & 31)) & 1u)) {
          m = any ? nan_max(m, v[j]) : v[j];
          any = true;
        }
      }
      const unsigned has = __ballot_sync(0xffffffffu, any);
      // max over the lanes that saw a cold key
      float mm = any ? m : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, mm, o);
        mm = nan_max(mm, other);
      }
      if (lane == 0) {
        skey[blk] = has ? desc_key64(static_cast<double>(mm)) : ~0ull;
        cmax[blk] = mm;  // reused: the cold maximum (cmax already saved to global)
        if (has) fl[blk] |= 16u;
      }
    }
    for (int i = nb + tid; i < d.nbp; i += kPolThreads) skey[i] = ~0ull;
    for (int i = tid; i < d.nbp; i += kPolThreads) sidx[i] = i < nb ? i : 0xFFFFFFFFu;
    cta_sort_pairs(skey, sidx, d.nbp);
    int c = 0;
    for (int blk = tid; blk < nb; blk += kPolThreads) c += (fl[blk] >> 4) & 1u;
    const int ncold = block_reduce_sum<int>(c, reinterpret_cast<int*>(red));
    int budget = ncold;
    if (!a.use_threshold)
      budget = min(ncold, static_cast<int>(ceil(a.rescue_fraction * static_cast<double>(ncold))));
    for (int r = tid; r < ncold; r += kPolThreads) {
      const int blk = static_cast<int>(sidx[r]);
      const bool take = a.use_threshold
                            ? static_cast<double>(cmax[blk]) >= a.promotion_threshold
                            : r < budget;
      if (take) fl[blk] |= 4u;
      if (a.ranking) a.ranking[so + r] = blk;
    }
    if (tid == 0) st[TDSA_PST_COLD_BLOCKS] = ncold;
    __syncthreads();
  }

  // outputs: masked row, keys-read bitmap, flags; counts
  float* mrow = a.masked + static_cast<int64_t>(b) * L;
  for (int j = tid; j < L; j += kPolThreads) {
    const bool ev = ((bits[j >> 5] >> (j & 31)) & 1u) || (fl[j >> lbs] & 6u);
    mrow[j] = ev ? s[j] : -INFINITY;
  }
  // keys-read bitmap (seed bits, then whole refreshed / rescued blocks) and the counts
  int tally[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};  // temporal, union, 4 x physical, 3 x flags
  uint32_t* eb = a.ebits + b * a.e_stride;
  auto block_mask = [&](int w, uint8_t bit) -> uint32_t {
    uint32_t m = 0u;
    const int w0 = w * 32;
    for (int blk = w0 >> lbs; blk <= min(nb - 1, (w0 + 31) >> lbs); ++blk) {
      if (!(fl[blk] & bit)) continue;
      const int lo = max(w0, blk * bs), hi = min(min(L, w0 + 32), (blk + 1) * bs);
      if (hi > lo) m |= ((hi - lo == 32) ? ~0u : ((1u << (hi - lo)) - 1u)) << (lo - w0);
    }
    return m;
  };
  for (int w = tid; w < d.words; w += kPolThreads) {
    const uint32_t word = bits[w] | block_mask(w, 2u);
    const uint32_t word_u = word | block_mask(w, 4u);
    eb[w] = word_u;
    tally[0] += __popc(word);
    tally[1] += __popc(word_u);
    tally[2] += ((word_u & 0xFFFFu) != 0) + ((word_u >> 16) != 0);
    tally[3] += word_u != 0;
  }
  __syncthreads();
  // 64- and 128-key physical blocks: words 2p, 2p+1 (and 4p..4p+3)
  for (int p = tid; p < (d.words + 1) / 2; p += kPolThreads) {
    const uint32_t w0 = eb[2 * p], w1 = 2 * p + 1 < d.words ? eb[2 * p + 1] : 0u;
    tally[4] += (w0 | w1) != 0;
  }
  for (int p = tid; p < (d.words + 3) / 4; p += kPolThreads) {
    uint32_t w = 0;
    for (int q = 0; q < 4; ++q)
      if (4 * p + q < d.words) w |= eb[4 * p + q];
    tally[5] += w != 0;
  }
  for (int blk = tid; blk < nb; blk += kPolThreads) {
    tally[6] += (fl[blk] >> 1) & 1u;
    tally[7] += (fl[blk] >> 2) & 1u;
    tally[8] += (fl[blk] >> 3) & 1u;
    a.flags[so + blk] = fl[blk];
  }
  block_reduce_sum_n<10>(tally, ired);
  const int ev_total = tally[0], union_total = tally[1], ref_total = tally[6], res_total = tally[7],
            sb_total = tally[8];
  const int phys_total[4] = {tally[2], tally[3], tally[4], tally[5]};
  if (tid == 0) {
    st[TDSA_PST_ERROR] = 0.0;
    if (!a.rescue) st[TDSA_PST_COLD_BLOCKS] = 0.0;
    st[TDSA_PST_TAU_SEED] = tau_seed;
    st[TDSA_PST_SCORED] = ev_total;
    st[TDSA_PST_UNION] = union_total;
    st[TDSA_PST_REFRESHED] = ref_total;
    st[TDSA_PST_SKIPPED] = nb - ref_total;
    st[TDSA_PST_RESCUED] = res_total;
    st[TDSA_PST_SEED_BLOCKS] = sb_total;
    for (int q = 0; q < 4; ++q) st[TDSA_PST_PHYS16 + q] = phys_total[q];
    st[TDSA_PST_BLOCKS] = nb;
  }
}

// ---------------------------------------------------------------------------- finalize
__global__ void __launch_bounds__(kPolThreads) policy_finalize_kernel(const PolicyArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int words = (a.length + 31) / 32;
  uint32_t* in_approx = reinterpret_cast<uint32_t*>(sm);
  uint32_t* in_old = in_approx + words;
  uint8_t* hot = reinterpret_cast<uint8_t*>(in_old + words);
  double* red = reinterpret_cast<double*>(sm + align_up(2 * words * 4 + a.nbc, 16));

  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x, tid = threadIdx.x;
  const int L = a.length, bs = a.bs, k = a.k;
  const int nb = (L + bs - 1) / bs;
  const int64_t so = static_cast<int64_t>(b) * a.nbc, ko = static_cast<int64_t>(b) * k;
  double* st = a.stats + static_cast<int64_t>(b) * TDSA_POLICY_NSTATS;
  if (st[TDSA_PST_ERROR] != 0.0) return;  // the decide step rejected the seed
  const float* s = a.scores + b * a.s_stride;
  const int32_t* ap = a.approx + ko;
  const int32_t* bn = a.base_new + ko;
  const int32_t* bo = a.baseline + ko;

  for (int w = tid; w < 2 * words; w += kPolThreads) in_approx[w] = 0u;
  for (int blk = tid; blk < nb; blk += kPolThreads) hot[blk] = 0;
  __syncthreads();
  float fmin = INFINITY;
  for (int i = tid; i < k; i += kPolThreads) {
    const int32_t x = ap[i], y = bo[i];
    atomicOr(&in_approx[x >> 5], 1u << (x & 31));
    fmin = fminf(fmin, s[x]);
    if (y >= 0 && y < L) atomicOr(&in_old[y >> 5], 1u << (y & 31));
    hot[(a.teacher ? bn[i] : x) / bs] = 1;
  }
  const float tau_final = block_reduce_min(fmin, reinterpret_cast<float*>(red));

  // metadata of the blocks observed this step (approx.py:274-293, verifier.py:147-159)
  const double al = a.ema_alpha;
  const float one_minus = static_cast<float>(__dsub_rn(1.0, al));
  for (int blk = tid; blk < nb; blk += kPolThreads) {
    const float obs = a.cmax[so + blk];
    const uint8_t f = a.flags[so + blk];
    int16_t ag = a.age[so + blk];
    if (a.teacher) {
      a.last_max[so + blk] = obs;
      a.ema[so + blk] = obs;
      a.vol[so + blk] = 0.f;
      ag = 0;
    } else if (f & 6u) {
      const double o = static_cast<double>(obs);
      const float e = a.ema[so + blk];
      const double mean = isfinite(e) ? static_cast<double>(e) : o;
      a.last_max[so + blk] = obs;
      a.ema[so + blk] =
          __double2float_rn(__dadd_rn(__dmul_rn(al, o), __dmul_rn(__dsub_rn(1.0, al), mean)));
      // float32(a * |obs - mean|) + float32(1 - a) * vol, float32 operations
      const float first = __double2float_rn(__dmul_rn(al, fabs(__dsub_rn(o, mean))));
      a.vol[so + blk] = __fadd_rn(first, __fmul_rn(one_minus, a.vol[so + blk]));
      ag = 0;
    } else {
      ag = static_cast<int16_t>(min(static_cast<int>(ag) + 1, 32767));
    }
    a.age[so + blk] = ag;
    const int c = a.cold[so + blk];
    a.cold[so + blk] = hot[blk] ? 0 : static_cast<int16_t>(min(c + 1, 32767));
  }

  // recall, misses, newly hot keys and the index mass (approx.py:296-330)
  int hits[5] = {0, 0, 0, 0, 0};
  int missed = 0, worst = 0x7FFFFFFF, newly = 0, newly_missed = 0;
  double num = 0.0, den = 0.0;
  float shift = -INFINITY;
  for (int i = tid; i < k; i += kPolThreads) shift = fmaxf(shift, s[bn[i]]);
  shift = -block_reduce_min(-shift, reinterpret_cast<float*>(red));
  for (int i = tid; i < k; i += kPolThreads) {
    const int32_t x = bn[i];
    const bool hit = (in_approx[x >> 5] >> (x & 31)) & 1u;
    const bool was = (in_old[x >> 5] >> (x & 31)) & 1u;
    if (hit) {
      hits[0] += i < 128;
      hits[1] += i < 256;
      hits[2] += i < 512;
      hits[3] += i < 1024;
      hits[4] += i < 2048;
    } else {
      ++missed;
      worst = min(worst, i + 1);
    }
    if (!was) {
      ++newly;
      newly_missed += !hit;
    }
    den += exp(static_cast<double>(s[x]) - static_cast<double>(shift));
    num += exp(static_cast<double>(s[ap[i]]) - static_cast<double>(shift));
  }
  int tot[5];
  for (int q = 0; q < 5; ++q) tot[q] = block_reduce_sum<int>(hits[q], reinterpret_cast<int*>(red));
  const int missed_t = block_reduce_sum<int>(missed, reinterpret_cast<int*>(red));
  const int newly_t = block_reduce_sum<int>(newly, reinterpret_cast<int*>(red));
  const int newly_missed_t = block_reduce_sum<int>(newly_missed, reinterpret_cast<int*>(red));
  const int worst_t = block_reduce_min_int(worst, reinterpret_cast<int*>(red));
  const double num_t = block_reduce_sum<double>(num, red);
  const double den_t = block_reduce_sum<double>(den, red);

  // the next state's lists (after every read of the old baseline above)
  for (int i = tid; i < k; i += kPolThreads) {
    a.topk[ko + i] = ap[i];
    a.baseline[ko + i] = bn[i];
  }
  if (tid == 0) {
    a.nblocks[b] = nb;
    st[TDSA_PST_TAU_FINAL] = tau_final;
    for (int q = 0; q < 5; ++q) st[TDSA_PST_TOP128 + q] = tot[q];
    st[TDSA_PST_MISSED] = missed_t;
    st[TDSA_PST_WORST_MISSED] = missed_t ? worst_t : 0;
    st[TDSA_PST_NEWLY_HOT] = newly_t;
    st[TDSA_PST_NEWLY_HOT_MISSED] = newly_missed_t;
    st[TDSA_PST_MASS_NUM] = num_t;
    st[TDSA_PST_MASS_DEN] = den_t;
  }
}

}  // namespace

size_t policy_state_bytes(int batch, int k, int nbc, int64_t* offsets) {
  const size_t B = static_cast<size_t>(batch);
  size_t o = 0;
  int64_t off[8];
  off[0] = o; o = align_up(o + B * k * 4, 256);      // topk
  off[1] = o; o = align_up(o + B * k * 4, 256);      // baseline_topk
  off[2] = o; o = align_up(o + B * nbc * 4, 256);    // last_max
  off[3] = o; o = align_up(o + B * nbc * 4, 256);    // ema
  off[4] = o; o = align_up(o + B * nbc * 4, 256);    // volatility
  off[5] = o; o = align_up(o + B * nbc * 2, 256);    // age
  off[6] = o; o = align_up(o + B * nbc * 2, 256);    // cold_streak
  off[7] = o; o = align_up(o + B * 4, 256);          // block count held
  if (offsets)
    for (int i = 0; i < 8; ++i) offsets[i] = off[i];
  return o;
}

size_t policy_decide_smem_bytes(int length, int bs, int k) {
  return decide_smem(length, bs, k).total;
}

int launch_policy(int init, uint8_t* state, int batch, int k, int nbc, const float* scores,
                  int64_t s_stride, const float* vscores, int64_t v_stride, int length,
                  int prev_length, int bs, const tdsa_policy* pol, int teacher,
                  int full_refresh, const tdsa_rescue* rescue, float* masked, float* cmax,
                  uint8_t* flags, int32_t* ranking, uint32_t* ebits, int64_t e_stride,
                  int32_t* base_new, int32_t* approx, void* topk_ws, size_t topk_ws_bytes,
                  double* stats, int* status, cudaStream_t stream) {
  int64_t off[8];
  policy_state_bytes(batch, k, nbc, off);
  PolicyArgs a = {};
  a.topk = reinterpret_cast<int32_t*>(state + off[0]);
  a.baseline = reinterpret_cast<int32_t*>(state + off[1]);
  a.last_max = reinterpret_cast<float*>(state + off[2]);
  a.ema = reinterpret_cast<float*>(state + off[3]);
  a.vol = reinterpret_cast<float*>(state + off[4]);
  a.age = reinterpret_cast<int16_t*>(state + off[5]);
  a.cold = reinterpret_cast<int16_t*>(state + off[6]);
  a.nblocks = reinterpret_cast<int32_t*>(state + off[7]);
  a.k = k;
  a.nbc = nbc;
  a.scores = scores;
  a.s_stride = s_stride;
  a.vscores = vscores;
  a.v_stride = v_stride;
  a.length = length;
  a.prev_length = prev_length;
  a.bs = bs;
  a.masked = masked;
  a.cmax = cmax;
  a.flags = flags;
  a.ranking = ranking;
  a.ebits = ebits;
  a.e_stride = e_stride;
  a.approx = approx;
  a.base_new = base_new;
  a.stats = stats;
  a.status = status;
  // the dense top-k of the current scores (sorted: the reference's stable_topk order)
  int rc = launch_topk(scores, s_stride, nullptr, 0, batch, length, k, 1, base_new, 4, k,
                       nullptr, 0, topk_ws, topk_ws_bytes, stream);
  if (rc) return rc;
  if (init) {
    TDSA_CUDA_CHECK(launch_pdl(policy_init_kernel, dim3(batch), dim3(kPolThreads), 0, stream,
                               a, static_cast<const int32_t*>(base_new)));
    return TDSA_OK;
  }
  a.gamma = pol->gamma;
  a.ema_alpha = pol->ema_alpha;
  a.vol_lambda = pol->volatility_lambda;
  a.age_slope = pol->age_slope;
  a.cold_streak = pol->cold_streak;
  a.dynamic = pol->dynamic_threshold;
  a.order = pol->order;
  a.buckets = pol->buckets;
  a.age_cap = pol->age_cap;
  a.recent_window = pol->recent_window;
  a.risk_ema = pol->risk_model == TDSA_RISK_EMA;
  a.teacher = teacher;
  a.full_refresh = full_refresh;
  if (rescue) {
    a.rescue = 1;
    a.use_threshold = rescue->use_threshold;
    a.rescue_fraction = rescue->rescue_fraction;
    a.promotion_threshold = rescue->promotion_threshold;
  }
  const size_t smem = decide_smem(length, bs, k).total;
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(policy_decide_kernel),
                                      static_cast<int>(smem)));
  TDSA_CUDA_CHECK(launch_pdl(policy_decide_kernel, dim3(batch), dim3(kPolThreads), smem, stream,
                             a));
  // the selection: stable top-k of the keys read
  rc = launch_topk(masked, length, nullptr, 0, batch, length, k, 1, approx, 4, k, nullptr, 0,
                   topk_ws, topk_ws_bytes, stream);
  if (rc) return rc;
  const size_t fsmem = align_up(2 * static_cast<size_t>((length + 31) / 32) * 4 + nbc, 16) +
                       64 * sizeof(double);
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(policy_finalize_kernel),
                                      static_cast<int>(fsmem)));
  TDSA_CUDA_CHECK(launch_pdl(policy_finalize_kernel, dim3(batch), dim3(kPolThreads), fsmem,
                             stream, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
