// Exact row-wise top-k by radix select over a shared-memory copy of the row (no global
// sort).
//
// One 1024-thread CTA owns one segment of a row (<= 32768 elements), copied into shared
// memory by bulk copies (TMA engine, 32 KB per mbarrier).  Thread t owns the P consecutive
// elements [P*t, P*t + P) (P = segment / 1024 rounded up to 4, 8, 16 or 32), so thread
// order is index order; a thread visits its elements rotated by its lane group, which
// keeps a warp's shared-memory reads on 32 distinct banks.
//   1. Live range [clo, chi] holding the k-th key: from the score kernel's 12-bit key
//      histogram when one is given (read while the copy is in flight), else the segment's
//      min/max (that pass also converts the floats to order-preserving keys in place).
//   2. Range-narrowing radix passes (256 bins, eight private histograms) only until the
//      keys >= clo fit the candidate list (8192 entries), or the range is one value.
//   3. One ordered compaction: each thread builds a bit mask of its elements to keep
//      (every key >= clo when they fit; otherwise keys > chi and the lowest-index keys of
//      the one-value range that complete k), one CTA-wide scan of the mask popcounts gives
//      list positions, and only the kept elements are written.
//   4. The list is narrowed to the exact k-th key T; keys > T and the lowest-index keys
//      == T are taken -- the tie rule of the reference's stable_topk (metrics.py:9-22).
//      Unsorted output is in ascending index order; sorted output is a bitonic sort of the
//      k taken (key, index) pairs in shared memory.
// Unsorted rows whose histogram gave the k-th key's bin take a shorter road (take_from_bin):
// one compare per key against the bin's lower edge fills the list, two histogram levels
// over the bin's list entries (11 + 9 key bits) give T, and one ordered pass takes.
//
// Rows longer than one segment run in levels: every segment emits its local top-k in index
// order, and the candidates (the global top-k is a subset of their union) are selected
// again with explicit indices until one segment remains.  The same explicit-index pass
// merges per-GPU candidates of an L-sharded cache.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "timeline.cuh"

namespace tdsa {

// (outside the unnamed namespace: the timeline readers keep external C linkage)
// timeline builds, per row of a one-segment launch (thread 0): 0 entry, 1 past the
// dependency wait, 2 row copy landed and the histogram's bin read, 3 candidate list written,
// 4 the k-th key found, 5 output written, 6 this thread's classification pass done (the
// histogram-started unsorted path)
TDSA_TL_DECL(topk, 64, 7)

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 256;
constexpr int kCap = 8192;  // candidate-list entries (keys >= the live range's low end)

struct TopkArgs {
  const float* vals;      // [rows][row_stride]
  int64_t vals_stride;
  const int32_t* idx;     // explicit indices (same layout as vals) or nullptr
  int64_t idx_stride;
  int row_len;            // elements per row
  int chunk;              // segment length (gridDim.x segments per row)
  int k;
  int sorted;
  void* out_idx;          // [rows * gridDim.x][out_idx_stride] (null: k-th value only)
  int idx_bytes;
  int64_t out_idx_stride;
  float* out_val;         // may be null
  int64_t out_val_stride;
  float* kth_out;         // per output row: the k-th largest value (may be null)
  uint32_t* hist;         // per (row, segment) [4096] key histogram of this level's input
                          // (from the score kernel, or from the previous level); consumed
                          // and re-zeroed, or null
  uint32_t* next_hist;    // per row [4096]: this level adds the key bins of the entries it
                          // outputs, for a one-segment next level (or null)
  int pad_to_k;           // a level feeding another: a segment shorter than k fills its
                          // remaining output slots with (-inf, index 0x7FFFFFFF)
  int row_words;          // shared-memory words of the segment copy (reused for sort pairs)
  int cap;                // candidate-list entries
  int* status;            // device status word (bounded-wait timeouts)
  int gather;             // merge of an exchange: gather the rows from peer memory first
  PeerGather pg;
  int hist_segs;          // cluster top-k: the row's 32768-key histogram segments (summed)
  int32_t* mirror;        // the last level also writes its indices here, int32
                          // ([rows][mirror_stride]; null: not)
  int64_t mirror_stride;
};

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ int bit_length(uint32_t x) { return x ? 32 - __clz(x) : 0; }

// Exclusive prefix over the 32 warps of per-warp values (run by warp 0), into out[32].
__device__ __forceinline__ void warp_totals_scan(const uint32_t* in, uint32_t* out) {
  const int lane = threadIdx.x & 31;
  const uint32_t v = in[lane];
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  out[lane] = x - v;
}

// Pick the bin of the k_rem-th key from the top out of the eight private histograms and
// narrow [clo, chi] to it (bin width 2^sh).  Returns with all threads agreeing.
__device__ __forceinline__ void narrow_to_bin(const uint32_t* hists, uint32_t* hist,
                                              uint32_t* res, int sh, uint32_t& clo,
                                              uint32_t& chi, uint32_t& k_rem,
                                              uint32_t& in_range) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < kBins) {
    uint32_t s = 0;
#pragma unroll
    for (int h = 0; h < 8; ++h) s += hists[h * kBins + tid];
    hist[tid] = s;
  }
  __syncthreads();
  if (warp == 0) {
    // bins from the top: lane l owns bins 255-8l .. 248-8l; suffix sums via a lane scan
    uint32_t c[8], tot = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      c[i] = hist[kBins - 1 - (lane * 8 + i)];
      tot += c[i];
    }
    uint32_t x = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    uint32_t above = x - tot;
    if (above < k_rem && k_rem <= x) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (above < k_rem && k_rem <= above + c[i]) {
          res[0] = kBins - 1 - (lane * 8 + i);
          res[1] = k_rem - above;
          res[2] = c[i];
        }
        above += c[i];
      }
    }
  }
  __syncthreads();
  const uint32_t d = res[0];
  k_rem = res[1];
  in_range = res[2];
  const uint64_t lo64 = static_cast<uint64_t>(clo) + (static_cast<uint64_t>(d) << sh);
  const uint64_t top = lo64 + (1ull << sh) - 1;
  const uint64_t hi64 = top < chi ? top : static_cast<uint64_t>(chi);
  clo = static_cast<uint32_t>(lo64);
  chi = static_cast<uint32_t>(hi64);
}

// Exclusive prefix of v over the CTA (thread order); *total gets the sum.  Two barriers.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* wa, uint32_t* wb,
                                                    uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wa[warp] = x;
  __syncthreads();
  if (warp == 0) {
    warp_totals_scan(wa, wb);
    if (lane == 31) *total = wb[31] + wa[31];
  }
  __syncthreads();
  return wb[warp] + x - v;
}

// The bin of the k_rem-th key counted from the top, thread t holding the counts c[0..3] of
// bins nbins-1-4t .. nbins-4-4t (zeros past nbins): res = {bin, k_rem within the bin, the
// bin's count, 1}, or res[3] = 0 when the counts total less than k_rem.  Three CTA
// barriers; all threads return with res readable.
__device__ __forceinline__ void pick_bin(const uint32_t (&c)[4], int nbins, uint32_t k_rem,
                                         uint32_t* wa, uint32_t* wb, uint32_t* res) {
  const int tid = threadIdx.x;
  const uint32_t tot = c[0] + c[1] + c[2] + c[3];
  if (tid == 0) res[3] = 0u;
  uint32_t dummy;
  uint32_t above = block_excl_scan(tot, wa, wb, &dummy);
  if (above < k_rem && k_rem <= above + tot) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (above < k_rem && k_rem <= above + c[i]) {
        res[0] = static_cast<uint32_t>(nbins - 1 - (4 * tid + i));
        res[1] = k_rem - above;
        res[2] = c[i];
        res[3] = 1u;
      }
      above += c[i];
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void bins_from_top(const uint32_t* h, int nbins, uint32_t (&c)[4]) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = 4 * tid + i < nbins ? h[nbins - 1 - (4 * tid + i)] : 0u;
}

// Unsorted selection once the score kernel's histogram has given the 12-bit key bin
// [clo, chi] of the k-th key (k_rem of its in_range keys are taken, and k - k_rem keys lie
// above it): every key >= clo goes to the list in index order -- straight to the output
// when the whole bin is taken -- the list is narrowed to the exact k-th key by two
// histogram levels over the bin's keys (key bits 19..9 in 2048 bins, then 8..0 in 512),
// and one ordered pass takes the keys above the final range and the lowest-index keys
// inside it that complete k (the tie rule of stable_topk, metrics.py:9-22).  Output in
// ascending index order, as the general path; a level feeding a merge level pads a segment
// shorter than k and adds its output's key bins to the next level's histogram, as the
// general path does.  `hists` (2048 words) is zero on entry; the
// list holds k - k_rem + in_range <= a.cap entries.  A row copy of kPer keys per thread sits
// in `rowf`.  `tl_launch`: the launch number of a timeline build (unused otherwise).
template <int kPer, bool kTail>
__device__ __forceinline__ void take_from_bin(const TopkArgs& a, int row, int seg, int start,
                                              int n, int k, const float* rowf,
                                              const int32_t* irow, uint32_t* list_key,
                                              uint32_t* list_idx, uint32_t* hists,
                                              uint32_t* wa, uint32_t* wb, uint32_t* res,
                                              uint32_t* s_total, uint32_t clo, uint32_t chi,
                                              uint32_t k_rem, uint32_t in_range,
                                              unsigned int tl_launch) {
  const int tid = threadIdx.x, lane = tid & 31;
  constexpr int kLog = kPer == 32 ? 5 : kPer == 16 ? 4 : kPer == 8 ? 3 : 2;
  const int rot = lane >> (5 - kLog);
  const int tbase = tid * kPer;
  const uint32_t uk = static_cast<uint32_t>(k);
  const bool whole = in_range == k_rem;  // every key >= clo is taken
  const int64_t out_row = static_cast<int64_t>(row) * gridDim.x + seg;
  int32_t* oi32 = a.idx_bytes == 4 ? static_cast<int32_t*>(a.out_idx) + out_row * a.out_idx_stride
                                   : nullptr;
  int64_t* oi64 = a.idx_bytes == 8 ? static_cast<int64_t*>(a.out_idx) + out_row * a.out_idx_stride
                                   : nullptr;
  float* ov = a.out_val ? a.out_val + out_row * a.out_val_stride : nullptr;
  int32_t* om = a.mirror ? a.mirror + out_row * a.mirror_stride : nullptr;
  // a level feeding a one-segment next level adds the bins of what it passes on
  uint32_t* nh = a.next_hist ? a.next_hist + static_cast<int64_t>(row) * kKeyHistBins : nullptr;
  // one output entry; `count` adds its key bin to the next level's histogram alone (the
  // ordered take below adds them per warp instead)
  auto put = [&](uint32_t p, uint32_t gi, uint32_t u, bool count) {
    if (p < uk) {
      if (oi32) oi32[p] = static_cast<int32_t>(gi);
      if (oi64) oi64[p] = static_cast<int64_t>(gi);
      if (om) om[p] = static_cast<int32_t>(gi);
      if (ov) ov[p] = key_to_float(u);
      if (nh && count) atomicAdd(&nh[u >> 20], 1u);
    }
  };
  if (a.pad_to_k && n < a.k) {
    // pads rank below every real candidate of the next level (-inf, then the largest index)
    for (int j = n + tid; j < a.k; j += kThreads) {
      if (oi32) oi32[j] = 0x7FFFFFFF;
      if (ov) ov[j] = -INFINITY;
    }
    if (tid == 0 && nh) atomicAdd(&nh[float_to_key(-INFINITY) >> 20], static_cast<uint32_t>(a.k - n));
  }
  auto gidx = [&](int e) -> uint32_t {
    return irow ? static_cast<uint32_t>(irow[e]) : static_cast<uint32_t>(start + e);
  };

  // ---- the thread's keys >= clo, bit j = element tbase + j
  uint32_t take = 0u;
  if (clo >= 0x00800000u && clo <= 0xFF800000u) {
    // key(x) >= clo  <=>  !(x < float(clo)) for a bin edge of finite floats or +inf, exact
    // for +-0 (one key) and NaN (above every key): one compare per key
    const float f_lo = key_to_float(clo);
    if (kPer == 32 && tbase + 32 <= n) {
      // eight conflict-free 16-byte reads per thread, rotated by lane
      const float4* r4 = reinterpret_cast<const float4*>(rowf) + tid * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int qq = (j + lane) & 7;
        const float4 v = r4[qq];
        const uint32_t nib = (!(v.x < f_lo) ? 1u : 0u) | (!(v.y < f_lo) ? 2u : 0u) |
                             (!(v.z < f_lo) ? 4u : 0u) | (!(v.w < f_lo) ? 8u : 0u);
        take |= nib << (4 * qq);
      }
    } else {
#pragma unroll 8
      for (int j = 0; j < kPer; ++j) {
        const int jj = (j + rot) & (kPer - 1);
        const int e = tbase + jj;
        if (e < n && !(rowf[e] < f_lo)) take |= 1u << jj;
      }
    }
  } else {
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int jj = (j + rot) & (kPer - 1);
      const int e = tbase + jj;
      if (e < n && float_to_key(rowf[e]) >= clo) take |= 1u << jj;
    }
  }
  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 6);
  // kTail: a wide row's tail keys [kPer * 1024 + 4 tid, + 4) (rows past one segment,
  // kPer = 32), listed after all the main keys
  const int tail0 = kPer * kThreads + 4 * tid;
  uint32_t take_tail = 0u;
  if constexpr (kTail) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (tail0 + c < n && float_to_key(rowf[tail0 + c]) >= clo) take_tail |= 1u << c;
  }
  // list (or output) positions in index order: the main keys, then the tail keys (a segment
  // holds < 65536 keys, so the packed halves do not carry)
  const uint32_t before = block_excl_scan(static_cast<uint32_t>(__popc(take)) |
                                              (static_cast<uint32_t>(__popc(take_tail)) << 16),
                                          wa, wb, s_total);
  const uint32_t main_total = kTail ? (*s_total & 0xFFFFu) : *s_total;
  const uint32_t m_all = kTail ? main_total + (*s_total >> 16) : main_total;
  // a listed key inside the bin is also counted at once by key bits 19..9 (the first
  // narrowing level below), so the level needs no pass of its own over the list
  auto place = [&](uint32_t pos, int e) {
    const uint32_t u = float_to_key(rowf[e]);
    if (whole) {
      put(pos, gidx(e), u, true);
    } else if (pos < static_cast<uint32_t>(a.cap)) {
      list_key[pos] = u;
      list_idx[pos] = gidx(e);
      if (u <= chi) atomicAdd(&hists[(u >> 9) & 0x7FFu], 1u);  // the bin's keys (>= clo)
    }
  };
  uint32_t pos = kTail ? (before & 0xFFFFu) : before;
  for (uint32_t t = take; t; t &= t - 1u) place(pos++, tbase + __ffs(t) - 1);
  if constexpr (kTail) {
    pos = main_total + (before >> 16);
    for (uint32_t t = take_tail; t; t &= t - 1u) place(pos++, tail0 + __ffs(t) - 1);
  }
  if (whole) return;
  __syncthreads();  // the list, in index order, and its first-level counts
  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 3);
  const uint32_t m = min(m_all, static_cast<uint32_t>(a.cap));

  // ---- the exact k-th key inside the bin: bits 19..9 (counted while listing), then 8..0
  uint32_t c4[4];
  bins_from_top(hists, 2048, c4);
  pick_bin(c4, 2048, k_rem, wa, wb, res);
  uint32_t flo = clo, fhi = chi, fk = k_rem;  // final range, and how many of it are taken
  if (res[3]) {
    flo = clo | (res[0] << 9);
    fhi = flo | 0x1FFu;
    fk = res[1];
    if (res[2] != fk) {
      if (tid < 512) hists[tid] = 0u;  // every thread holds its level-2 counts already
      __syncthreads();
      for (uint32_t i = tid; i < m; i += kThreads) {
        const uint32_t u = list_key[i];
        if (u >= flo && u <= fhi) atomicAdd(&hists[u & 0x1FFu], 1u);
      }
      __syncthreads();
      bins_from_top(hists, 512, c4);
      pick_bin(c4, 512, fk, wa, wb, res);
      if (res[3]) {
        flo |= res[0];
        fhi = flo;
        fk = res[1];
      }
    }
  }

  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 4);
  // ---- the taken keys: above the final range, and the first fk inside it; thread t takes
  // list entries [t * per, t * per + per)
  const int per = (static_cast<int>(m) + kThreads - 1) / kThreads;
  const int i0 = min(static_cast<int>(m), tid * per), i1 = min(static_cast<int>(m), i0 + per);
  uint32_t gc = 0u, ec = 0u;
  for (int i = i0; i < i1; ++i) {
    const uint32_t u = list_key[i];
    gc += u > fhi ? 1u : 0u;
    ec += (u >= flo && u <= fhi) ? 1u : 0u;
  }
  // a list holds <= 8192 entries, so the packed halves do not carry
  const uint32_t b2 = block_excl_scan(gc | (ec << 16), wa, wb, s_total);
  uint32_t g = b2 & 0xFFFFu, eb = b2 >> 16;
  for (int j = 0; j < per; ++j) {  // uniform trip count: the bins are added per warp
    const int i = i0 + j;
    const uint32_t u = i < i1 ? list_key[i] : 0u;
    uint32_t p = 0xFFFFFFFFu;
    if (i < i1 && u > fhi) {
      p = g + min(eb, fk);
      ++g;
    } else if (i < i1 && u >= flo) {
      if (eb < fk) p = g + eb;
      ++eb;
    }
    if (p != 0xFFFFFFFFu) put(p, list_idx[i], u, false);
    if (nh) add_to_bin(nh, p < uk, u >> 20);
  }
  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 5);
}

// key(x) >= c for an order-preserving key threshold c, as float compares where that is exact:
// c in [key(-FLT_MAX's bin edge), key(+inf)] compares against float(c) (+-0 one key, NaN
// above all keys), c at or below the key of -inf holds for every x, c above +inf's key only
// for NaN.
struct KeyGE {
  float f;
  int mode;  // 0: !(x < f), 1: always, 2: NaN only
};
__device__ __forceinline__ KeyGE key_ge_of(uint64_t c) {
  if (c <= 0x007FFFFFull) return {0.f, 1};
  if (c > 0xFF800000ull) return {0.f, 2};
  return {key_to_float(static_cast<uint32_t>(c)), 0};
}
__device__ __forceinline__ bool key_ge(float x, const KeyGE& g) {
  return g.mode == 0 ? !(x < g.f) : (g.mode == 1 ? true : x != x);
}

constexpr int kWideTail = 4 * kThreads;  // keys past one segment a single CTA also takes

// Unsorted selection for a row of up to 32768 + 4096 keys in one CTA (a row just past one
// histogram segment, started from the summed histograms of its two segments): thread t owns
// its 32 keys [32t, 32t + 32) and the four tail keys [32768 + 4t, 32768 + 4t + 4), so thread
// order is index order within each part.  There is no candidate list: both narrowing levels
// (key bits 19..9 in 2048 bins, then 8..0 in 512, counted over the row copy itself) and the
// ordered take run over the row, so the k-th key's bin may hold any number of keys.  The
// take writes the keys above the final range and the lowest-index keys inside it that
// complete k, in ascending index order, like the general path.  `hists` (2048 words) is zero
// on entry.
// (a separate function, so that its registers do not weigh on the common path; the output
// row pointers come in by value)
__device__ __noinline__ void take_wide(int n, int k, const float* rowf, const int32_t* irow,
                                       uint32_t* hists, uint32_t* wa, uint32_t* wb,
                                       uint32_t* res, uint32_t* s_total, uint32_t clo,
                                       uint32_t chi, uint32_t k_rem, int32_t* oi32,
                                       int64_t* oi64, float* ov, int32_t* om) {
  constexpr int kMain = 32 * kThreads;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tbase = tid * 32, tail0 = kMain + 4 * tid;
  const uint32_t uk = static_cast<uint32_t>(k);
  // the thread's keys as floats: register slot (j, c) holds element tbase + 4 qq + c with
  // qq = (j + lane) & 7 (rotated, conflict-free 16-byte reads); bit b of a main mask is
  // element tbase + b, so masks are in index order whatever the slot order
  float xm[32], xt[4];
  uint32_t vm = 0u;  // slots inside the row, bit 4 j + c
  {
    const float4* r4 = reinterpret_cast<const float4*>(rowf) + tid * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int qq = (j + lane) & 7;
      const float4 v = r4[qq];
      xm[4 * j] = v.x;
      xm[4 * j + 1] = v.y;
      xm[4 * j + 2] = v.z;
      xm[4 * j + 3] = v.w;
#pragma unroll
      for (int c = 0; c < 4; ++c) vm |= (tbase + 4 * qq + c < n ? 1u : 0u) << (4 * j + c);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) xt[c] = tail0 + c < n ? rowf[tail0 + c] : -INFINITY;
  }
  const uint32_t vtail = tail0 + 4 <= n ? 0xFu : (tail0 >= n ? 0u : (1u << (n - tail0)) - 1u);

  // ---- the exact k-th key inside [clo, chi]: bits 19..9, then 8..0
  uint32_t flo = clo, fhi = chi, fk = k_rem;
  for (int level = 0; level < 2; ++level) {
    const int sh = level == 0 ? 9 : 0;
    const uint32_t mask = level == 0 ? 0x7FFu : 0x1FFu;
    const int nb = level == 0 ? 2048 : 512;
    if (level == 1) {
      if (tid < 512) hists[tid] = 0u;  // every thread holds its level-1 counts already
      __syncthreads();
    }
    const KeyGE lo = key_ge_of(flo), hi = key_ge_of(static_cast<uint64_t>(fhi) + 1u);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (((vm >> j) & 1u) && key_ge(xm[j], lo) && !key_ge(xm[j], hi))
        atomicAdd(&hists[(float_to_key(xm[j]) >> sh) & mask], 1u);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (((vtail >> c) & 1u) && key_ge(xt[c], lo) && !key_ge(xt[c], hi))
        atomicAdd(&hists[(float_to_key(xt[c]) >> sh) & mask], 1u);
    __syncthreads();
    uint32_t c4[4];
    bins_from_top(hists, nb, c4);
    pick_bin(c4, nb, fk, wa, wb, res);
    if (!res[3]) break;  // counts short of fk: the histogram did not describe the row
    flo |= res[0] << sh;
    fhi = level == 0 ? (flo | 0x1FFu) : flo;
    const bool done = res[2] == res[1];  // every key of the range is taken
    fk = res[1];
    if (done) break;
  }

  // ---- the take: keys above [flo, fhi], and the first fk inside it, in index order
  const KeyGE lo = key_ge_of(flo), hi = key_ge_of(static_cast<uint64_t>(fhi) + 1u);
  uint32_t gm = 0u, em = 0u, gtl = 0u, etl = 0u;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const bool v = (vm >> j) & 1u;
    const bool gt = v && key_ge(xm[j], hi), ge = v && key_ge(xm[j], lo);
    const int b = 4 * (((j >> 2) + lane) & 7) + (j & 3);  // the slot's element, as a bit
    gm |= (gt ? 1u : 0u) << b;
    em |= (ge && !gt ? 1u : 0u) << b;
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const bool v = (vtail >> c) & 1u;
    const bool gt = v && key_ge(xt[c], hi), ge = v && key_ge(xt[c], lo);
    gtl |= (gt ? 1u : 0u) << c;
    etl |= (ge && !gt ? 1u : 0u) << c;
  }
  // the main part's counts, then the tail's after all of it; a row holds < 65536 keys, so
  // the packed halves do not carry
  const uint32_t bm = block_excl_scan(static_cast<uint32_t>(__popc(gm)) |
                                          (static_cast<uint32_t>(__popc(em)) << 16),
                                      wa, wb, s_total);
  const uint32_t main_total = *s_total;
  const uint32_t bt = block_excl_scan(static_cast<uint32_t>(__popc(gtl)) |
                                          (static_cast<uint32_t>(__popc(etl)) << 16),
                                      wa, wb, s_total);
  auto emit = [&](uint32_t& g, uint32_t& eb, bool gt, int e, float x) {
    uint32_t p = 0xFFFFFFFFu;
    if (gt) {
      p = g + min(eb, fk);
      ++g;
    } else {
      if (eb < fk) p = g + eb;
      ++eb;
    }
    if (p < uk) {
      const uint32_t gi = irow ? static_cast<uint32_t>(irow[e]) : static_cast<uint32_t>(e);
      if (oi32) oi32[p] = static_cast<int32_t>(gi);
      if (oi64) oi64[p] = static_cast<int64_t>(gi);
      if (om) om[p] = static_cast<int32_t>(gi);
      if (ov) ov[p] = key_to_float(float_to_key(x));
    }
  };
  uint32_t g = bm & 0xFFFFu, eb = bm >> 16;
  for (uint32_t t = gm | em; t; t &= t - 1u) {  // index order
    const int b = __ffs(t) - 1;
    emit(g, eb, (gm >> b) & 1u, tbase + b, rowf[tbase + b]);
  }
  g = (main_total & 0xFFFFu) + (bt & 0xFFFFu);
  eb = (main_total >> 16) + (bt >> 16);
#pragma unroll
  for (int c = 0; c < 4; ++c)
    if (((gtl | etl) >> c) & 1u) emit(g, eb, (gtl >> c) & 1u, tail0 + c, xt[c]);
}

// Merge of an exchange (topk_segment_kernel with a.gather set), before the selection:
//   1. the step's epoch is the region's last one + 1; the grid's last CTA to read it stores
//      it back for the next step;
//   2. this rank's row of the local top-k (indices made global) goes into the region under
//      the epoch's parity, and one release store per rank (system scope: over NVLink for a
//      peer) puts the epoch into that rank's flag (parity, this rank, row);
//   3. a bounded wait until every rank's flag for this row holds the epoch (acquire);
//   4. the ranks' rows are copied from their regions (loads that bypass L1) into this row of
//      the local scratch, which the selection reads as its input (a.vals / a.idx).
// A wait that runs out raises TDSA_ERR_TIMEOUT and leaves the scratch as it was.  Reuse is
// safe with two parities: a rank publishes step s + 2 only after its step s + 1 merge saw
// every rank's step s + 1 flag, raised at the start of that rank's next launch after its
// step s merge had finished reading.
__device__ void gather_peer_row(const TopkArgs& a, int row) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_late;
  const PeerGather& g = a.pg;
  const int tid = threadIdx.x;
  uint32_t* ctr = reinterpret_cast<uint32_t*>(g.own + g.ctr_off);
  if (tid == 0) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(ctr) + 1u;
    s_epoch = epoch;
    s_late = 0;
    __threadfence();
    if (atomicAdd(ctr + 1, 1u) == gridDim.x * gridDim.y - 1u) {  // every CTA has read it
      ctr[1] = 0u;
      *reinterpret_cast<volatile uint32_t*>(ctr) = epoch;
    }
  }
  __syncthreads();
  const uint32_t epoch = s_epoch, parity = epoch & 1u;
  const int64_t slot = (static_cast<int64_t>(parity) * g.rows + row) * g.k;
  {
    float* dv = reinterpret_cast<float*>(g.own + g.vals_off) + slot;
    int32_t* di = reinterpret_cast<int32_t*>(g.own + g.idx_off) + slot;
    const float* sv = g.local_vals + static_cast<int64_t>(row) * g.local_stride;
    const int32_t* si = g.local_idx + static_cast<int64_t>(row) * g.local_stride;
    for (int e = tid; e < g.k; e += blockDim.x) {
      dv[e] = sv[e];
      di[e] = si[e] + g.offset;
    }
  }
  __syncthreads();  // the row, written by the whole CTA, before the release stores
  if (tid < g.world) {
    uint32_t* f = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(g.peer_base[tid]) +
                                              g.flags_off) +
                  (static_cast<int64_t>(parity) * g.world + g.rank) * g.rows + row;
    st_release_sys(f, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(g.own + g.flags_off) +
                           (static_cast<int64_t>(parity) * g.world + tid) * g.rows + row;
    const long long t0 = clock64();
    while (ld_acquire_sys(mine) != epoch) {
      if (clock64() - t0 > kWaitLimitCycles) {
        s_late = 1;
        atomicOr(a.status, TDSA_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  if (!s_late) {
    const int64_t count = static_cast<int64_t>(g.world) * g.k;
    float* dv = reinterpret_cast<float*>(g.own + g.scratch_v_off) + row * count;
    int32_t* di = reinterpret_cast<int32_t*>(g.own + g.scratch_i_off) + row * count;
    for (int r = 0; r < g.world; ++r) {
      const float* sv = reinterpret_cast<const float*>(g.peer_base[r] + g.vals_off) + slot;
      const int32_t* si = reinterpret_cast<const int32_t*>(g.peer_base[r] + g.idx_off) + slot;
      float* ov = dv + static_cast<int64_t>(r) * g.k;
      int32_t* oi = di + static_cast<int64_t>(r) * g.k;
      if ((g.k & 3) == 0) {
        for (int e = tid; e < g.k / 4; e += blockDim.x) {
          reinterpret_cast<float4*>(ov)[e] = __ldcv(reinterpret_cast<const float4*>(sv) + e);
          reinterpret_cast<int4*>(oi)[e] = __ldcv(reinterpret_cast<const int4*>(si) + e);
        }
      } else {
        for (int e = tid; e < g.k; e += blockDim.x) {
          ov[e] = __ldcv(sv + e);
          oi[e] = __ldcv(si + e);
        }
      }
    }
  }
  fence_proxy_async_global();  // the bulk copies of the selection read these stores
  __syncthreads();
}

// kPer keys per thread: segments of up to kPer * 1024 keys.  Thread t owns the kPer
// consecutive elements [kPer*t, kPer*t + kPer) (thread order is index order) and visits
// them rotated by its lane group, so a warp's 32 shared-memory reads hit 32 banks.
// kWide (kPer = 32): a row of up to 32768 + 4096 keys in one CTA, the unsorted final level of
// a row just past one histogram segment (launch_segments picks it by the chunk); the common
// instantiations carry none of its code.
template <int kPer, bool kWide>
__global__ void __launch_bounds__(kThreads, 1) topk_segment_kernel(const TopkArgs a) {
  static_assert(!kWide || kPer == 32, "wide rows run 32 keys per thread");
  extern __shared__ __align__(16) uint32_t sm[];
  __shared__ uint32_t wa[kWarps], wb[kWarps], wc[kWarps];
  __shared__ uint32_t res[4];
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t s_kth, s_total;
  __shared__ __align__(8) uint64_t s_bar[kWide ? 5 : 4];  // 32 KB pieces of the row
  __shared__ int s_abort;

  const int row = blockIdx.y, seg = blockIdx.x;
  const int start = seg * a.chunk;
  const int n = min(a.row_len - start, a.chunk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned lt = lanemask_lt();
  constexpr int kHists = 8;  // private histograms, one per 4 warps
  constexpr int kLog = kPer == 32 ? 5 : kPer == 16 ? 4 : kPer == 8 ? 3 : 2;
  static_assert((1 << kLog) == kPer, "kPer must be 4, 8, 16 or 32");
  const int rot = lane >> (5 - kLog);
  const int tbase = tid * kPer;
  // shared memory: [segment (floats, or keys) | sort pairs][list keys][list indices][hists]
  float* rowf = reinterpret_cast<float*>(sm);
  uint32_t* list_key = sm + a.row_words;
  uint32_t* list_idx = list_key + a.cap;
  uint32_t* hists = list_idx + a.cap;
  uint32_t* my_hist = hists + (warp & (kHists - 1)) * kBins;
  uint64_t* pairs = reinterpret_cast<uint64_t*>(sm);  // the segment copy is dead by then

  const float* vrow = a.vals + static_cast<int64_t>(row) * a.vals_stride + start;
  const int32_t* irow = a.idx ? a.idx + static_cast<int64_t>(row) * a.idx_stride + start : nullptr;
  const int k = min(a.k, n);

  // ---- 0. the segment into shared memory: bulk copies on the TMA engine (32 KB per
  // mbarrier) of its first n & ~3 keys when the row is 16-byte aligned, issued before the
  // histogram prologue so the two overlap, each thread then loading its own keys past them
  // (fewer than four in a row); else coalesced loads.  A thread's elements lie in one 32 KB
  // piece.
  // (common rows: whole rows of a multiple of four keys only, loads otherwise)
  const bool aligned = (reinterpret_cast<uintptr_t>(vrow) & 15u) == 0u;
  const int nbulk = kWide ? (aligned ? (n & ~3) : 0) : ((aligned && n % 4 == 0) ? n : 0);
  const bool bulk = nbulk > 0;
  const uint32_t bytes = static_cast<uint32_t>(nbulk) * 4u;
  const int npieces = static_cast<int>((bytes + 32767u) / 32768u);
  unsigned int tl_launch = 0;
  if (tid == 0) {
    tl_launch = TDSA_TL_TICKET(topk);
    if (seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 0);
    s_abort = 0;
    s_kth = 0xFFFFFFFFu;
    if (bulk) {
      for (int c = 0; c < npieces; ++c) mbar_init(&s_bar[c], 1);
      fence_mbar_init();
    }
  }
  for (int i = tid; i < kHists * kBins; i += kThreads) hists[i] = 0u;
  __syncthreads();
  pdl_wait();  // the scores and the histogram come from the previous kernel
  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 1);
  // Full-segment rows started from the histogram let the next kernel launch only once their
  // row copy has landed (below): a dependent query projection that starts staging its
  // weights during the copy slows this kernel's later phases more than it gains (config-4
  // step, same box: 0.8985 -> 0.8944 ms).
  const bool late_trigger = kPer == 32 && !kWide && a.hist != nullptr;
  if (!late_trigger) pdl_launch_dependents();
  if (a.gather) gather_peer_row(a, row);
  if (bulk) {
    if (tid == 0) {
      for (int c = 0; c < npieces; ++c) {
        const uint32_t off = static_cast<uint32_t>(c) * 32768u;
        const uint32_t len = min(32768u, bytes - off);
        mbar_arrive_expect_tx(&s_bar[c], len);
        bulk_load(reinterpret_cast<uint8_t*>(rowf) + off,
                  reinterpret_cast<const uint8_t*>(vrow) + off, len, &s_bar[c]);
      }
    }
  } else {
    const int w0 = warp * kPer * 32;
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int e = w0 + j * 32 + lane;
      if (e < n) rowf[e] = __ldg(vrow + e);
    }
    if constexpr (kWide)
      for (int e = kPer * kThreads + tid; e < n; e += kThreads) rowf[e] = __ldg(vrow + e);
    __syncwarp();
  }

  // ---- 1. initial live range [clo, chi] holding the k-th key; k - k_rem keys lie above
  uint32_t k_rem = static_cast<uint32_t>(k), in_range = static_cast<uint32_t>(n);
  uint32_t clo = 0u, chi = 0xFFFFFFFFu;
  bool hist_hit = false;  // the histogram gave the k-th key's 12-bit bin
  if (a.hist) {
    // The score kernel already counted this row's keys by their top 12 bits: find the bin of
    // the k-th key (thread t owns bins 4095-4t .. 4092-4t).
    // (a wide row covers two histogram segments: their sum)
    constexpr int hsegs = kWide ? 2 : 1;
    uint32_t* rh = a.hist + (static_cast<int64_t>(row) * gridDim.x + seg) * hsegs * kKeyHistBins;
    // the first segment's four bins outside any loop, so their loads go out together
    uint32_t c[4], tot = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = rh[kKeyHistBins - 1 - (4 * tid + i)];
    for (int g = 1; g < hsegs; ++g) {
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] += rh[g * kKeyHistBins + kKeyHistBins - 1 - (4 * tid + i)];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) tot += c[i];
    if (tid == 0) res[3] = 0u;
    uint32_t dummy;
    uint32_t above = block_excl_scan(tot, wa, wb, &dummy);
    if (above < k_rem && k_rem <= above + tot) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (above < k_rem && k_rem <= above + c[i]) {
          res[0] = kKeyHistBins - 1 - (4 * tid + i);
          res[1] = k_rem - above;
          res[2] = c[i];
          res[3] = 1u;
        }
        above += c[i];
      }
    }
    for (int g = 0; g < hsegs; ++g)  // ready for reuse
#pragma unroll
      for (int i = 0; i < 4; ++i) rh[g * kKeyHistBins + kKeyHistBins - 1 - (4 * tid + i)] = 0u;
    __syncthreads();
    if (res[3]) {  // (a histogram that does not describe the row leaves the full range)
      clo = res[0] << 20;
      chi = clo | 0xFFFFFu;
      k_rem = res[1];
      in_range = res[2];
      hist_hit = true;
    }
  }
  if constexpr (kWide) {
    const int tail0 = kPer * kThreads + 4 * tid;  // this thread's four tail keys
    if (bulk) {
      if (tbase < nbulk) mbar_wait(&s_bar[(tbase * 4) >> 15], 0, &s_abort);
      if (tail0 < nbulk) mbar_wait(&s_bar[(tail0 * 4) >> 15], 0, &s_abort);
      for (int e = max(tbase, nbulk); e < min(tbase + kPer, n); ++e) rowf[e] = __ldg(vrow + e);
      for (int e = max(tail0, nbulk); e < min(tail0 + 4, n); ++e) rowf[e] = __ldg(vrow + e);
    }
  } else {
    if (bulk && tbase < n) mbar_wait(&s_bar[(tbase * 4) >> 15], 0, &s_abort);
  }

  // Keys are computed from the floats on the fly, or (no histogram: the min/max pass
  // visits every element anyway) converted once in place.
  const bool stored = a.hist == nullptr;
  auto key_at = [&](int e) -> uint32_t {
    return stored ? sm[e] : float_to_key(rowf[e]);
  };
  if (stored) {
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int e = tbase + ((j + rot) & (kPer - 1));
      if (e < n) {
        const uint32_t u = float_to_key(rowf[e]);
        sm[e] = u;
        kmin = min(kmin, u);
        kmax = max(kmax, u);
      }
    }
    kmin = __reduce_min_sync(0xffffffffu, kmin);
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) {
      wa[warp] = kmin;
      wc[warp] = kmax;
    }
  }
  __syncthreads();
  if (tid == 0 && seg == 0) TDSA_TL_REC(topk, 64, 7, tl_launch, row, 2);
  if (late_trigger) pdl_launch_dependents();
  if (s_abort) {
    // a bulk copy did not land in time: report, and let the copies in flight finish
    if (tid == 0) {
      atomicOr(a.status, TDSA_ERR_TIMEOUT);
      volatile int no_abort = 0;
      for (int c = 0; c < npieces; ++c) mbar_wait(&s_bar[c], 0, &no_abort);
    }
    return;
  }
  if (stored) {
    clo = __reduce_min_sync(0xffffffffu, wa[lane]);
    chi = __reduce_max_sync(0xffffffffu, wc[lane]);
  }
  if constexpr (kWide) {
    {  // the host routes only unsorted final levels here
      if (hist_hit && static_cast<uint32_t>(k) - k_rem + in_range <= static_cast<uint32_t>(a.cap)) {
        take_from_bin<kPer, true>(a, row, seg, start, n, k, rowf, irow, list_key, list_idx,
                                  hists, wa, wc, res, &s_total, clo, chi, k_rem, in_range,
                                  tl_launch);
      } else if (hist_hit) {  // the k-th key's bin holds more keys than the list: no list
        const int64_t orow = row;  // one segment per row
        take_wide(n, k, rowf, irow, hists, wa, wc, res, &s_total, clo, chi, k_rem,
                  a.idx_bytes == 4 ? static_cast<int32_t*>(a.out_idx) + orow * a.out_idx_stride
                                   : nullptr,
                  a.idx_bytes == 8 ? static_cast<int64_t*>(a.out_idx) + orow * a.out_idx_stride
                                   : nullptr,
                  a.out_val ? a.out_val + orow * a.out_val_stride : nullptr,
                  a.mirror ? a.mirror + orow * a.mirror_stride : nullptr);
      } else if (tid == 0) {
        atomicOr(a.status, TDSA_STATUS_HIST);  // the histograms did not describe the row
      }
      return;
    }
  }
  if (hist_hit && !a.sorted && !a.kth_out && a.out_idx &&
      static_cast<uint32_t>(k) - k_rem + in_range <= static_cast<uint32_t>(a.cap)) {
    take_from_bin<kPer, false>(a, row, seg, start, n, k, rowf, irow, list_key, list_idx, hists,
                               wa, wc, res, &s_total, clo, chi, k_rem, in_range, tl_launch);
    return;
  }

  // ---- 2. narrow over the segment until the keys >= clo fit the list.  A k larger than
  // the list is written straight to the output, which needs the exact k-th key first.
  const bool direct = k > a.cap;
  bool dirty = false;
  for (int pass = 0; pass < 4 && clo != chi && in_range != k_rem &&
                     (direct || static_cast<uint32_t>(k) - k_rem + in_range > a.cap);
       ++pass) {
    const int sh = max(0, bit_length(chi - clo) - 8);
    if (dirty) {
      for (int i = tid; i < kHists * kBins; i += kThreads) hists[i] = 0u;
      __syncthreads();
    }
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int e = tbase + ((j + rot) & (kPer - 1));
      const uint32_t u = e < n ? key_at(e) : 0u;
      const bool in = e < n && u >= clo && u <= chi;
      add_to_bin(my_hist, in, in ? (u - clo) >> sh : 0u);
    }
    __syncthreads();
    narrow_to_bin(hists, hist, res, sh, clo, chi, k_rem, in_range);
    dirty = true;
  }
  // All keys in [clo, chi] join the list when they fit; otherwise the range is one value
  // (or all of it is taken) and only the first k_rem of them by index do.
  const bool fits = !direct && static_cast<uint32_t>(k) - k_rem + in_range <= a.cap;

  // ---- 3. ordered compaction into the list (or the output, when direct): per-thread bit
  // masks of the elements taken, bit j = element tbase + j, then one scan for positions.
  uint32_t take = 0;
  if (fits && !stored && kPer == 32 && clo <= 0xFF800000u) {
    // Compare the floats themselves: key(x) >= clo  <=>  !(x < f_lo), f_lo the float of
    // clo (-inf when clo is at or below the key of -inf).  Exact for +-0 (one key) and
    // NaN (the largest key; every comparison with NaN is false).  Eight conflict-free
    // 16-byte reads per thread, rotated by lane.
    const float f_lo = clo <= 0x007FFFFFu ? -INFINITY : key_to_float(clo);
    const float4* r4 = reinterpret_cast<const float4*>(rowf) + tid * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int qq = (j + lane) & 7;
      const float4 v = r4[qq];
      const int e0 = tbase + 4 * qq;
      uint32_t b = 0;
      b |= (e0 + 0 < n && !(v.x < f_lo)) ? 1u : 0u;
      b |= (e0 + 1 < n && !(v.y < f_lo)) ? 2u : 0u;
      b |= (e0 + 2 < n && !(v.z < f_lo)) ? 4u : 0u;
      b |= (e0 + 3 < n && !(v.w < f_lo)) ? 8u : 0u;
      take |= b << (4 * qq);
    }
  } else if (fits) {
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int jj = (j + rot) & (kPer - 1);
      const int e = tbase + jj;
      if (e < n && key_at(e) >= clo) take |= 1u << jj;
    }
  } else {
    uint32_t gtm = 0, eqm = 0;
#pragma unroll 8
    for (int j = 0; j < kPer; ++j) {
      const int jj = (j + rot) & (kPer - 1);
      const int e = tbase + jj;
      if (e < n) {
        const uint32_t u = key_at(e);
        if (u > chi) gtm |= 1u << jj;
        else if (u >= clo) eqm |= 1u << jj;
      }
    }
    uint32_t dummy;
    const uint32_t eq_before = block_excl_scan(__popc(eqm), wa, wb, &dummy);
    const uint32_t n_eq = eq_before >= k_rem ? 0u : min(static_cast<uint32_t>(__popc(eqm)),
                                                        k_rem - eq_before);
    uint32_t rest = eqm;
    for (uint32_t i = 0; i < n_eq; ++i) rest &= rest - 1u;  // drop the lowest n_eq
    take = gtm | (eqm ^ rest);
  }
  uint32_t pos = block_excl_scan(__popc(take), wa, wc, &s_total);

  const int64_t out_row = static_cast<int64_t>(row) * gridDim.x + seg;
  int32_t* oi32 = a.out_idx && a.idx_bytes == 4
                      ? static_cast<int32_t*>(a.out_idx) + out_row * a.out_idx_stride : nullptr;
  int64_t* oi64 = a.out_idx && a.idx_bytes == 8
                      ? static_cast<int64_t*>(a.out_idx) + out_row * a.out_idx_stride : nullptr;
  float* ov = a.out_idx && a.out_val ? a.out_val + out_row * a.out_val_stride : nullptr;
  int32_t* om = a.mirror ? a.mirror + out_row * a.mirror_stride : nullptr;
  if (a.pad_to_k && n < a.k) {
    // pads rank below every real candidate of the next level (-inf, then the largest index)
    for (int j = n + tid; j < a.k; j += kThreads) {
      if (oi32) oi32[j] = 0x7FFFFFFF;
      if (ov) ov[j] = -INFINITY;
    }
    if (tid == 0 && a.next_hist)
      atomicAdd(a.next_hist + static_cast<int64_t>(row) * kKeyHistBins +
                    (float_to_key(-INFINITY) >> 20),
                static_cast<uint32_t>(a.k - n));
  }
  uint32_t kth_local = 0xFFFFFFFFu;
  while (take) {
    const int jb = __ffs(take) - 1;
    take &= take - 1u;
    const int e = tbase + jb;
    const uint32_t u = key_at(e);
    const uint32_t gi = irow ? static_cast<uint32_t>(irow[e]) : static_cast<uint32_t>(start + e);
    if (direct) {
      if (oi32) oi32[pos] = static_cast<int32_t>(gi);
      if (oi64) oi64[pos] = static_cast<int64_t>(gi);
      if (om) om[pos] = static_cast<int32_t>(gi);
      if (ov) ov[pos] = key_to_float(u);
      if (u <= chi) kth_local = min(kth_local, u);
    } else if (pos < static_cast<uint32_t>(a.cap)) {
      list_key[pos] = u;
      list_idx[pos] = gi;
    }
    ++pos;
  }
  if (direct) {  // the output is complete; the k-th key is the smallest taken in range
    kth_local = __reduce_min_sync(0xffffffffu, kth_local);
    if (lane == 0 && kth_local != 0xFFFFFFFFu) atomicMin(&s_kth, kth_local);
    __syncthreads();
    if (tid == 0 && a.kth_out) a.kth_out[out_row] = key_to_float(s_kth);
    return;
  }
  __syncthreads();
  const int m = min(static_cast<int>(s_total), a.cap);

  // ---- 4. narrow the list to the exact k-th key (keys in the list above chi are taken)
  for (int pass = 0; pass < 4 && clo != chi && in_range != k_rem; ++pass) {
    const int sh = max(0, bit_length(chi - clo) - 8);
    for (int i = tid; i < kHists * kBins; i += kThreads) hists[i] = 0u;
    __syncthreads();
    for (int i = tid; i < m; i += kThreads) {
      const uint32_t u = list_key[i];
      if (u >= clo && u <= chi) atomicAdd(&my_hist[(u - clo) >> sh], 1u);
    }
    __syncthreads();
    narrow_to_bin(hists, hist, res, sh, clo, chi, k_rem, in_range);
  }
  const bool whole = in_range == k_rem;  // every key in [clo, chi] is taken

  // Final take over the list in index order: warp w owns list entries [w*span, (w+1)*span).
  const int span = ((m + kWarps * 32 - 1) / (kWarps * 32)) * 32;
  const int lbase = warp * span + lane;
  uint32_t leq_w = 0;
  if (!whole) {
    for (int i = lbase; i < warp * span + span; i += 32) {
      const uint32_t u = i < m ? list_key[i] : 0u;
      leq_w += __popc(__ballot_sync(0xffffffffu, i < m && u >= clo && u <= chi));
    }
    if (lane == 0) wa[warp] = leq_w;
    __syncthreads();
    if (warp == 0) warp_totals_scan(wa, wb);
    __syncthreads();
  }
  uint32_t lgt_w = 0, ltake = 0;
  {
    // taken entries in earlier warps = list entries before them minus untaken in-range ones
    const uint32_t eqb = whole ? 0u : wb[warp];
    ltake = whole ? 0u : (eqb >= k_rem ? 0u : min(leq_w, k_rem - eqb));
    for (int i = lbase; i < warp * span + span; i += 32) {
      const uint32_t u = i < m ? list_key[i] : 0u;
      lgt_w += __popc(__ballot_sync(0xffffffffu, i < m && (u > chi || (whole && u >= clo))));
    }
    if (lane == 0) wa[warp] = lgt_w + ltake;
    __syncthreads();
    if (warp == 0) warp_totals_scan(wa, wc);
    __syncthreads();
  }
  const bool write_pairs = a.sorted != 0;
  uint32_t pos_base = wc[warp], eq_seen = 0;
  kth_local = 0xFFFFFFFFu;
  for (int i = lbase; i < warp * span + span; i += 32) {
    const bool valid = i < m;
    const uint32_t u = valid ? list_key[i] : 0u;
    const bool eq = valid && u >= clo && u <= chi;
    const bool gt = valid && (u > chi || (whole && eq));
    bool take = gt;
    unsigned bt = __ballot_sync(0xffffffffu, gt);
    if (!whole) {
      const unsigned be = __ballot_sync(0xffffffffu, eq);
      if (be) {
        take = gt || (eq && eq_seen + __popc(be & lt) < ltake);
        bt = __ballot_sync(0xffffffffu, take);
        eq_seen += __popc(be);
      }
    }
    if (take && (eq || whole)) kth_local = min(kth_local, u);
    const uint32_t pos = pos_base + __popc(bt & lt);
    if (a.next_hist)  // the next level starts from the bins of what this segment passes on
      add_to_bin(a.next_hist + static_cast<int64_t>(row) * kKeyHistBins,
                 take && pos < static_cast<uint32_t>(k), u >> 20);
    if (take && pos < static_cast<uint32_t>(k)) {
      const uint32_t gi = list_idx[i];
      if (write_pairs) {
        // pairs alias the segment copy, which no thread reads any more
        pairs[pos] = (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - gi);
      } else {
        if (oi32) oi32[pos] = static_cast<int32_t>(gi);
        if (oi64) oi64[pos] = static_cast<int64_t>(gi);
        if (om) om[pos] = static_cast<int32_t>(gi);
        if (ov) ov[pos] = key_to_float(u);
      }
    }
    pos_base += __popc(bt);
  }
  kth_local = __reduce_min_sync(0xffffffffu, kth_local);
  if (lane == 0 && kth_local != 0xFFFFFFFFu) atomicMin(&s_kth, kth_local);
  __syncthreads();
  if (tid == 0 && a.kth_out) a.kth_out[out_row] = key_to_float(s_kth);
  if (!a.sorted) return;

  // Bitonic sort of the k selected (key, ~index) pairs, descending; padding sorts last.
  int kp = 1;
  while (kp < k) kp <<= 1;
  for (int i = k + tid; i < kp; i += kThreads) pairs[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= kp; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < (kp >> 1); i += kThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const uint64_t x = pairs[lo], y = pairs[hi];
        const bool desc = (lo & size) == 0;
        if (desc ? (x < y) : (x > y)) {
          pairs[lo] = y;
          pairs[hi] = x;
        }
      }
      __syncthreads();
    }
  }
  if (!a.out_idx) return;
  for (int j = tid; j < k; j += kThreads) {
    const uint64_t p = pairs[j];
    const uint32_t gi = 0xFFFFFFFFu - static_cast<uint32_t>(p & 0xFFFFFFFFull);
    if (oi64) oi64[j] = static_cast<int64_t>(gi);
    if (oi32) oi32[j] = static_cast<int32_t>(gi);
    if (om) om[j] = static_cast<int32_t>(gi);
    if (ov) ov[j] = key_to_float(static_cast<uint32_t>(p >> 32));
  }
}

// ---------------------------------------------------------------------------------------
// Cluster top-k: one row over the kC CTAs of a cluster, for batches too small to fill the
// GPU one CTA per row: rows of up to 32768 keys (one histogram segment) over 2-8 CTAs, and
// rows of up to 131072 keys over 8 CTAs in place of the levels.  Unsorted output, and the
// score kernel's 12-bit key histograms of the row's 32768-key segments (summed).  CTA r of
// the cluster holds keys
// [r*kPer*1024, (r+1)*kPer*1024) in registers: warp w the 32*kPer keys from
// r*kPer*1024 + w*32*kPer, in chunks of 32*kV (kV = min(kPer, 4)) with lane l holding kV
// consecutive keys of each chunk, so every load is one coalesced 128-512 byte access and
// index order is (rank, warp, chunk, lane, element).
//   1. The bin of the k-th key in the score kernel's histogram (every CTA scans it; the
//      histogram loads go out with the score loads).
//   2. Then bits 19..8 and 7..0 of the key: each CTA counts its keys of the live range into a
//      local histogram, adds the non-zero bins into every CTA's copy of the cluster's
//      histogram (distributed shared memory, `red.shared::cluster`), one cluster barrier,
//      and every CTA picks the same bin.  Narrowing stops once the range holds exactly the
//      keys still to take, or is one key.
//   3. Keys above the range are taken, and the lowest-index keys inside it complete k (the
//      tie rule of stable_topk, metrics.py:9-22).  Output positions follow index order: the
//      CTAs' (above, inside) counts go to every CTA of the cluster, warps are offset by a
//      CTA scan of their totals, lanes by a warp scan per chunk.
// The row's histogram is zeroed for the next score launch after every CTA has read it.
constexpr int kClusterHistWords = 2 * kKeyHistBins + 256;  // cluster levels 2 and 3

template <int kPer, int kC>
__global__ void __cluster_dims__(kC, 1, 1) __launch_bounds__(kThreads, 1)
    topk_cluster_kernel(const TopkArgs a) {
  static_assert(kPer >= 1 && kPer <= 16 && (kPer & (kPer - 1)) == 0, "kPer: 1..16, power of 2");
  constexpr int kV = kPer < 4 ? kPer : 4;  // consecutive keys per lane in a chunk
  constexpr int kChunks = kPer / kV;
  constexpr uint32_t kVMask = (1u << kV) - 1u;
  extern __shared__ __align__(16) uint32_t csm[];
  __shared__ uint32_t hloc[kKeyHistBins];  // this CTA's keys of the live range, by bin
  __shared__ uint32_t wa[kWarps], wb[kWarps], res[4];
  __shared__ uint32_t s_cnt[kC];  // per rank: above | inside << 16
  uint32_t* hred2 = csm;                     // cluster counts, bits 19..8 (4096 bins)
  uint32_t* hred1 = csm + kKeyHistBins;      // bits 31..20, when the histogram is unusable
  uint32_t* hred3 = csm + 2 * kKeyHistBins;  // cluster counts, bits 7..0 (256 bins)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  const int row = blockIdx.y;
  const int n = a.row_len;
  const uint32_t k = static_cast<uint32_t>(min(a.k, n));
  const int wbase = static_cast<int>(rank) * (kPer * kThreads) + warp * (32 * kPer);

  for (int i = tid; i < kClusterHistWords; i += kThreads) csm[i] = 0u;
  cluster_arrive();  // waited for before the first add into a peer's histogram
  pdl_wait();        // the scores and the histogram come from the previous kernel
  pdl_launch_dependents();

  // ---- the row's histogram counts and the keys (loads issued together)
  uint32_t* gh = a.hist + static_cast<int64_t>(row) * a.hist_segs * kKeyHistBins;
  uint32_t c4[4];
  bins_from_top(gh, kKeyHistBins, c4);
  for (int sg = 1; sg < a.hist_segs; ++sg) {  // a row of several segments: their sum
    uint32_t t4[4];
    bins_from_top(gh + sg * kKeyHistBins, kKeyHistBins, t4);
#pragma unroll
    for (int i = 0; i < 4; ++i) c4[i] += t4[i];
  }
  const float* vrow = a.vals + static_cast<int64_t>(row) * a.vals_stride;
  const bool vec = (reinterpret_cast<uintptr_t>(vrow) & (kV * 4 - 1)) == 0;
  uint32_t u[kPer];
  uint32_t valid = 0;  // bit i: key i of this lane lies inside the row
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int e0 = wbase + j * 32 * kV + lane * kV;
    if (vec && e0 + kV <= n) {
      if constexpr (kV == 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(vrow + e0));
        u[4 * j] = float_to_key(v.x);
        u[4 * j + 1] = float_to_key(v.y);
        u[4 * j + 2] = float_to_key(v.z);
        u[4 * j + 3] = float_to_key(v.w);
      } else if constexpr (kV == 2) {
        const float2 v = __ldg(reinterpret_cast<const float2*>(vrow + e0));
        u[2 * j] = float_to_key(v.x);
        u[2 * j + 1] = float_to_key(v.y);
      } else {
        u[j] = float_to_key(__ldg(vrow + e0));
      }
      valid |= kVMask << (j * kV);
    } else {
#pragma unroll
      for (int s = 0; s < kV; ++s) {
        const bool in = e0 + s < n;
        u[j * kV + s] = in ? float_to_key(__ldg(vrow + e0 + s)) : 0u;
        valid |= (in ? 1u : 0u) << (j * kV + s);
      }
    }
  }

  // ---- 1. the k-th key's top-12-bit bin from the score kernel's histogram
  uint32_t clo = 0u, chi = 0xFFFFFFFFu, k_rem = k, in_range = static_cast<uint32_t>(n);
  pick_bin(c4, kKeyHistBins, k_rem, wa, wb, res);
  int level = 0;
  if (res[3]) {
    clo = res[0] << 20;
    chi = clo | 0xFFFFFu;
    k_rem = res[1];
    in_range = res[2];
    level = 1;
  }
  cluster_wait();  // every CTA's cluster histograms are zero

  // ---- 2. cluster narrowing levels (level 0 only when the histogram does not describe
  // the row: its counts total less than k)
  for (; level < 3 && clo != chi && in_range != k_rem; ++level) {
    const int sh = level == 0 ? 20 : level == 1 ? 8 : 0;
    const int nb = level == 2 ? 256 : kKeyHistBins;
    uint32_t* hr = level == 0 ? hred1 : level == 1 ? hred2 : hred3;
    for (int i = tid; i < nb; i += kThreads) hloc[i] = 0u;
    __syncthreads();
    // a range holding many keys (ties) is counted with per-warp aggregation
    const bool heavy = in_range > static_cast<uint32_t>(n) / 16u;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const bool in = ((valid >> i) & 1u) && u[i] >= clo && u[i] <= chi;
      const uint32_t bin = (u[i] >> sh) & static_cast<uint32_t>(nb - 1);
      if (heavy) add_to_bin(hloc, in, in ? bin : 0u);
      else if (in) atomicAdd(&hloc[bin], 1u);
    }
    __syncthreads();
    for (int i = tid; i < nb; i += kThreads) {
      const uint32_t c = hloc[i];
      if (c) {
        const uint32_t la = smem_u32(hr + i);
#pragma unroll
        for (int r = 0; r < kC; ++r) red_cluster_add_u32(mapa_shared(la, r), c);
      }
    }
    cluster_sync_all();
    bins_from_top(hr, nb, c4);
    pick_bin(c4, nb, k_rem, wa, wb, res);
    if (!res[3]) break;  // counts short of k_rem: the histogram did not match the scores
    clo |= res[0] << sh;
    chi = clo | ((1u << sh) - 1u);
    k_rem = res[1];
    in_range = res[2];
  }

  // ---- 3. take: keys above chi, and the first k_rem keys of [clo, chi] in index order
  uint32_t gtm = 0u, eqm = 0u;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    if ((valid >> i) & 1u) {
      if (u[i] > chi) gtm |= 1u << i;
      else if (u[i] >= clo) eqm |= 1u << i;
    }
  }
  // warp totals (above | inside << 16) -> warp offsets in the CTA -> CTA offsets in the row
  const uint32_t wt = __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(__popc(gtm)) |
                                                         (static_cast<uint32_t>(__popc(eqm)) << 16));
  if (lane == 0) wa[warp] = wt;
  __syncthreads();
  if (warp == 0) {
    warp_totals_scan(wa, wb);
    __syncwarp();
    const uint32_t cta_total = wb[31] + wa[31];
    if (lane < kC) st_cluster_u32(mapa_shared(smem_u32(&s_cnt[rank]), lane), cta_total);
  }
  cluster_sync_all();  // the last access to a peer's shared memory
  for (int sg = 0; sg < a.hist_segs; ++sg)
    for (int i = static_cast<int>(rank) * (kKeyHistBins / kC) + tid;
         i < static_cast<int>(rank + 1) * (kKeyHistBins / kC); i += kThreads)
      gh[sg * kKeyHistBins + i] = 0u;  // every CTA has read the histogram: ready for reuse
  // running (above, inside) counts before this warp's keys: 32-bit each, since a row of
  // several segments can hold more than 65535 of either (the packed halves hold one CTA's)
  uint32_t run_gt = wb[warp] & 0xFFFFu, run_eq = wb[warp] >> 16;
  for (uint32_t r = 0; r < rank; ++r) {
    run_gt += s_cnt[r] & 0xFFFFu;
    run_eq += s_cnt[r] >> 16;
  }

  const int64_t orow = static_cast<int64_t>(row);
  int32_t* oi32 = a.out_idx && a.idx_bytes == 4
                      ? static_cast<int32_t*>(a.out_idx) + orow * a.out_idx_stride : nullptr;
  int64_t* oi64 = a.out_idx && a.idx_bytes == 8
                      ? static_cast<int64_t*>(a.out_idx) + orow * a.out_idx_stride : nullptr;
  float* ov = a.out_val ? a.out_val + orow * a.out_val_stride : nullptr;
  int32_t* om = a.mirror ? a.mirror + orow * a.mirror_stride : nullptr;
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const uint32_t g = (gtm >> (j * kV)) & kVMask, q = (eqm >> (j * kV)) & kVMask;
    const uint32_t mine = static_cast<uint32_t>(__popc(g)) | (static_cast<uint32_t>(__popc(q)) << 16);
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t chunk_total = __shfl_sync(0xffffffffu, incl, 31);
    if (g | q) {
      const uint32_t ex = incl - mine;
      uint32_t gtb = run_gt + (ex & 0xFFFFu), eqb = run_eq + (ex >> 16);
      const int e0 = wbase + j * 32 * kV + lane * kV;
#pragma unroll
      for (int s = 0; s < kV; ++s) {
        uint32_t pos = 0xFFFFFFFFu;
        if ((g >> s) & 1u) {
          pos = gtb + min(eqb, k_rem);
          ++gtb;
        } else if ((q >> s) & 1u) {
          if (eqb < k_rem) pos = gtb + eqb;
          ++eqb;
        }
        if (pos < k) {
          if (oi32) oi32[pos] = e0 + s;
          if (oi64) oi64[pos] = e0 + s;
          if (om) om[pos] = e0 + s;
          if (ov) ov[pos] = key_to_float(u[j * kV + s]);
        }
      }
    }
    run_gt += chunk_total & 0xFFFFu;
    run_eq += chunk_total >> 16;
  }
}

int kpow2(int k) {
  int p = 1;
  while (p < k) p <<= 1;
  return p;
}

// Words of the segment region: the segment copy, reused for the sort pairs.
int row_words(int chunk, int k, int sorted) {
  const int pairs = sorted ? 2 * kpow2(k) : 0;
  return ((std::max(chunk, pairs) + 3) / 4) * 4;
}

int list_cap(int chunk) { return std::min(kCap, ((chunk + 3) / 4) * 4); }

size_t segment_smem(int chunk, int k, int sorted) {
  return static_cast<size_t>(row_words(chunk, k, sorted)) * 4 +
         static_cast<size_t>(list_cap(chunk)) * 8 + static_cast<size_t>(8) * kBins * 4;
}

int launch_segments(TopkArgs a, int rows, int nseg, cudaStream_t stream) {
  const size_t smem = segment_smem(a.chunk, a.k, a.sorted);
  a.row_words = row_words(a.chunk, a.k, a.sorted);
  a.cap = list_cap(a.chunk);
  a.status = device_status_ptr();
  if (!a.status) return fail(TDSA_ERR_CUDA, "device status word not available");
  auto run = [&](auto kern) -> int {
    TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(kern),
                                        static_cast<int>(smem)));
    TDSA_CUDA_CHECK(launch_pdl(kern, dim3(nseg, rows), dim3(kThreads), smem, stream, a));
    TDSA_CUDA_CHECK(cudaGetLastError());
    return TDSA_OK;
  };
  if (a.chunk <= 4 * kThreads) return run(topk_segment_kernel<4, false>);
  if (a.chunk <= 8 * kThreads) return run(topk_segment_kernel<8, false>);
  if (a.chunk <= 16 * kThreads) return run(topk_segment_kernel<16, false>);
  if (a.chunk <= 32 * kThreads) return run(topk_segment_kernel<32, false>);
  return run(topk_segment_kernel<32, true>);  // a row just past one segment (make_plan)
}

template <int kC>
int launch_cluster(const TopkArgs& a, int rows, int per, cudaStream_t stream) {
  auto run = [&](auto kern) -> int {
    constexpr int smem = kClusterHistWords * 4;
    TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
    TDSA_CUDA_CHECK(launch_pdl(kern, dim3(kC, rows), dim3(kThreads), smem, stream, a));
    TDSA_CUDA_CHECK(cudaGetLastError());
    return TDSA_OK;
  };
  if (per <= 1) return run(topk_cluster_kernel<1, kC>);
  if (per <= 2) return run(topk_cluster_kernel<2, kC>);
  if (per <= 4) return run(topk_cluster_kernel<4, kC>);
  if (per <= 8) return run(topk_cluster_kernel<8, kC>);
  if (per <= 16) return run(topk_cluster_kernel<16, kC>);
  return fail(TDSA_ERR_UNSUPPORTED, "cluster top-k: row too long for the cluster");
}

// Clusters of kC top-k CTAs the current device runs at once (one CTA per SM), queried once
// per device; 0 when the query fails (a failed query is not cached: the next call asks
// again, e.g. once the device has a context).
template <int kC>
int max_active_clusters() {
  static std::mutex mu;
  static int cache[64] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] <= 0) {
    const void* kern = reinterpret_cast<const void*>(topk_cluster_kernel<4, kC>);
    constexpr int smem = kClusterHistWords * 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kC, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    int nc = 0;
    if (ensure_dynamic_smem(kern, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      nc = 0;
    }
    cache[dev] = nc > 0 ? nc : 0;
  }
  return cache[dev];
}

// CTAs per row for the cluster top-k: the largest of 8, 4, 2 that runs the whole batch in
// one wave, leaves each CTA at least 2048 keys and each thread at most 8 (measured on
// B200 at 32768 keys per row, k = 2048: 8 CTAs 7.3 us, 4 CTAs 9.0 us, one CTA 10.5-12.7 us,
// but 2 CTAs of 16 keys per thread 12.2-14.5 us); 1 = one CTA per row (topk_segment_kernel).
int cluster_size(int batch, int length) {
  if (length >= 8 * 2048 && batch <= max_active_clusters<8>()) return 8;
  if (length >= 4 * 2048 && length <= 4 * 8 * kThreads && batch <= max_active_clusters<4>())
    return 4;
  if (length >= 2 * 2048 && length <= 2 * 8 * kThreads && batch <= max_active_clusters<2>())
    return 2;
  return 1;
}

// Level plan: segments per level while the candidate count exceeds one segment.
struct Plan {
  int levels = 0;
  int nseg[8] = {0};
  int chunk[8] = {0};
  int count[8] = {0};  // input count of the level
};

// First level: at least ceil(length / 32768) segments; more (up to one per 8k keys, so the
// merge level stays <= length / 8) when rows are too few to fill the GPU.
// With per-segment key histograms (`hist`) the first level uses the histograms' fixed
// 32768-key segments; an unsorted final selection (`wide`) of a row just past one segment
// (up to 32768 + 4096 keys) is one level of one CTA per row started from both histograms.
Plan make_plan(int batch, int length, int k, bool hist = false, bool wide = false) {
  Plan p;
  if (hist && wide && length > kTopkSegment && length <= kTopkSegment + kWideTail) {
    p.levels = 1;
    p.nseg[0] = 1;
    p.chunk[0] = length;
    p.count[0] = length;
    return p;
  }
  int count = length;
  const int nmin = (length + kTopkSegment - 1) / kTopkSegment;
  const int nmax = std::max(nmin, length / std::max(8 * k, 4096));
  int nseg = hist ? nmin : std::min(std::max(nmin, (128 + batch - 1) / batch), nmax);
  while (true) {
    const int chunk = (hist && p.levels == 0 && nseg > 1) ? kTopkSegment
                                                           : (count + nseg - 1) / nseg;
    p.nseg[p.levels] = nseg;
    p.chunk[p.levels] = chunk;
    p.count[p.levels] = count;
    ++p.levels;
    if (nseg == 1 || p.levels == 8) break;
    count = nseg * k;
    nseg = (count + kTopkSegment - 1) / kTopkSegment;
  }
  return p;
}

}  // namespace

int topk_cluster_rows(int batch, int length) {
  return length <= kTopkSegment ? cluster_size(batch, length) : 1;
}

size_t topk_workspace_bytes(int batch, int length, int k) {
  const Plan p = make_plan(batch, length, k);
  const Plan ph = make_plan(batch, length, k, true);
  if (p.levels <= 1 && ph.levels <= 1) return 0;
  // two ping-pong candidate buffers (value f32 + index i32), sized by the first level (the
  // larger of the two plans), then the next-level key histograms [batch][4096]
  const size_t cand = static_cast<size_t>(batch) * std::max(p.nseg[0], ph.nseg[0]) * k;
  return 2 * cand * 8 + 256 + static_cast<size_t>(batch) * kKeyHistBins * 4;
}

int topk_levels(int batch, int length, int k, int flags) {
  const bool hist = (flags & 1) != 0, sorted = (flags & 2) != 0;
  return make_plan(batch, length, k, hist, hist && !sorted).levels;
}

int topk_check(int length, int k, int sorted) {
  if (k < 1 || k > length) return fail(TDSA_ERR_INVALID, "top-k needs 1 <= k <= length");
  if ((sorted || length > kTopkSegment) && k > kTopkMaxSorted)
    return fail(TDSA_ERR_UNSUPPORTED, "k > 8192 is only supported unsorted on rows <= 32768");
  return TDSA_OK;
}

int launch_topk(const float* scores, int64_t s_stride, const int32_t* idx, int64_t idx_stride,
                int batch, int length, int k, int sorted, void* out_idx, int idx_bytes,
                int64_t oi_stride, float* out_val, int64_t ov_stride, void* ws, size_t ws_bytes,
                cudaStream_t stream, float* kth_out, uint32_t* key_hist, int32_t* mirror,
                int64_t mirror_stride) {
  int rc = topk_check(length, k, sorted);
  if (rc) return rc;
  // an unsorted final selection of rows just past one segment: one level (take_wide)
  const bool wide = key_hist && !idx && !sorted && !kth_out && out_idx;
  const Plan p = make_plan(batch, length, k, key_hist != nullptr, wide);
  if (p.levels > 1 && ws_bytes < topk_workspace_bytes(batch, length, k))
    return fail(TDSA_ERR_WORKSPACE, "top-k workspace too small");
  if (key_hist && !idx && !sorted && !kth_out) {
    // few rows: the cluster top-k spreads each row over several SMs -- a one-segment row
    // over 2 to 8 CTAs, a longer one (up to 131072 keys, several histogram segments) over
    // 8 CTAs in place of the levels
    const int c = p.levels == 1 ? cluster_size(batch, length)
                  : (length <= 8 * kThreads * 16 && batch <= max_active_clusters<8>()) ? 8
                                                                                      : 1;
    if (c > 1) {
      TopkArgs a = {};
      a.vals = scores;
      a.vals_stride = s_stride;
      a.row_len = length;
      a.chunk = length;
      a.k = k;
      a.out_idx = out_idx;
      a.idx_bytes = idx_bytes;
      a.out_idx_stride = oi_stride;
      a.out_val = out_val;
      a.out_val_stride = ov_stride;
      a.hist = key_hist;
      a.hist_segs = (length + kTopkSegment - 1) / kTopkSegment;
      a.mirror = mirror;
      a.mirror_stride = mirror_stride;
      const int cap = c * kThreads;
      const int per = (length + cap - 1) / cap;
      if (c == 2) return launch_cluster<2>(a, batch, per, stream);
      if (c == 4) return launch_cluster<4>(a, batch, per, stream);
      return launch_cluster<8>(a, batch, per, stream);
    }
  }
  const Plan pn = make_plan(batch, length, k);
  const size_t cand = static_cast<size_t>(batch) * std::max(p.nseg[0], pn.nseg[0]) * k;
  float* bufv[2] = {nullptr, nullptr};
  int32_t* bufi[2] = {nullptr, nullptr};
  uint32_t* lvl_hist = nullptr;  // [batch][4096]: a level's output bins for a one-segment next
  if (p.levels > 1) {
    uint8_t* base = static_cast<uint8_t*>(ws);
    bufv[0] = reinterpret_cast<float*>(base);
    bufi[0] = reinterpret_cast<int32_t*>(base + cand * 4);
    bufv[1] = reinterpret_cast<float*>(base + cand * 8);
    bufi[1] = reinterpret_cast<int32_t*>(base + cand * 12);
    lvl_hist = reinterpret_cast<uint32_t*>(base + 2 * cand * 8 + 256);
    TDSA_CUDA_CHECK(cudaMemsetAsync(lvl_hist, 0, static_cast<size_t>(batch) * kKeyHistBins * 4,
                                    stream));
  }
  uint32_t* in_hist = key_hist;
  const float* in_v = scores;
  const int32_t* in_i = idx;
  int64_t in_vs = s_stride, in_is = idx_stride;
  for (int level = 0; level < p.levels; ++level) {
    TopkArgs a = {};
    a.vals = in_v;
    a.vals_stride = in_vs;
    a.idx = in_i;
    a.idx_stride = in_is;
    a.row_len = p.count[level];
    a.chunk = p.chunk[level];
    a.k = k;
    a.kth_out = nullptr;
    a.pad_to_k = 0;
    a.hist = in_hist;
    const bool last = level == p.levels - 1;
    // the next level, when it is one segment, starts from this level's output bins
    a.next_hist = (!last && p.nseg[level + 1] == 1) ? lvl_hist : nullptr;
    in_hist = a.next_hist;
    if (last) {
      a.sorted = sorted;
      a.out_idx = out_idx;
      a.idx_bytes = idx_bytes;
      a.out_idx_stride = oi_stride;
      a.out_val = out_val;
      a.out_val_stride = ov_stride;
      a.kth_out = kth_out;
      a.mirror = mirror;
      a.mirror_stride = mirror_stride;
    } else {
      const int b = level & 1;
      a.sorted = 0;
      a.pad_to_k = 1;
      a.out_idx = bufi[b];
      a.idx_bytes = 4;
      a.out_idx_stride = k;
      a.out_val = bufv[b];
      a.out_val_stride = k;
    }
    rc = launch_segments(a, batch, p.nseg[level], stream);
    if (rc) return rc;
    if (!last) {
      const int b = level & 1;
      in_v = bufv[b];
      in_i = bufi[b];
      in_vs = static_cast<int64_t>(p.nseg[level]) * k;
      in_is = in_vs;
    }
  }
  return TDSA_OK;
}

int launch_exchange_topk(const PeerGather& g, int sorted, void* out_idx, int idx_bytes,
                         int64_t oi_stride, float* out_val, int64_t ov_stride,
                         cudaStream_t stream) {
  const int count = g.world * g.k;
  int rc = topk_check(count, g.k, sorted);
  if (rc) return rc;
  if (count > kTopkSegment)
    return fail(TDSA_ERR_UNSUPPORTED, "an exchange merges at most 32768 candidates per row");
  TopkArgs a = {};
  a.vals = reinterpret_cast<const float*>(g.own + g.scratch_v_off);
  a.vals_stride = count;
  a.idx = reinterpret_cast<const int32_t*>(g.own + g.scratch_i_off);
  a.idx_stride = count;
  a.row_len = count;
  a.chunk = count;
  a.k = g.k;
  a.sorted = sorted;
  a.out_idx = out_idx;
  a.idx_bytes = idx_bytes;
  a.out_idx_stride = oi_stride;
  a.out_val = out_val;
  a.out_val_stride = ov_stride;
  a.gather = 1;
  a.pg = g;
  return launch_segments(a, g.rows, 1, stream);
}

}  // namespace tdsa
