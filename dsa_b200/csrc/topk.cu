// Exact row-wise top-k by radix select in shared memory (no global sort).
//
// One 1024-thread CTA owns one segment of a row (<= 32768 elements, held in shared memory
// as order-preserving uint32 keys).  Up to four histogram passes over 8-bit digits (one
// private histogram per warp, lanes with equal digits combined before the atomic) pin the
// k-th key T exactly, stopping early when a digit bin is taken whole; an ordered
// compaction then takes every key > T plus the first (k - #greater) keys == T in index
// order, which is the tie rule of the reference's stable_topk (metrics.py:9-22).  The
// selection is written in ascending index order, or, when sorted output is asked for,
// bitonic-sorted in shared memory by (key descending, index ascending).
//
// Rows longer than one segment run in levels: every segment emits its local top-k in
// index order, and the candidates (global top-k is a subset of their union) are selected
// again with explicit indices until one segment remains.  The same explicit-index pass
// merges per-GPU candidates of an L-sharded cache.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 256;  // 8-bit radix digits

struct TopkArgs {
  const float* vals;      // [rows][row_stride]
  int64_t vals_stride;
  const int32_t* idx;     // explicit indices (same layout as vals) or nullptr
  int64_t idx_stride;
  int row_len;            // elements per row
  int chunk;              // segment length (gridDim.x segments per row)
  int k;
  int sorted;
  void* out_idx;          // [rows * gridDim.x][out_idx_stride]
  int idx_bytes;
  int64_t out_idx_stride;
  float* out_val;         // may be null
  int64_t out_val_stride;
  float* kth_out;         // per output row: the k-th largest value (may be null)
};

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Suffix scan over the block: returns sum of v over threads >= this thread (inclusive).
__device__ __forceinline__ uint32_t block_suffix_sum(uint32_t v, uint32_t* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += y;
  }
  if (lane == 0) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t t = wsum[lane];
    uint32_t s = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_down_sync(0xffffffffu, s, o);
      if (lane + o < 32) s += y;
    }
    wsum[32 + lane] = s - t;  // sum over warps strictly after `lane`
  }
  __syncthreads();
  const uint32_t r = x + wsum[32 + warp];
  __syncthreads();
  return r;
}

// Finds the digit bin holding the k_rem-th largest key among the histogrammed keys.
// Writes {bin, k_rem within the bin, count of the bin} to res[0..2].
__device__ void find_bin(const uint32_t* hist, int nbins, uint32_t k_rem, uint32_t* wsum,
                         uint32_t* res) {
  const int per = nbins > kThreads ? nbins / kThreads : 1;
  const int lo = threadIdx.x * per;
  uint32_t local = 0;
  if (lo < nbins)
    for (int i = 0; i < per; ++i) local += hist[lo + i];
  const uint32_t incl = block_suffix_sum(local, wsum);
  uint32_t above = incl - local;
  if (local > 0 && above < k_rem && k_rem <= incl) {
    for (int i = per - 1; i >= 0; --i) {
      const uint32_t c = hist[lo + i];
      if (above + c >= k_rem) {
        res[0] = lo + i;
        res[1] = k_rem - above;
        res[2] = c;
        break;
      }
      above += c;
    }
  }
  __syncthreads();
}

// Sums the per-warp histograms into hist[kBins].
__device__ __forceinline__ void merge_warp_hists(const uint32_t* whist, uint32_t* hist) {
  __syncthreads();
  if (threadIdx.x < kBins) {
    uint32_t s = 0;
#pragma unroll 8
    for (int w = 0; w < kWarps; ++w) s += whist[w * kBins + threadIdx.x];
    hist[threadIdx.x] = s;
  }
  __syncthreads();
}

__device__ __forceinline__ int bit_length(uint32_t x) { return x ? 32 - __clz(x) : 0; }

// Digit of key u for a pass binning [blo, bhi] with bin width 2^s: keys below / above the
// binned range clamp into the first / last bin (the mapping stays monotone).
__device__ __forceinline__ uint32_t range_digit(uint32_t u, uint32_t blo, uint32_t bhi, int s) {
  if (u < blo) return 0u;
  if (u > bhi) return kBins - 1;
  return (u - blo) >> s;
}

__device__ __forceinline__ void block_minmax(uint32_t& mn, uint32_t& mx, uint32_t* sbuf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  mn = __reduce_min_sync(0xffffffffu, mn);
  mx = __reduce_max_sync(0xffffffffu, mx);
  if (lane == 0) {
    sbuf[warp] = mn;
    sbuf[32 + warp] = mx;
  }
  __syncthreads();
  mn = __reduce_min_sync(0xffffffffu, sbuf[lane]);
  mx = __reduce_max_sync(0xffffffffu, sbuf[32 + lane]);
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) topk_segment_kernel(const TopkArgs a) {
  extern __shared__ __align__(16) uint32_t sm[];
  __shared__ uint32_t wsum[64];
  __shared__ uint32_t res[4];
  __shared__ uint32_t wcnt[2][kWarps];
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t s_kth;

  const int row = blockIdx.y, seg = blockIdx.x;
  const int start = seg * a.chunk;
  const int n = min(a.row_len - start, a.chunk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* keys = sm;
  // per-warp digit histograms; the same space holds the sort pairs after selection
  uint32_t* whist = sm + ((a.chunk + 3) & ~3);
  uint32_t* my_hist = whist + warp * kBins;
  uint64_t* pairs = reinterpret_cast<uint64_t*>(whist);

  const float* vrow = a.vals + static_cast<int64_t>(row) * a.vals_stride + start;
  const int32_t* irow = a.idx ? a.idx + static_cast<int64_t>(row) * a.idx_stride + start : nullptr;
  constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // float_to_key(-inf)
  constexpr uint32_t kNanKey = 0xFFFFFFFFu;

  // ---- load: keys to shared memory, min/max of the regular keys (not -inf, not NaN)
  uint32_t rmin = 0xFFFFFFFFu, rmax = 0u, amin = 0xFFFFFFFFu, amax = 0u;
  auto note = [&](uint32_t u) {
    amin = min(amin, u);
    amax = max(amax, u);
    if (u != kNegInfKey && u != kNanKey) {
      rmin = min(rmin, u);
      rmax = max(rmax, u);
    }
  };
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(vrow) & 15u) == 0u) {
    const float4* v4 = reinterpret_cast<const float4*>(vrow);
    uint4* k4 = reinterpret_cast<uint4*>(keys);
    const int n4 = n >> 2;
    for (int i = tid; i < n4; i += kThreads) {
      const float4 v = __ldg(v4 + i);
      const uint4 u = make_uint4(float_to_key(v.x), float_to_key(v.y), float_to_key(v.z),
                                 float_to_key(v.w));
      k4[i] = u;
      note(u.x);
      note(u.y);
      note(u.z);
      note(u.w);
    }
    done = n4 << 2;
  }
  for (int i = done + tid; i < n; i += kThreads) {
    const uint32_t u = float_to_key(__ldg(vrow + i));
    keys[i] = u;
    note(u);
  }
  for (int i = lane; i < kBins; i += 32) my_hist[i] = 0u;
  block_minmax(rmin, rmax, wsum);
  block_minmax(amin, amax, wsum);
  if (rmin > rmax) {  // no regular key: bin over everything
    rmin = amin;
    rmax = amax;
  }

  // ---- range-narrowing radix select: the k-th key lies in [clo, chi]
  const int k = min(a.k, n);
  uint32_t k_rem = static_cast<uint32_t>(k);
  uint32_t clo = 0u, chi = 0xFFFFFFFFu;
  uint32_t blo = rmin, bhi = rmax;  // pass 1 bins the regular keys, clamping the rest
  bool whole = false;
  for (int pass = 0; pass < 6 && !whole && clo != chi; ++pass) {
    const int sh = max(0, bit_length(bhi - blo) - 8);
    if (pass > 0) {
      for (int i = lane; i < kBins; i += 32) my_hist[i] = 0u;
    }
    __syncwarp();
    const uint4* k4 = reinterpret_cast<const uint4*>(keys);
    const int n4 = n >> 2;
    for (int i = tid; i < n4; i += kThreads) {
      const uint4 u = k4[i];
      const uint32_t e[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (e[j] >= clo && e[j] <= chi) atomicAdd(&my_hist[range_digit(e[j], blo, bhi, sh)], 1u);
    }
    for (int i = (n4 << 2) + tid; i < n; i += kThreads) {
      const uint32_t u = keys[i];
      if (u >= clo && u <= chi) atomicAdd(&my_hist[range_digit(u, blo, bhi, sh)], 1u);
    }
    merge_warp_hists(whist, hist);
    find_bin(hist, kBins, k_rem, wsum, res);
    const uint32_t d = res[0];
    k_rem = res[1];
    whole = (res[2] == k_rem);
    // key range of bin d (64-bit: blo + 255 * 2^sh can pass 2^32)
    const uint64_t step = 1ull << sh;
    uint64_t lo64 = d == 0 ? clo : static_cast<uint64_t>(blo) + d * step;
    uint64_t hi64 = d == kBins - 1 ? chi
                                   : min(static_cast<uint64_t>(blo) + (d + 1) * step - 1,
                                         static_cast<uint64_t>(bhi));
    if (d == kBins - 1) lo64 = min(lo64, static_cast<uint64_t>(bhi) + 1);  // + clamped-high keys
    clo = static_cast<uint32_t>(lo64);
    chi = static_cast<uint32_t>(hi64);
    blo = clo;
    bhi = chi;
  }
  __syncthreads();  // the histogram space becomes the pair buffer below
  if (tid == 0) s_kth = 0xFFFFFFFFu;
  const uint32_t need_eq = k_rem;  // keys in [clo, chi] to take, lowest index first
  // Ordered compaction.  Warp w scans positions [w*span, (w+1)*span) in 32-wide steps.
  const int span = ((n + kWarps * 32 - 1) / (kWarps * 32)) * 32;
  const int w0 = warp * span, w1 = min(n, w0 + span);
  uint32_t cgt = 0, ceq = 0;
  for (int base = w0; base < w1; base += 32) {
    const int i = base + lane;
    bool gt = false, eq = false;
    if (i < w1) {
      const uint32_t u = keys[i];
      gt = u > chi;
      eq = u >= clo && u <= chi;
    }
    cgt += __popc(__ballot_sync(0xffffffffu, gt));
    ceq += __popc(__ballot_sync(0xffffffffu, eq));
  }
  if (lane == 0) {
    wcnt[0][warp] = cgt;
    wcnt[1][warp] = ceq;
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive prefix over warps
    uint32_t g = wcnt[0][lane], e = wcnt[1][lane];
    uint32_t gs = g, es = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t yg = __shfl_up_sync(0xffffffffu, gs, o);
      const uint32_t ye = __shfl_up_sync(0xffffffffu, es, o);
      if (lane >= o) {
        gs += yg;
        es += ye;
      }
    }
    __syncwarp();
    wcnt[0][lane] = gs - g;
    wcnt[1][lane] = es - e;
  }
  __syncthreads();

  const int64_t out_row = static_cast<int64_t>(row) * gridDim.x + seg;
  uint32_t gbase = wcnt[0][warp], ebase = wcnt[1][warp];
  const unsigned lt = lanemask_lt();
  for (int base = w0; base < w1; base += 32) {
    const int i = base + lane;
    bool gt = false, eq = false;
    uint32_t u = 0;
    if (i < w1) {
      u = keys[i];
      gt = u > chi;
      eq = u >= clo && u <= chi;
    }
    const unsigned bg = __ballot_sync(0xffffffffu, gt);
    const unsigned be = __ballot_sync(0xffffffffu, eq);
    const uint32_t g_before = gbase + __popc(bg & lt);
    const uint32_t e_before = ebase + __popc(be & lt);
    bool take = false;
    uint32_t pos = 0;
    if (gt) {
      take = true;
      pos = g_before + min(e_before, need_eq);
    } else if (eq && e_before < need_eq) {
      take = true;
      pos = g_before + e_before;
    }
    if (take) {
      const uint32_t gi = irow ? static_cast<uint32_t>(irow[i]) : static_cast<uint32_t>(start + i);
      if (eq) atomicMin(&s_kth, u);
      if (a.sorted) {
        pairs[pos] = (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - gi);
      } else if (a.out_idx) {
        if (a.idx_bytes == 8)
          static_cast<int64_t*>(a.out_idx)[out_row * a.out_idx_stride + pos] = static_cast<int64_t>(gi);
        else
          static_cast<int32_t*>(a.out_idx)[out_row * a.out_idx_stride + pos] = static_cast<int32_t>(gi);
        if (a.out_val) a.out_val[out_row * a.out_val_stride + pos] = key_to_float(u);
      }
    }
    gbase += __popc(bg);
    ebase += __popc(be);
  }
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
    if (a.idx_bytes == 8)
      static_cast<int64_t*>(a.out_idx)[out_row * a.out_idx_stride + j] = static_cast<int64_t>(gi);
    else
      static_cast<int32_t*>(a.out_idx)[out_row * a.out_idx_stride + j] = static_cast<int32_t>(gi);
    if (a.out_val) a.out_val[out_row * a.out_val_stride + j] = key_to_float(static_cast<uint32_t>(p >> 32));
  }
}

int kpow2(int k) {
  int p = 1;
  while (p < k) p <<= 1;
  return p;
}

size_t segment_smem(int chunk, int k, int sorted) {
  const size_t hists = static_cast<size_t>(kWarps) * kBins * 4;
  const size_t pairs = sorted ? static_cast<size_t>(kpow2(k)) * 8 : 0;
  return static_cast<size_t>((chunk + 3) & ~3) * 4 + (hists > pairs ? hists : pairs);
}

int launch_segments(const TopkArgs& a, int rows, int nseg, cudaStream_t stream) {
  const size_t smem = segment_smem(a.chunk, a.k, a.sorted);
  TDSA_CUDA_CHECK(cudaFuncSetAttribute(topk_segment_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
  topk_segment_kernel<<<dim3(nseg, rows), kThreads, smem, stream>>>(a);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

// Level plan: segments per level while the candidate count exceeds one segment.
struct Plan {
  int levels = 0;
  int nseg[8] = {0};
  int chunk[8] = {0};
  int count[8] = {0};  // input count of the level
};

Plan make_plan(int length, int k) {
  Plan p;
  int count = length;
  while (true) {
    const int nseg = (count + kTopkSegment - 1) / kTopkSegment;
    const int chunk = (count + nseg - 1) / nseg;
    p.nseg[p.levels] = nseg;
    p.chunk[p.levels] = chunk;
    p.count[p.levels] = count;
    ++p.levels;
    if (nseg == 1 || p.levels == 8) break;
    count = nseg * k;
  }
  return p;
}

}  // namespace

size_t topk_workspace_bytes(int batch, int length, int k) {
  const Plan p = make_plan(length, k);
  if (p.levels <= 1) return 0;
  // two ping-pong candidate buffers (value f32 + index i32), sized by the first level
  const size_t cand = static_cast<size_t>(batch) * p.nseg[0] * k;
  return 2 * cand * 8 + 256;
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
                cudaStream_t stream, float* kth_out) {
  int rc = topk_check(length, k, sorted);
  if (rc) return rc;
  const Plan p = make_plan(length, k);
  if (p.levels > 1 && ws_bytes < topk_workspace_bytes(batch, length, k))
    return fail(TDSA_ERR_WORKSPACE, "top-k workspace too small");
  const size_t cand = static_cast<size_t>(batch) * p.nseg[0] * k;
  float* bufv[2] = {nullptr, nullptr};
  int32_t* bufi[2] = {nullptr, nullptr};
  if (p.levels > 1) {
    uint8_t* base = static_cast<uint8_t*>(ws);
    bufv[0] = reinterpret_cast<float*>(base);
    bufi[0] = reinterpret_cast<int32_t*>(base + cand * 4);
    bufv[1] = reinterpret_cast<float*>(base + cand * 8);
    bufi[1] = reinterpret_cast<int32_t*>(base + cand * 12);
  }
  const float* in_v = scores;
  const int32_t* in_i = idx;
  int64_t in_vs = s_stride, in_is = idx_stride;
  for (int level = 0; level < p.levels; ++level) {
    TopkArgs a;
    a.vals = in_v;
    a.vals_stride = in_vs;
    a.idx = in_i;
    a.idx_stride = in_is;
    a.row_len = p.count[level];
    a.chunk = p.chunk[level];
    a.k = k;
    a.kth_out = nullptr;
    const bool last = level == p.levels - 1;
    if (last) {
      a.sorted = sorted;
      a.out_idx = out_idx;
      a.idx_bytes = idx_bytes;
      a.out_idx_stride = oi_stride;
      a.out_val = out_val;
      a.out_val_stride = ov_stride;
      a.kth_out = kth_out;
    } else {
      const int b = level & 1;
      a.sorted = 0;
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

}  // namespace tdsa
