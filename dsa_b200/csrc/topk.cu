// Exact row-wise top-k by radix select, keys held in registers (no global sort).
//
// One 1024-thread CTA owns one segment of a row (<= 32768 elements).  Thread t holds the
// 32 consecutive elements [32t, 32t+32) as order-preserving uint32 keys in registers.
// Range-narrowing radix passes (256 bins over the live key range, one private histogram
// per warp in shared memory) pin the k-th key T; every key > T is taken and keys == T are
// taken lowest index first, which is the tie rule of the reference's stable_topk
// (metrics.py:9-22).  Because each thread owns a contiguous run, two block-wide scans give
// every taken key its output position in ascending index order; sorted output is a bitonic
// sort of the k taken (key, index) pairs in shared memory.
//
// Rows longer than one segment run in levels: every segment emits its local top-k in index
// order, and the candidates (the global top-k is a subset of their union) are selected
// again with explicit indices until one segment remains.  The same explicit-index pass
// merges per-GPU candidates of an L-sharded cache.
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kPer = kTopkSegment / kThreads;  // 32 keys per thread
constexpr int kBins = 256;

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
};

// Inclusive block-wide prefix sum of v (thread order), with the block total.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* wsum, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const uint32_t t = wsum[lane];
    uint32_t s = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    wsum[32 + lane] = s - t;  // exclusive prefix over warps
    if (lane == 31) wsum[64] = s;
  }
  __syncthreads();
  const uint32_t r = x + wsum[32 + warp];
  total = wsum[64];
  __syncthreads();
  return r;
}

// The bin (of kBins) holding the k_rem-th largest counted key: res = {bin, k_rem within the
// bin, count of the bin}.  Threads 0..255 each own one bin; suffix sums via a reversed scan.
__device__ void find_bin(const uint32_t* hist, uint32_t k_rem, uint32_t* wsum, uint32_t* res) {
  // thread t takes bin (kBins-1-t) so the inclusive prefix over threads is a suffix over bins
  const int t = threadIdx.x;
  const uint32_t c = t < kBins ? hist[kBins - 1 - t] : 0u;
  uint32_t total;
  const uint32_t incl = block_scan(c, wsum, total);
  if (t < kBins && c > 0 && incl - c < k_rem && k_rem <= incl) {
    res[0] = kBins - 1 - t;
    res[1] = k_rem - (incl - c);
    res[2] = c;
  }
  __syncthreads();
}

__device__ __forceinline__ int bit_length(uint32_t x) { return x ? 32 - __clz(x) : 0; }

__global__ void __launch_bounds__(kThreads, 1) topk_segment_kernel(const TopkArgs a) {
  extern __shared__ __align__(16) uint32_t sm[];
  __shared__ uint32_t wsum[72];
  __shared__ uint32_t res[4];
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t s_kth;

  const int row = blockIdx.y, seg = blockIdx.x;
  const int start = seg * a.chunk;
  const int n = min(a.row_len - start, a.chunk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* my_hist = sm + warp * kBins;  // per-warp histograms (32 KiB) ...
  uint64_t* pairs = reinterpret_cast<uint64_t*>(sm);  // ... later the sort buffer

  const float* vrow = a.vals + static_cast<int64_t>(row) * a.vals_stride + start;
  const int32_t* irow = a.idx ? a.idx + static_cast<int64_t>(row) * a.idx_stride + start : nullptr;
  const int e0 = tid * kPer;  // first element of this thread
  const int cnt = max(0, min(kPer, n - e0));

  // ---- keys to registers; key 0 (below every real key) pads past the end
  uint32_t key[kPer];
  if (cnt == kPer && (reinterpret_cast<uintptr_t>(vrow + e0) & 15u) == 0u) {
    const float4* v4 = reinterpret_cast<const float4*>(vrow + e0);
#pragma unroll
    for (int j = 0; j < kPer / 4; ++j) {
      const float4 v = __ldg(v4 + j);
      key[4 * j + 0] = float_to_key(v.x);
      key[4 * j + 1] = float_to_key(v.y);
      key[4 * j + 2] = float_to_key(v.z);
      key[4 * j + 3] = float_to_key(v.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kPer; ++j) key[j] = j < cnt ? float_to_key(__ldg(vrow + e0 + j)) : 0u;
  }
  // live key range: min over real keys, max
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (j < cnt) {
      kmin = min(kmin, key[j]);
      kmax = max(kmax, key[j]);
    }
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  if (lane == 0) {
    wsum[warp] = kmin;
    wsum[32 + warp] = kmax;
  }
  for (int i = lane; i < kBins; i += 32) my_hist[i] = 0u;
  __syncthreads();
  kmin = __reduce_min_sync(0xffffffffu, wsum[lane]);
  kmax = __reduce_max_sync(0xffffffffu, wsum[32 + lane]);
  __syncthreads();

  // ---- range-narrowing radix select: the k-th key lies in [clo, chi]
  const int k = min(a.k, n);
  uint32_t k_rem = static_cast<uint32_t>(k);
  uint32_t clo = kmin, chi = kmax;
  bool whole = false;
  for (int pass = 0; pass < 5 && !whole && clo != chi; ++pass) {
    const int sh = max(0, bit_length(chi - clo) - 8);
    if (pass > 0) {
      for (int i = lane; i < kBins; i += 32) my_hist[i] = 0u;
      __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const uint32_t u = key[j];
      if (j < cnt && u >= clo && u <= chi) atomicAdd(&my_hist[(u - clo) >> sh], 1u);
    }
    __syncthreads();
    if (tid < kBins) {
      uint32_t s = 0;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) s += sm[w * kBins + tid];
      hist[tid] = s;
    }
    __syncthreads();
    find_bin(hist, k_rem, wsum, res);
    const uint32_t d = res[0];
    k_rem = res[1];
    whole = (res[2] == k_rem);
    const uint64_t lo64 = static_cast<uint64_t>(clo) + (static_cast<uint64_t>(d) << sh);
    const uint64_t top = lo64 + (1ull << sh) - 1;
    const uint64_t hi64 = top < chi ? top : static_cast<uint64_t>(chi);
    clo = static_cast<uint32_t>(lo64);
    chi = static_cast<uint32_t>(hi64);
  }
  const uint32_t need_eq = k_rem;  // keys in [clo, chi] to take, lowest index first

  // ---- ordered output: positions from two block scans over per-thread counts
  uint32_t ngt = 0, neq = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t u = key[j];
    ngt += (j < cnt && u > chi) ? 1u : 0u;
    neq += (j < cnt && u >= clo && u <= chi) ? 1u : 0u;
  }
  uint32_t tot;
  const uint32_t eq_before = block_scan(neq, wsum, tot) - neq;
  const uint32_t eq_take = eq_before >= need_eq ? 0u : min(neq, need_eq - eq_before);
  const uint32_t sel = ngt + eq_take;
  const uint32_t sel_before = block_scan(sel, wsum, tot) - sel;
  if (tid == 0) s_kth = 0xFFFFFFFFu;
  __syncthreads();  // the histograms are dead from here on (pairs may reuse the space)

  const int64_t out_row = static_cast<int64_t>(row) * gridDim.x + seg;
  uint32_t pos = sel_before, eq_seen = 0, kth_local = 0xFFFFFFFFu;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const uint32_t u = key[j];
    bool take = false;
    if (j < cnt) {
      if (u > chi) {
        take = true;
      } else if (u >= clo) {
        take = eq_seen < eq_take;
        ++eq_seen;
        if (take) kth_local = min(kth_local, u);
      }
    }
    if (take) {
      const int e = e0 + j;
      const uint32_t gi = irow ? static_cast<uint32_t>(irow[e]) : static_cast<uint32_t>(start + e);
      if (a.sorted) {
        pairs[pos] = (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - gi);
      } else if (a.out_idx) {
        if (a.idx_bytes == 8)
          static_cast<int64_t*>(a.out_idx)[out_row * a.out_idx_stride + pos] = static_cast<int64_t>(gi);
        else
          static_cast<int32_t*>(a.out_idx)[out_row * a.out_idx_stride + pos] = static_cast<int32_t>(gi);
        if (a.out_val) a.out_val[out_row * a.out_val_stride + pos] = key_to_float(u);
      }
      ++pos;
    }
  }
  if (eq_take) atomicMin(&s_kth, kth_local);
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
  (void)chunk;
  const size_t hists = static_cast<size_t>(kWarps) * kBins * 4;
  const size_t pairs = sorted ? static_cast<size_t>(kpow2(k)) * 8 : 0;
  return hists > pairs ? hists : pairs;
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
