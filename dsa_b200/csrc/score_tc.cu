// Dense Lightning-Indexer scoring on the sm_100a tensor cores.
//
//   score[b][s] = sum_h w[b][h] * ReLU(q[b][h] . k[b][s]),   H = 64, D = 128
//
// One persistent CTA per SM walks a contiguous range of 128-key tiles (tiles of all
// sequences are numbered b * tiles_per_seq + t).  Warp roles:
//   warp 0      TMA producer: key tiles [128 keys x 128 dims] into a 4-stage smem ring
//               (two 64-column boxes, 128-byte swizzle); the sequence's q [64 x 128] into
//               one of two q slots when the sequence changes.
//   warp 1      tcgen05 issuer: UMMA M=128 (keys) x N=64 (heads) x K=128 (8 x K16 steps),
//               A = key tile, B = q, accumulator in TMEM (4 buffers x 64 f32 columns).
//   warps 2..9  epilogue, two groups of four warps taking alternate tiles (one warp alone
//               per TMEM lane quadrant does not keep up with the key stream): each thread
//               owns one key (one TMEM lane), loads its 64 head dots with tcgen05.ld,
//               applies ReLU * w_h and sums the heads in registers -- no cross-thread
//               reduction -- and stores one float per key (coalesced), plus optionally its
//               float16 rounding into a score-trace row.
// HBM traffic per key = its 256 bytes, read once; q/w per sequence come from L2.
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "score_epilogue.cuh"
#include "timeline.cuh"

namespace tdsa {

// (outside the unnamed namespace: the timeline readers keep external C linkage)
// timeline builds: per CTA (thread 0, the TMA producer) entry, past the dependency wait,
// last key tile issued, exit
TDSA_TL_DECL(score, 148, 4)

namespace {

constexpr int kTileKeys = 128;
constexpr int kStages = 4;
constexpr int kQSlots = 2;  // q buffers: the next sequence's q loads while the MMA uses one
constexpr int kStageBytes = kTileKeys * kHeadDim * 2;  // 32 KiB
constexpr int kHalfBytes = kStageBytes / 2;            // 128 rows x 128 B
constexpr int kQBytes = kHeads * kHeadDim * 2;         // 16 KiB
constexpr int kQHalf = kQBytes / 2;                    // 64 rows x 128 B
constexpr int kEpiGroups = 2;  // epilogue groups of four warps, alternate tiles
constexpr int kAccBufs = 4;    // TMEM accumulators: two per epilogue group
constexpr int kTmemCols = kAccBufs * kHeads;
constexpr int kThreads = 64 + 128 * kEpiGroups;
constexpr int kBarrierBytes = 1024;
constexpr int kSmemBytes = kStages * kStageBytes + kQSlots * kQBytes + kBarrierBytes + 1024;
constexpr int kHistBins = 4096;  // key histogram bins (top 12 bits of the order-preserving key)
constexpr int kHistBytes = kHistBins * 4 * kEpiGroups;  // one histogram per epilogue group
constexpr int kHistSegment = 32768;  // keys per histogram (one top-k segment)
static_assert(kHistSegment == 256 * kTileKeys, "a segment is 256 tiles");

struct DenseArgs {
  const float* w;
  int64_t w_stride;
  float* out;
  int64_t out_stride;
  int length;
  int tiles_per_seq;
  int64_t total_tiles;
  uint32_t* hist;  // [batch][hist_segs][4096] key histograms (kHist kernels), one per
                   // 32768-key segment of a row: counts are added
  int hist_segs;
  __half* trace;   // optional float16 copy of the scores (score trace rows), or null
  int64_t trace_stride;
  int* status;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// kHist: the epilogue also counts every score's order-preserving key by its top 12 bits in a
// shared-memory histogram (one per epilogue group), flushed to a.hist[sequence][segment]
// whenever the group moves to the next sequence or 32768-key segment (the top-k then starts
// each segment from the bin holding its k-th key instead of a full pass).
template <bool kBF16, bool kHist>
__global__ void __launch_bounds__(kThreads, 1)
    score_dense_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap qmap, const DenseArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* stage_base = smem;
  uint8_t* q_base = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(q_base + kQSlots * kQBytes);
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* accfull = qempty + 2;
  uint64_t* accempty = accfull + kAccBufs;
  uint64_t* done = accempty + kAccBufs;
  uint64_t* hbar = done + 1;  // [kEpiGroups] epilogue-group handshakes around histogram flushes
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(hbar + kEpiGroups);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint32_t* shist = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + kBarrierBytes);
  unsigned int tl_launch = 0;
  if (threadIdx.x == 0) {
    tl_launch = TDSA_TL_TICKET(score);
    TDSA_TL_REC(score, 148, 4, tl_launch, blockIdx.x, 0);
  }

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
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], 1);
    }
    for (int s = 0; s < kAccBufs; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);  // the four warps of the group that owns the buffer
    }
    mbar_init(done, 1);
    for (int g = 0; g < kEpiGroups; ++g) mbar_init(&hbar[g], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (kHist)
    for (int i = threadIdx.x; i < kHistBins * kEpiGroups; i += kThreads) shist[i] = 0u;
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
  pdl_wait();  // q, w and the histogram may come from the previous kernel
  if (threadIdx.x == 0) TDSA_TL_REC(score, 148, 4, tl_launch, blockIdx.x, 1);
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
          uint8_t* qd = q_base + slot * kQBytes;
          tma_load_3d(qd, &qmap, &qfull[slot], 0, 0, b, pol_q);
          tma_load_3d(qd + kQHalf, &qmap, &qfull[slot], 64, 0, b, pol_q);
          ++qcount;
          prev_b = b;
        }
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        uint8_t* dst = stage_base + s * kStageBytes;
        tma_load_3d(dst, &kmap, &full[s], 0, tt * kTileKeys, b, pol_k);
        tma_load_3d(dst + kHalfBytes, &kmap, &full[s], 64, tt * kTileKeys, b, pol_k);
        ++it;
      }
      TDSA_TL_REC(score, 148, 4, tl_launch, blockIdx.x, 2);
      // Let every issued copy land before the CTA can exit (bounded, abort or not).
      volatile int no_abort = 0;
      for (uint32_t s = 0; s < kStages && s < it; ++s) {
        const uint32_t n = (it - s + kStages - 1) / kStages;  // loads issued into stage s
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
      constexpr uint32_t idesc = umma_idesc_f16(kBF16, 128, kHeads);
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
        const uint32_t acc = acc_it % kAccBufs, aph = (acc_it / kAccBufs) & 1u;
        if (!mbar_wait(&accempty[acc], aph ^ 1u, abort_flag)) break;
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(stage_base + s * kStageBytes);
        const uint32_t b_addr = smem_u32(q_base + slot * kQBytes);
        const uint32_t d_tmem = tmem_base + acc * kHeads;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k) {
          const uint64_t ad = sw128_kmajor_desc(a_addr + (k >> 2) * kHalfBytes + (k & 3) * 32);
          const uint64_t bd = sw128_kmajor_desc(b_addr + (k >> 2) * kQHalf + (k & 3) * 32);
          umma_f16(d_tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&accfull[acc]);
        ++it;
        ++acc_it;
      }
      // All MMAs must be complete before TMEM is released.
      umma_commit(done);
      volatile int no_abort = 0;
      mbar_wait(done, 0, &no_abort);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    // group g (warps 2 + 4g .. 5 + 4g, one per TMEM lane quadrant) takes the CTA's local
    // tiles i = g, g + 2, ... from accumulator i % 4
    const uint32_t quad = static_cast<uint32_t>(warp & 3);
    const int group = (warp - 2) >> 2;
    const int etid = (warp - 2 - 4 * group) * 32 + lane;  // 0..127 within the group
    uint32_t* ghist = shist + group * kHistBins;
    uint64_t* gbar = hbar + group;
    int prev_b = -1, prev_slot = -1;
    uint32_t hph = 0;
    float wr[kHeads];
    // the group's four warps meet (bounded wait); false when the CTA aborts
    auto hist_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(gbar);
      const bool ok = mbar_wait(gbar, hph & 1u, abort_flag);
      ++hph;
      return ok;
    };
    auto hist_flush = [&](int slot) -> bool {
      if (!hist_sync()) return false;
      uint32_t* dst = a.hist + static_cast<int64_t>(slot) * kHistBins;
      for (int i = etid; i < kHistBins; i += 128) {
        const uint32_t c = ghist[i];
        if (c) {
          atomicAdd(dst + i, c);
          ghist[i] = 0u;
        }
      }
      return hist_sync();
    };
    bool ok = true;
    for (int64_t t = t0 + group; t < t1; t += kEpiGroups) {
      const uint32_t acc_it = static_cast<uint32_t>(t - t0);
      const int b = static_cast<int>(t / tps);
      const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tps);
      if (kHist) {  // one histogram per (sequence, 32768-key segment): 256 tiles
        const int slot = b * a.hist_segs + (tt >> 8);
        if (slot != prev_slot) {
          if (prev_slot >= 0 && !hist_flush(prev_slot)) {
            ok = false;
            break;
          }
          prev_slot = slot;
        }
      }
      if (b != prev_b) {
        load_head_weights(a.w + static_cast<int64_t>(b) * a.w_stride, wr);
        prev_b = b;
      }
      const uint32_t acc = acc_it % kAccBufs, aph = (acc_it / kAccBufs) & 1u;
      if (!mbar_wait(&accfull[acc], aph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + acc * kHeads;
      tmem_ld32(taddr, r0);
      tmem_ld32(taddr + 32, r1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[acc]);
      const float score = relu_weighted_sum(r0, r1, wr);
      const int row = tt * kTileKeys + static_cast<int>(quad) * 32 + lane;
      if (row < a.length) {
        a.out[static_cast<int64_t>(b) * a.out_stride + row] = score;
        // round to nearest even, as numpy's float32 -> float16 cast of the trace writer
        if (a.trace)
          a.trace[static_cast<int64_t>(b) * a.trace_stride + row] = __float2half_rn(score);
      }
      if (kHist) add_to_bin(ghist, row < a.length, float_to_key(score) >> 20);
    }
    if (kHist && ok && prev_slot >= 0) hist_flush(prev_slot);
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
  if (threadIdx.x == 0) TDSA_TL_REC(score, 148, 4, tl_launch, blockIdx.x, 3);
}

template <bool kBF16>
int launch_dense_tc_t(const void* q, int64_t q_bs, const float* w, int64_t w_bs, const void* k,
                      int64_t k_bs, int64_t k_rs, int batch, int length, float* out,
                      int64_t o_bs, cudaStream_t stream, int* status, uint32_t* hist,
                      void* trace, int64_t trace_bs) {
  const CUtensorMapDataType dt =
      kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap kmap, qmap;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(length),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(k_bs) * 2
                                       : static_cast<uint64_t>(k_rs) * 2 * length;
    const uint64_t strides[2] = {static_cast<uint64_t>(k_rs) * 2, bstride};
    const uint32_t box[3] = {64, kTileKeys, 1};
    int rc = encode_tmap(&kmap, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(kHeads),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(q_bs) * 2
                                       : static_cast<uint64_t>(kHeads * kHeadDim * 2);
    const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim) * 2, bstride};
    const uint32_t box[3] = {64, kHeads, 1};
    int rc = encode_tmap(&qmap, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  DenseArgs a;
  a.w = w;
  a.w_stride = w_bs;
  a.out = out;
  a.out_stride = o_bs;
  a.length = length;
  a.tiles_per_seq = (length + kTileKeys - 1) / kTileKeys;
  a.total_tiles = static_cast<int64_t>(a.tiles_per_seq) * batch;
  a.status = status;
  a.hist = hist;
  a.hist_segs = (length + kHistSegment - 1) / kHistSegment;
  a.trace = static_cast<__half*>(trace);
  a.trace_stride = trace_bs;
  const int dev = current_device();
  const int sms = device_sm_count(dev);
  const int64_t grid = a.total_tiles < sms ? a.total_tiles : sms;
  const int smem = kSmemBytes + (hist ? kHistBytes : 0);
  auto kern = hist ? score_dense_tc_kernel<kBF16, true> : score_dense_tc_kernel<kBF16, false>;
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  TDSA_CUDA_CHECK(launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem,
                             stream, kmap, qmap, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace

int launch_score_dense_tc(const void* q, int64_t q_bs, const float* w, int64_t w_bs,
                          const void* k, int64_t k_bs, int64_t k_rs, int dtype, int batch,
                          int length, float* out, int64_t o_bs, cudaStream_t stream,
                          int* status, uint32_t* hist, void* trace, int64_t trace_bs) {
  if (dtype == TDSA_BF16)
    return launch_dense_tc_t<true>(q, q_bs, w, w_bs, k, k_bs, k_rs, batch, length, out, o_bs,
                                   stream, status, hist, trace, trace_bs);
  return launch_dense_tc_t<false>(q, q_bs, w, w_bs, k, k_bs, k_rs, batch, length, out, o_bs,
                                  stream, status, hist, trace, trace_bs);
}

}  // namespace tdsa
