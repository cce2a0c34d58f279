// Block-structured indexer scoring on the sm_100a tensor cores.
//
// A 128-key MMA tile is assembled from 128/bs key blocks (bs = 16, 32, 64, 128) of one
// sequence; each block is its own TMA box, and a block whose keys are not needed is never
// loaded.  The pipeline is the dense kernel's (TMA producer warp, tcgen05 issuer warp, two
// epilogue groups of four warps taking alternate tiles, each thread owning one key, four
// TMEM accumulators); the epilogue differs by mode:
//
//   kModeH8           8-head probe score on cold blocks, -inf elsewhere, per-block max
//                     (reference _h8_block_max_kernel, progressive_kernel.py:218-246)
//   kModeMasked       dense score on kept blocks, -inf elsewhere; dropped blocks unread
//                     (reference _masked_full_kernel, :249-274)
//   kModeProgressive  direct blocks: all 64 heads; cold blocks: 8-head probe, promotion
//                     when its block max >= threshold, then + the other 56 heads
//                     (reference _progressive_kernel, :277-346)
//   kModeExact        waves of the exact progressive path: dense score of the listed
//                     blocks (bit-identical to the dense kernel) and their exact block max
//
// Block maxima reduce per 16-row group in registers, then across the epilogue warps through
// shared memory, synchronised by an mbarrier (bounded wait) per TMEM buffer.
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"
#include "score_epilogue.cuh"

namespace tdsa {

namespace {

constexpr int kTileKeys = 128;
constexpr int kStages = 4;
constexpr int kStageBytes = kTileKeys * kHeadDim * 2;
constexpr int kHalfBytes = kStageBytes / 2;
constexpr int kQBytes = kHeads * kHeadDim * 2;
constexpr int kQHalf = kQBytes / 2;
constexpr int kEpiGroups = 2;  // epilogue groups of four warps, alternate tiles
constexpr int kAccBufs = 4;    // TMEM accumulators: two per epilogue group
constexpr int kTmemCols = kAccBufs * kHeads;
constexpr int kThreads = 64 + 128 * kEpiGroups;
constexpr int kBarrierBytes = 1024;
constexpr int kSmemBytes = kStages * kStageBytes + 2 * kQBytes + kBarrierBytes + 1024;
constexpr int kHistSmemBytes = kKeyHistBins * 4 * kEpiGroups;  // exact mode: one per group
constexpr int kMaxSlots = 8;  // blocks per tile at bs = 16
static_assert(kTopkSegment == 1 << 15, "a key's histogram segment is its index >> 15");

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

struct Tile {
  int seq;
  int nslots;
  int block[kMaxSlots];  // -1: empty slot
};

// Tile t of the launch: contiguous (tile_blocks == nullptr) or from the exact-path list.
__device__ __forceinline__ void get_tile(const BlockArgs& a, int64_t t, Tile& tile) {
  tile.nslots = a.bpt;
  if (a.tile_blocks == nullptr) {
    tile.seq = static_cast<int>(t / a.tiles_per_seq);
    const int first = static_cast<int>(t - static_cast<int64_t>(tile.seq) * a.tiles_per_seq) * a.bpt;
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j)
      tile.block[j] = (j < a.bpt && first + j < a.nblocks) ? first + j : -1;
  } else {
    tile.seq = a.tile_seq[t];
#pragma unroll
    for (int j = 0; j < kMaxSlots; ++j)
      tile.block[j] = j < a.bpt ? a.tile_blocks[t * a.bpt + j] : -1;
  }
}

// The launch's per-block mask: cold (H8, or direct blocks inverted), keep (masked; with
// `accept_max`, the second half of the two-pass path: kept when direct or when the block's
// probe maximum reaches the threshold), direct (progressive).
template <int kMode>
__device__ __forceinline__ bool mask_set(const BlockArgs& a, int seq, int blk) {
  const bool m = a.mask[static_cast<int64_t>(seq) * a.mask_stride + blk] != 0;
  if (kMode == kModeMasked && a.accept_max != nullptr)
    return m || a.accept_max[static_cast<int64_t>(seq) * a.bm_stride + blk] >= *a.threshold;
  return m != (a.mask_invert != 0);
}

template <int kMode>
__device__ __forceinline__ bool block_loaded(const BlockArgs& a, int seq, int blk) {
  if (blk < 0) return false;
  if (kMode == kModeH8 || kMode == kModeMasked) return mask_set<kMode>(a, seq, blk);
  return true;
}

// ReLU-weighted sums over the heads in `mask` and over the others, ascending head order.
__device__ __forceinline__ void split_head_sums(const uint32_t (&lo)[32], const uint32_t (&hi)[32],
                                                const float (&wr)[64], uint64_t mask, float& sel,
                                                float& rest) {
  float s0 = 0.f, s1 = 0.f, r0 = 0.f, r1 = 0.f;
#pragma unroll
  for (int h = 0; h < 64; ++h) {
    const float d = fmaxf(__uint_as_float(h < 32 ? lo[h] : hi[h - 32]), 0.f);
    const bool in = (mask >> h) & 1ull;
    if (h & 1) {
      s1 = fmaf(in ? wr[h] : 0.f, d, s1);
      r1 = fmaf(in ? 0.f : wr[h], d, r1);
    } else {
      s0 = fmaf(in ? wr[h] : 0.f, d, s0);
      r0 = fmaf(in ? 0.f : wr[h], d, r0);
    }
  }
  sel = s0 + s1;
  rest = r0 + r1;
}

__device__ __forceinline__ uint64_t head_mask(const int32_t* ids, int n) {
  uint64_t m = 0;
  for (int i = 0; i < n; ++i) {
    const int h = ids[i];
    if (h >= 0 && h < 64) m |= 1ull << h;
  }
  return m;
}

// kmap loads one block (bs rows); kmap_tile loads 128 rows, used for a tile whose blocks are
// consecutive and all needed (two large boxes instead of 2 * bpt small ones).
template <int kMode, bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    score_blocks_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap kmap_tile,
                        const __grid_constant__ CUtensorMap qmap, const BlockArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* stage_base = smem;
  uint8_t* q_base = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(q_base + 2 * kQBytes);
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* accfull = qempty + 2;
  uint64_t* accempty = accfull + kAccBufs;
  uint64_t* grp = accempty + kAccBufs;  // epilogue group-max exchange, one per TMEM buffer
  uint64_t* done = grp + kAccBufs;
  uint64_t* hbar = done + 1;  // [kEpiGroups] epilogue-group handshakes around histogram flushes
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(hbar + kEpiGroups);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* gmax = reinterpret_cast<float*>(tmem_holder + 4);  // [kAccBufs][8]
  // exact mode with a histogram: 4096 bins per epilogue group behind the barrier region
  uint32_t* shist = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + kBarrierBytes);
  const bool use_hist = kMode == kModeExact && a.hist != nullptr;
  if (use_hist)
    for (int i = threadIdx.x; i < kKeyHistBins * kEpiGroups; i += kThreads) shist[i] = 0u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bs = a.bs;
  const uint32_t box_bytes = static_cast<uint32_t>(bs) * 128u;  // one half (64 dims)

  // prologue (touches no memory the previous kernel writes): barriers, tensor maps, TMEM --
  // under programmatic dependent launch it overlaps the previous kernel's tail
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
      mbar_init(&accempty[s], 4);
      mbar_init(&grp[s], 4);
    }
    mbar_init(done, 1);
    for (int g = 0; g < kEpiGroups; ++g) mbar_init(&hbar[g], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&kmap_tile);
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
  pdl_wait();  // the tile count, tile lists, q, w and masks may come from the previous kernel
  pdl_launch_dependents();
  const int64_t total = a.tile_count ? static_cast<int64_t>(*a.tile_count) : a.total_tiles;
  const int64_t t0 = total * blockIdx.x / gridDim.x;
  const int64_t t1 = total * (blockIdx.x + 1) / gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      const uint64_t pol_k = policy_evict_first();
      const uint64_t pol_q = policy_evict_last();
      int prev_seq = -1;
      uint32_t qcount = 0, it = 0;
      Tile tile;
      for (int64_t t = t0; t < t1; ++t) {
        get_tile(a, t, tile);
        if (tile.seq != prev_seq) {
          const uint32_t slot = qcount & 1u, ph = (qcount >> 1) & 1u;
          if (!mbar_wait(&qempty[slot], ph ^ 1u, abort_flag)) break;
          mbar_arrive_expect_tx(&qfull[slot], kQBytes);
          uint8_t* qd = q_base + slot * kQBytes;
          tma_load_3d(qd, &qmap, &qfull[slot], 0, 0, tile.seq, pol_q);
          tma_load_3d(qd + kQHalf, &qmap, &qfull[slot], 64, 0, tile.seq, pol_q);
          ++qcount;
          prev_seq = tile.seq;
        }
        const uint32_t s = it % kStages, ph = (it / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) break;
        uint32_t nload = 0;
        bool consecutive = a.bpt > 1;
        for (int j = 0; j < a.bpt; ++j) {
          const bool ld = block_loaded<kMode>(a, tile.seq, tile.block[j]);
          nload += ld;
          consecutive = consecutive && ld && tile.block[j] == tile.block[0] + j;
        }
        uint8_t* dst = stage_base + s * kStageBytes;
        if (consecutive) {  // the tile is 128 consecutive keys: two large boxes
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          const int row0 = tile.block[0] * bs;
          tma_load_3d(dst, &kmap_tile, &full[s], 0, row0, tile.seq, pol_k);
          tma_load_3d(dst + kHalfBytes, &kmap_tile, &full[s], 64, row0, tile.seq, pol_k);
        } else {
          mbar_arrive_expect_tx(&full[s], nload * box_bytes * 2u);
          for (int j = 0; j < a.bpt; ++j) {
            const int blk = tile.block[j];
            if (!block_loaded<kMode>(a, tile.seq, blk)) continue;
            tma_load_3d(dst + j * box_bytes, &kmap, &full[s], 0, blk * bs, tile.seq, pol_k);
            tma_load_3d(dst + kHalfBytes + j * box_bytes, &kmap, &full[s], 64, blk * bs,
                        tile.seq, pol_k);
          }
        }
        ++it;
      }
      volatile int no_abort = 0;
      for (uint32_t s = 0; s < kStages && s < it; ++s) {
        const uint32_t n = (it - s + kStages - 1) / kStages;
        mbar_wait(&full[s], (n - 1) & 1u, &no_abort);
      }
      for (uint32_t s = 0; s < 2 && s < qcount; ++s) {
        const uint32_t n = (qcount - s + 1) / 2;
        mbar_wait(&qfull[s], (n - 1) & 1u, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ UMMA issuer
      constexpr uint32_t idesc = umma_idesc_f16(kBF16, 128, kHeads);
      int prev_seq = -1;
      uint32_t qcount = 0, it = 0, acc_it = 0, slot = 0;
      for (int64_t t = t0; t < t1; ++t) {
        const int seq = a.tile_blocks ? a.tile_seq[t] : static_cast<int>(t / a.tiles_per_seq);
        if (seq != prev_seq) {
          if (prev_seq >= 0) umma_commit(&qempty[slot]);
          slot = qcount & 1u;
          if (!mbar_wait(&qfull[slot], (qcount >> 1) & 1u, abort_flag)) break;
          ++qcount;
          prev_seq = seq;
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
    const int row = static_cast<int>(quad) * 32 + lane;  // row of the 128-key tile
    const int slot_j = row / bs;
    const int ingroup = row % bs;
    uint64_t selmask = 0, restmask = 0;
    if (kMode == kModeH8 || kMode == kModeProgressive) {
      selmask = head_mask(a.selected, kVerifierHeads);
      restmask = a.remaining ? head_mask(a.remaining, kHeads - kVerifierHeads) : ~selmask;
    }
    const float thr = (kMode == kModeProgressive) ? *a.threshold : 0.f;
    int prev_seq = -1, prev_slot = -1;  // prev_slot: the (sequence, segment) histogram the
                                        // group's shared counts belong to
    uint32_t hph = 0;
    uint32_t* ghist = shist + group * kKeyHistBins;
    uint64_t* gbar = hbar + group;
    float wr[kHeads];
    Tile tile;
    const int etid = (warp - 2 - 4 * group) * 32 + lane;  // 0..127 within the group
    // the group's four warps meet (bounded wait); false when the CTA aborts
    auto hist_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(gbar);
      const bool ok = mbar_wait(gbar, hph & 1u, abort_flag);
      ++hph;
      return ok;
    };
    // adds this CTA's counts of histogram `slot` (sequence * hist_segs + segment) to it and
    // clears them
    auto hist_flush = [&](int slot) -> bool {
      if (!hist_sync()) return false;
      uint32_t* dst = a.hist + static_cast<int64_t>(slot) * kKeyHistBins;
      for (int i = etid; i < kKeyHistBins; i += 128) {
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
      get_tile(a, t, tile);
      const int seq = tile.seq;
      if (seq != prev_seq) {
        load_head_weights(a.w + static_cast<int64_t>(seq) * a.w_stride, wr);
        prev_seq = seq;
      }
      if (use_hist) {  // the slot of the tile's first block (a tile may end in the next one)
        const int tslot = seq * a.hist_segs + ((max(tile.block[0], 0) * bs) >> 15);
        if (tslot != prev_slot) {
          if (prev_slot >= 0 && !hist_flush(prev_slot)) {
            ok = false;
            break;
          }
          prev_slot = tslot;
        }
      }
      const int blk = tile.block[slot_j];
      const int key = blk * bs + ingroup;
      const bool valid = blk >= 0 && key < a.length;
      const bool flag = (kMode != kModeExact && blk >= 0) ? mask_set<kMode>(a, seq, blk) : false;

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

      float out = -INFINITY, probe = -INFINITY;
      bool accept = false;
      if (kMode == kModeMasked) {
        if (flag) out = relu_weighted_sum(r0, r1, wr);
      } else if (kMode == kModeExact) {
        out = relu_weighted_sum(r0, r1, wr);
        probe = valid ? out : -INFINITY;
      } else {
        float sel, rest;
        split_head_sums(r0, r1, wr, selmask, sel, rest);
        if (kMode == kModeH8) {
          out = (flag && valid) ? sel : -INFINITY;
          probe = out;
        } else {  // progressive: flag = direct block
          probe = (valid && !flag) ? sel : -INFINITY;
          if (flag) {
            out = relu_weighted_sum(r0, r1, wr);
          } else {
            // rest over the listed remaining heads (complement of the selected ones by default)
            if (restmask != ~selmask) {
              float s2, r2;
              split_head_sums(r0, r1, wr, restmask, s2, r2);
              rest = s2;
            }
            out = sel + rest;
          }
        }
      }

      float bmax = -INFINITY;
      if (kMode != kModeMasked) {
        // max over 16-row groups, then over the block's groups across warps
        float m = probe;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((lane & 15) == 0) gmax[acc * 8 + quad * 2 + (lane >> 4)] = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(&grp[acc]);
        if (!mbar_wait(&grp[acc], aph, abort_flag)) {
          ok = false;
          break;
        }
        const int g0 = (slot_j * bs) >> 4, ng = bs >> 4;
        for (int g = 0; g < ng; ++g) bmax = fmaxf(bmax, gmax[acc * 8 + g0 + g]);
      }
      if (kMode == kModeProgressive) {
        accept = flag || (bmax >= thr);
        if (!accept) out = -INFINITY;
      }

      if (valid && (kMode != kModeH8 || a.out != nullptr))
        a.out[static_cast<int64_t>(seq) * a.out_stride + key] = out;
      if (use_hist) {
        const uint32_t bin = float_to_key(out) >> 20;
        const int kslot = seq * a.hist_segs + (key >> 15);
        add_to_bin(ghist, valid && kslot == prev_slot, bin);
        if (valid && kslot != prev_slot)
          atomicAdd(a.hist + static_cast<int64_t>(kslot) * kKeyHistBins + bin, 1u);
      }
      if (blk >= 0 && ingroup == 0) {
        if (kMode == kModeMasked) {
          if (a.accepted) a.accepted[static_cast<int64_t>(seq) * a.bm_stride + blk] = flag ? 1 : 0;
        } else if (kMode == kModeH8 || kMode == kModeExact) {
          a.block_max[static_cast<int64_t>(seq) * a.bm_stride + blk] = bmax;
        } else if (kMode == kModeProgressive) {
          a.block_max[static_cast<int64_t>(seq) * a.bm_stride + blk] = flag ? -INFINITY : bmax;
          a.accepted[static_cast<int64_t>(seq) * a.bm_stride + blk] = accept ? 1 : 0;
        }
      }
    }
    if (use_hist && ok && prev_slot >= 0) hist_flush(prev_slot);
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(a.status, TDSA_ERR_TIMEOUT);
}

template <int kMode, bool kBF16>
int launch_t(const CUtensorMap& kmap, const CUtensorMap& kmap_tile, const CUtensorMap& qmap,
             const BlockArgs& a, int grid, cudaStream_t stream) {
  auto kern = score_blocks_kernel<kMode, kBF16>;
  const int smem = kSmemBytes + (a.hist ? kHistSmemBytes : 0);
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem));
  TDSA_CUDA_CHECK(launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, kmap, kmap_tile,
                             qmap, a));
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

template <int kMode>
int launch_mode(bool bf16, const CUtensorMap& kmap, const CUtensorMap& kmap_tile,
                const CUtensorMap& qmap, const BlockArgs& a, int grid, cudaStream_t stream) {
  return bf16 ? launch_t<kMode, true>(kmap, kmap_tile, qmap, a, grid, stream)
              : launch_t<kMode, false>(kmap, kmap_tile, qmap, a, grid, stream);
}

}  // namespace

int make_key_maps(const void* q, int64_t q_bs, const void* k, int64_t k_bs, int64_t k_rs,
                  int dtype, int batch, int length, int box_rows, CUtensorMap* kmap,
                  CUtensorMap* qmap) {
  const CUtensorMapDataType dt =
      dtype == TDSA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(length),
                              static_cast<uint64_t>(batch)};
    const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(k_bs) * 2
                                       : static_cast<uint64_t>(k_rs) * 2 * length;
    const uint64_t strides[2] = {static_cast<uint64_t>(k_rs) * 2, bstride};
    const uint32_t box[3] = {64, static_cast<uint32_t>(box_rows), 1};
    int rc = encode_tmap(kmap, dt, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(kHeads),
                            static_cast<uint64_t>(batch)};
  const uint64_t bstride = batch > 1 ? static_cast<uint64_t>(q_bs) * 2
                                     : static_cast<uint64_t>(kHeads * kHeadDim * 2);
  const uint64_t strides[2] = {static_cast<uint64_t>(kHeadDim) * 2, bstride};
  const uint32_t box[3] = {64, kHeads, 1};
  return encode_tmap(qmap, dt, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_score_blocks(int mode, const void* q, int64_t q_bs, const void* k, int64_t k_bs,
                        int64_t k_rs, int dtype, int batch, const BlockArgs& args, int grid,
                        cudaStream_t stream) {
  CUtensorMap kmap, kmap_tile, qmap;
  int rc = make_key_maps(q, q_bs, k, k_bs, k_rs, dtype, batch, args.length, args.bs, &kmap,
                         &qmap);
  if (rc) return rc;
  if (args.bs == kTileKeys) {
    kmap_tile = kmap;
  } else {
    rc = make_key_maps(q, q_bs, k, k_bs, k_rs, dtype, batch, args.length, kTileKeys,
                       &kmap_tile, &qmap);
    if (rc) return rc;
  }
  const bool bf16 = dtype == TDSA_BF16;
  switch (mode) {
    case kModeH8: return launch_mode<kModeH8>(bf16, kmap, kmap_tile, qmap, args, grid, stream);
    case kModeMasked:
      return launch_mode<kModeMasked>(bf16, kmap, kmap_tile, qmap, args, grid, stream);
    case kModeProgressive:
      return launch_mode<kModeProgressive>(bf16, kmap, kmap_tile, qmap, args, grid, stream);
    case kModeExact:
      return launch_mode<kModeExact>(bf16, kmap, kmap_tile, qmap, args, grid, stream);
    default: return fail(TDSA_ERR_INVALID, "unknown block scoring mode");
  }
}

}  // namespace tdsa
