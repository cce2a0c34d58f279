// Ordered compaction of flagged key blocks into the tile lists of the block-structured
// scoring kernel (score_blocks.cu), run by one 1024-thread CTA per sequence.
#pragma once

#include <cstdint>

namespace tdsa {

constexpr int kTileListThreads = 1024;  // threads of the CTA that calls emit_tiles

// Ordered compaction of the blocks with flag == want into tiles of bpt blocks.  Warp w
// takes the contiguous span of blocks [w * span, (w + 1) * span) (span a multiple of 32),
// counts its blocks with ballots and, after one exchange of the 32 warp counts and one
// atomic for the sequence's place in the list, writes them in order: two barriers whatever
// the block count.  A grid of one CTA (one sequence) owns the list from tile 0: it stores
// the count (the counter is zero on entry) instead of waiting on an atomic.  `reserved`
// (shared memory), when given, already holds the sequence's first tile, written before the
// call by a thread that took the atomic itself, and the list's second barrier is skipped.
// `flag` may be shared or global memory; `wtot` (32 words) and `sbase` are shared scratch.
__device__ __forceinline__ void emit_tiles(const int8_t* flag, int nb, int want, int bpt, int seq,
                           int32_t* tile_seq, int32_t* tile_blk, int32_t* counter,
                           uint32_t* wtot, uint32_t* sbase,
                           const uint32_t* reserved = nullptr) {
  constexpr int kWarps = kTileListThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int span = ((nb + kTileListThreads - 1) / kTileListThreads) * 32;
  const int lo = warp * span, hi = min(nb, lo + span);
  uint32_t cnt = 0;
  for (int b0 = lo; b0 < hi; b0 += 32) {
    const int b = b0 + lane;
    cnt += __popc(__ballot_sync(0xffffffffu, b < hi && flag[b] == want));
  }
  if (lane == 0) wtot[warp] = cnt;
  __syncthreads();
  uint32_t before = 0, total = 0;
#pragma unroll 8
  for (int i = 0; i < kWarps; ++i) {
    const uint32_t c = wtot[i];
    before += i < warp ? c : 0u;
    total += c;
  }
  uint32_t tile0;
  if (reserved) {
    tile0 = *reserved;
  } else if (gridDim.x * gridDim.y * gridDim.z == 1) {
    tile0 = 0u;
    if (threadIdx.x == 0) *counter = static_cast<int32_t>((total + bpt - 1) / bpt);
  } else {
    if (threadIdx.x == 0) {
      const int ntiles = static_cast<int>((total + bpt - 1) / bpt);
      sbase[0] = ntiles ? static_cast<uint32_t>(atomicAdd(counter, ntiles)) : 0u;
    }
    __syncthreads();
    tile0 = sbase[0];
  }
  const unsigned lt = (1u << lane) - 1u;
  uint32_t pos = before;
  for (int b0 = lo; b0 < hi; b0 += 32) {
    const int b = b0 + lane;
    const bool take = b < hi && flag[b] == want;
    const unsigned bal = __ballot_sync(0xffffffffu, take);
    if (take) {
      const uint32_t p = pos + __popc(bal & lt);
      const uint32_t t = tile0 + p / bpt;
      tile_blk[static_cast<int64_t>(t) * bpt + p % bpt] = b;
      if (p % bpt == 0) tile_seq[t] = seq;
    }
    pos += __popc(bal);
  }
  // pad the last tile with empty slots
  if (threadIdx.x < bpt && total % bpt) {
    const uint32_t p = total + threadIdx.x;
    if (p % bpt != 0 && p / bpt == (total - 1) / bpt)
      tile_blk[static_cast<int64_t>(tile0 + p / bpt) * bpt + p % bpt] = -1;
  }
}

}  // namespace tdsa
