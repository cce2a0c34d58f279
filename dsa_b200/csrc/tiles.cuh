// Ordered compaction of flagged key blocks into the tile lists of the block-structured
// scoring kernel (score_blocks.cu), run by one 1024-thread CTA per sequence.
#pragma once

#include <cstdint>

namespace tdsa {

constexpr int kTileListThreads = 1024;  // threads of the CTA that calls emit_tiles

// Ordered compaction of the blocks with flag == want into tiles of bpt blocks.
__device__ __forceinline__ void emit_tiles(const int8_t* flag, int nb, int want, int bpt, int seq,
                           int32_t* tile_seq, int32_t* tile_blk, int32_t* counter,
                           uint32_t* wtot, uint32_t* sbase) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // count
  uint32_t cnt = 0;
  for (int b = threadIdx.x; b < nb; b += kTileListThreads) cnt += flag[b] == want;
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) wtot[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t total = 0;
    for (int i = 0; i < 32; ++i) total += wtot[i];
    const int ntiles = static_cast<int>((total + bpt - 1) / bpt);
    sbase[0] = ntiles ? static_cast<uint32_t>(atomicAdd(counter, ntiles)) : 0u;
    sbase[1] = 0;  // running position
    sbase[2] = total;
  }
  __syncthreads();
  const uint32_t tile0 = sbase[0], total = sbase[2];
  // ordered positions, 1024 blocks per round
  for (int base = 0; base < nb; base += kTileListThreads) {
    const int b = base + threadIdx.x;
    const bool take = b < nb && flag[b] == want;
    const unsigned bal = __ballot_sync(0xffffffffu, take);
    if (lane == 0) wtot[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, round = 0;
    for (int i = 0; i < 32; ++i) {
      const uint32_t c = wtot[i];
      before += i < warp ? c : 0u;
      round += c;
    }
    const uint32_t pos = sbase[1] + before + __popc(bal & ((1u << lane) - 1u));
    if (take) {
      const uint32_t t = tile0 + pos / bpt;
      tile_blk[static_cast<int64_t>(t) * bpt + pos % bpt] = b;
      if (pos % bpt == 0) tile_seq[t] = seq;
    }
    __syncthreads();
    if (threadIdx.x == 0) sbase[1] += round;
    __syncthreads();
  }
  // pad the last tile with empty slots
  if (threadIdx.x < bpt && total % bpt) {
    const uint32_t pos = total + threadIdx.x;
    if (pos % bpt != 0 && pos / bpt == (total - 1) / bpt)
      tile_blk[static_cast<int64_t>(tile0 + pos / bpt) * bpt + pos % bpt] = -1;
  }
}

}  // namespace tdsa
