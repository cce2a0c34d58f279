// Host-side launchers of the indexer kernels (one definition per .cu file).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/tdsa.h"

namespace tdsa {

constexpr int kTopkSegment = 32768;    // keys one top-k CTA holds in shared memory
constexpr int kTopkMaxSorted = 8192;   // largest k sorted in shared memory
constexpr int kKeyHistBins = 4096;     // score-kernel key histogram: top 12 bits of the key

int launch_score_dense_tc(const void* q, int64_t q_bs, const float* w, int64_t w_bs,
                          const void* k, int64_t k_bs, int64_t k_rs, int dtype, int batch,
                          int length, float* out, int64_t o_bs, cudaStream_t stream,
                          int* status, uint32_t* hist = nullptr, void* trace = nullptr,
                          int64_t trace_bs = 0);

// Error-compensated TF32 scoring of float32 keys on the tensor cores (score_tf32.cu); needs
// 16-byte aligned q and keys and strides that are multiples of 4 floats.
bool score_dense_tf32_supported(const float* q, int64_t q_bs, const float* k, int64_t k_bs,
                                int64_t k_rs, int batch);
int launch_score_dense_tf32(const float* q, int64_t q_bs, const float* w, int64_t w_bs,
                            const float* k, int64_t k_bs, int64_t k_rs, int batch, int length,
                            float* out, int64_t o_bs, cudaStream_t stream, int* status);

int launch_score_dense_f32(const float* q, int64_t q_bs, const float* w, int64_t w_bs,
                           const float* k, int64_t k_bs, int64_t k_rs, int batch, int length,
                           float* out, int64_t o_bs, cudaStream_t stream);

// ---- block-structured scoring (score_blocks.cu)
enum BlockMode { kModeH8 = 0, kModeMasked = 1, kModeProgressive = 2, kModeExact = 3 };

struct BlockArgs {
  int bs = 64;                 // block size: 16, 32, 64 or 128
  int bpt = 2;                 // blocks per 128-key tile
  int length = 0;              // keys per sequence
  int nblocks = 0;             // ceil(length / bs)
  int tiles_per_seq = 0;       // contiguous tiles: ceil(nblocks / bpt)
  int64_t total_tiles = 0;     // contiguous tiles of the launch
  const int32_t* tile_seq = nullptr;     // listed tiles: sequence of tile t
  const int32_t* tile_blocks = nullptr;  // listed tiles: [t][bpt] block ids, -1 empty
  const int32_t* tile_count = nullptr;   // listed tiles: device count
  const int8_t* mask = nullptr;          // per block: cold (H8), keep (masked), direct (prog.)
  int64_t mask_stride = 0;
  const int32_t* selected = nullptr;     // 8 head ids (device)
  const int32_t* remaining = nullptr;    // 56 head ids (device) or null = complement
  const float* threshold = nullptr;      // progressive promotion threshold (device scalar)
  const float* w = nullptr;
  int64_t w_stride = 0;
  float* out = nullptr;                  // [batch][out_stride] per-key output
  int64_t out_stride = 0;
  float* block_max = nullptr;            // [batch][bm_stride]
  int64_t bm_stride = 0;
  int8_t* accepted = nullptr;            // [batch][bm_stride]
  int mask_invert = 0;                   // H8: a block is cold where the mask is zero
  const float* accept_max = nullptr;     // masked: keep = mask || accept_max >= *threshold
                                         // ([batch][bm_stride]), written to `accepted`
  uint32_t* hist = nullptr;              // exact: [batch][hist_segs][4096] key histograms
                                         // (top 12 bits of the order-preserving key), one
                                         // per 32768-key segment of a row, the epilogue adds
                                         // every scored key to
  int hist_segs = 1;
  int* status = nullptr;
};

int launch_score_blocks(int mode, const void* q, int64_t q_bs, const void* k, int64_t k_bs,
                        int64_t k_rs, int dtype, int batch, const BlockArgs& args, int grid,
                        cudaStream_t stream);

int launch_compact_blocks(const float* scores, int64_t s_stride, const int8_t* accepted,
                          int64_t a_stride, int batch, int length, int block_size,
                          float* out_scores, int32_t* out_indices, int64_t o_stride,
                          int32_t* out_count, cudaStream_t stream);

// ---- exact progressive path (exact.cu)
struct ExactLayout {
  size_t upper = 0, maxsq = 0, bound = 0, bmax = 0, flag = 0, topk = 0, qprev = 0, wprev = 0;
  size_t scores = 0, tau = 0, stats = 0, tile_seq = 0, tile_blk = 0, counters = 0, topk_ws = 0;
  size_t hist = 0;  // [batch][4096] key histogram of the step's scores (rows <= 32768)
  size_t topk_ws_bytes = 0, total = 0;
  int64_t nb_stride = 0, tcap = 0;
  int bpt = 0;
};

ExactLayout exact_layout(int batch, int max_length, int k, int block_size);

int run_exact(int init, uint8_t* state, const ExactLayout& L, const void* q, int64_t q_bs,
              const float* w, int64_t w_bs, const void* keys, int64_t k_bs, int64_t k_rs,
              int dtype, int batch, int prev_length, int length, int max_length, int k,
              int block_size, int sorted, void* out_idx, int idx_bytes, int64_t idx_bs,
              float* out_val, int64_t val_bs, cudaStream_t stream);

// ---- certified-bound helpers, float64 (certified.cu)
int launch_block_key_norms(const double* keys, int tokens, int heads, int dim, int bs,
                           double* out, cudaStream_t stream);
int launch_temporal_radius(const double* qn, const double* qp, const double* wn,
                           const double* wp, const double* norms, int heads, int dim, int nb,
                           double* coeff_ws, double* out, cudaStream_t stream);
int launch_relu_index_score(const double* q, const double* keys, const double* w, int heads,
                            int dim, int tokens, double* out, cudaStream_t stream);

// The exchange of an L-sharded merge over peer memory (exchange.cu: the region and the C
// ABI; topk.cu: the kernel).  Every rank owns one exchange region, mapped into the node's
// other ranks through CUDA IPC:
//   vals [2][rows][k] f32, idx [2][rows][k] i32: the rank's candidates, by step parity;
//   flags [2][world][rows] u32: (parity, src, row) holds the step's epoch once rank src has
//     published that row;
//   ctr [4] u32: the epoch of the last step, a CTA counter;
//   scratch vals / idx [rows][world * k]: the merge's gathered rows (local only).
constexpr int kMaxExchangeWorld = 16;
struct PeerGather {
  const uint8_t* const* peer_base;  // device array [world]: every rank's region (own included)
  uint8_t* own;                     // this rank's region
  int world, rank, rows, k;
  int64_t vals_off, idx_off, flags_off, ctr_off, scratch_v_off, scratch_i_off;
  const float* local_vals;          // this step's local top-k [rows][k] (from the previous
  const int32_t* local_idx;         // kernel), indices local to the shard
  int64_t local_stride;
  int32_t offset;                   // the shard's first global index
};
// One launch per step: each CTA publishes its row of the local top-k into the region and
// raises that row's flag in every rank's region, waits (bounded) for the row's flag from
// every rank, copies the ranks' rows into its scratch row and selects the top-k.
int launch_exchange_topk(const PeerGather& g, int sorted, void* out_idx, int idx_bytes,
                         int64_t oi_stride, float* out_val, int64_t ov_stride,
                         cudaStream_t stream);

size_t topk_workspace_bytes(int batch, int length, int k);
// CTAs per row the cluster top-k would use for rows of one histogram segment (1: none).
int topk_cluster_rows(int batch, int length);
// Key histograms [batch][4096] of score rows (<= 32768 keys), each row split over up to 16
// CTAs; hist is zeroed first.
int launch_row_hist_parts(const float* scores, int64_t l_stride, int batch, int length,
                          uint32_t* hist, cudaStream_t stream);
int topk_levels(int batch, int length, int k, int hist);
int topk_check(int length, int k, int sorted);
int launch_topk(const float* scores, int64_t s_stride, const int32_t* idx, int64_t idx_stride,
                int batch, int length, int k, int sorted, void* out_idx, int idx_bytes,
                int64_t oi_stride, float* out_val, int64_t ov_stride, void* ws, size_t ws_bytes,
                cudaStream_t stream, float* kth_out = nullptr, uint32_t* key_hist = nullptr,
                int32_t* mirror = nullptr, int64_t mirror_stride = 0);

// ---- certified INT8 key sketch (sketch.cu)
size_t sketch_workspace_bytes(int batch, int max_length, int k);
void sketch_workspace_offsets(int batch, int max_length, int k, int64_t* out);
int launch_sketch_keys(const void* keys, int64_t k_bs, int64_t k_rs, int dtype, int batch,
                       int first, int length, int8_t* sketch, int64_t sk_bs, float* scale,
                       void* bounds, int64_t sc_bs, cudaStream_t stream);
int run_sketch_topk(const void* q, int64_t q_bs, const float* w, int64_t w_bs, const void* keys,
                    int64_t k_bs, int64_t k_rs, int dtype, const int8_t* sketch, int64_t sk_bs,
                    const float* scale, const void* bounds, int64_t sc_bs, int batch,
                    int length, int max_length, int k, int sorted, void* out_idx,
                    int idx_bytes, int64_t idx_bs, float* out_val, int64_t val_bs,
                    unsigned long long* stats, void* ws, cudaStream_t stream);

int launch_hadamard128(const void* in, int64_t in_stride, int64_t rows, int dtype, void* out,
                       int64_t out_stride, cudaStream_t stream);
int launch_select_quantize(const void* in, int64_t in_stride, int64_t rows, int width,
                           int dtype, const int8_t* keep, int bits, double scale,
                           uint32_t* absmax, void* out, int64_t out_stride,
                           cudaStream_t stream);
int launch_bounded_wait_selftest(long long limit_cycles, cudaStream_t stream, int* status);
size_t packed_wq_bytes(int hidden);
int launch_pack_wq(const void* wq, int64_t stride, int hidden, void* out, cudaStream_t stream);
// ---- temporal policy state machine (policy.cu)
size_t policy_state_bytes(int batch, int k, int nbc, int64_t* offsets);
size_t policy_decide_smem_bytes(int length, int bs, int k);
int launch_policy(int init, uint8_t* state, int batch, int k, int nbc, const float* scores,
                  int64_t s_stride, const float* vscores, int64_t v_stride, int length,
                  int prev_length, int bs, const tdsa_policy* pol, int teacher,
                  int full_refresh, const tdsa_rescue* rescue, float* masked, float* cmax,
                  uint8_t* flags, int32_t* ranking, uint32_t* ebits, int64_t e_stride,
                  int32_t* base_new, int32_t* approx, void* topk_ws, size_t topk_ws_bytes,
                  double* stats, int* status, cudaStream_t stream);

// ---- decode-step key append (key_append.cu)
int launch_key_append(const void* hidden, int64_t hidden_stride, int hidden_size,
                      const void* wk, int64_t wk_stride, const float* ln_w, const float* ln_b,
                      float eps, const int64_t* positions, const int64_t* slots, void* cache,
                      int64_t cache_bs, int64_t cache_rs, int64_t cache_rows, int dtype,
                      int batch, int rope_dim, float theta, int* status, cudaStream_t stream);

int launch_query_project(const void* x, int64_t x_stride, int hidden, const void* wq,
                         int64_t wq_stride, int packed, const float* ww,
                         const int64_t* positions, void* q,
                         int64_t q_stride, float* w, int64_t w_stride, int dtype, int batch,
                         int rope_dim, float theta, float scale, void* qraw,
                         int64_t qraw_stride, cudaStream_t stream, int* status);

int launch_qprep(const void* qraw, int64_t qraw_stride, const void* x, int64_t x_stride,
                 int hidden, const float* ww, const int64_t* positions, void* q,
                 int64_t q_stride, float* w, int64_t w_stride, int dtype, int batch,
                 int rope_dim, float theta, float scale, cudaStream_t stream);

// Device status word of the current device (allocated with the module, never freed).
int* device_status_ptr();

}  // namespace tdsa
