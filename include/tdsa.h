/*
 * tdsa.h -- C ABI of the B200 (sm_100a) Lightning-Indexer decode path.
 *
 * Plain pointers, sizes and strides; no framework types.  Every device pointer must point
 * into memory of the CUDA device current on the calling thread; `stream` is a cudaStream_t
 * (NULL = legacy default stream).  Calls are asynchronous on `stream` unless noted.
 * Return value: TDSA_OK or an error code; tdsa_last_error() gives the message
 * (thread-local).  Argument errors are detected on the host before any launch.
 *
 * Index semantics follow the reference project temporal_dsa (psa1582/dsa):
 *   score[s] = sum_h w[h] * ReLU(q[h] . k[s]),  H = 64 heads, D = 128 dims;
 *   top-k order = descending score, equal scores by ascending index.
 * Strides are in elements of the pointed-to type.
 */
#ifndef TDSA_H_
#define TDSA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tdsa_status {
  TDSA_OK = 0,
  TDSA_ERR_INVALID = 1,     /* bad shape, stride, size or pointer argument           */
  TDSA_ERR_UNSUPPORTED = 2, /* valid request this build does not implement            */
  TDSA_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed                      */
  TDSA_ERR_TIMEOUT = 4,     /* device status bit: a bounded in-kernel wait ran out    */
  TDSA_ERR_ALIGN = 5,       /* a pointer or stride breaks the 16-byte TMA alignment   */
  TDSA_ERR_WORKSPACE = 6    /* workspace missing or smaller than the query said       */
};

/* Device status bit (tdsa_device_status) besides TDSA_ERR_TIMEOUT: a device-side index
 * (a key-append slot) was outside its buffer; that store was skipped. */
#define TDSA_STATUS_RANGE 8
/* Device status bit: a top-k over rows just past one 32768-key segment, started from the
 * caller's key histograms, found histograms that do not describe the row (their counts
 * miss the k-th key); that row's output was not written. */
#define TDSA_STATUS_HIST 16

enum tdsa_dtype { TDSA_F32 = 0, TDSA_F16 = 1, TDSA_BF16 = 2 };

/*
 * Dimension-sparse verifier scorer (src/temporal_dsa/verifier_scoring.py:9-139).
 * tdsa_hadamard128 -- replaces normalized_hadamard (:9-26) for 128-wide rows: out[r] =
 *   H_128 in[r] / sqrt(128) (orthonormal Walsh-Hadamard, Sylvester order), float32
 *   arithmetic in the reference's butterfly order, rounded once to `dtype`.
 * tdsa_select_quantize -- the selection and fake_symmetric_quantize (:29-41) steps of
 *   score_dim_sparse (:95-139) on [rows][width] rows: out = in on the dimensions with
 *   keep[d] != 0 (keep: device int8 [width], NULL = all), 0 elsewhere; with bits in
 *   {2, 4, 8} the kept values become clamp(rint(x / s), -L, L) * s, L = 2^(bits-1) - 1,
 *   s = scale if scale > 0 else (max |x| over the kept entries) / L (the max is left in
 *   *absmax_word as float bits).  score_dim_sparse is then tdsa_score_dense on the
 *   transformed queries and keys.
 */
int tdsa_hadamard128(const void* in, int64_t in_row_stride, int64_t rows, int dtype, void* out,
                     int64_t out_row_stride, void* stream);
int tdsa_select_quantize(const void* in, int64_t in_row_stride, int64_t rows, int width,
                         int dtype, const int8_t* keep, int bits, double scale,
                         uint32_t* absmax_word, void* out, int64_t out_row_stride,
                         void* stream);

/*
 * Decode-step key append.
 * Replaces: LightningIndexerSidecar.encode_keys (src/temporal_dsa/sidecar.py:74-76) for one
 *   new token per sequence, followed by the write of that key into the cache.
 * For b < batch: raw = hidden[b] @ w_k^T (float32 accumulation, rounded to `dtype`, the
 *   Linear's output), y = LayerNorm(raw) (float32, biased variance, eps, then *ln_weight
 *   + ln_bias; NULL weight = 1, NULL bias = 0), RoPE on the first rope_dim features
 *   (non-interleaved halves, angle = float32(positions[b]) * rope_theta^(-j/(rope_dim/2)),
 *   sidecar.py:10-28), stored rounded to `dtype` at cache[b * cache_batch_stride +
 *   slot * cache_row_stride + 0..127], slot = slots[b] (slots NULL: positions[b]).
 *   A slot outside [0, cache_rows) skips that row's store and raises TDSA_STATUS_RANGE.
 *   w_k is read as a constant (fetched before the wait on the previous kernel of `stream`):
 *   it must not be written by a kernel still running on that stream.
 * hidden [batch][hidden_size] and w_k [128][hidden_size] are 16-bit (dtype TDSA_BF16 or
 *   TDSA_F16), 16-byte aligned, row strides multiples of 8 elements; hidden_size a
 *   multiple of 8; positions/slots device int64 [batch]; rope_dim even, <= 128.
 * One launch on `stream`.
 */
int tdsa_key_append(const void* hidden, int64_t hidden_stride, int hidden_size,
                    const void* w_k, int64_t wk_row_stride, const float* ln_weight,
                    const float* ln_bias, float eps, const int64_t* positions,
                    const int64_t* slots, void* cache, int64_t cache_batch_stride,
                    int64_t cache_row_stride, int64_t cache_rows, int dtype, int batch,
                    int rope_dim, float rope_theta, void* stream);

/*
 * Temporal policy state machine on the device (no host round trip per step).
 * Replaces: approx.initialize_state / approx.replay_step (src/temporal_dsa/approx.py:112-364)
 *   and verifier.verifier_step's rescue and rerank (src/temporal_dsa/verifier.py:103-375),
 *   which the reference runs in numpy on a copy of each step's scores
 *   (scripts/evaluate_teacher_forced.py:163-230).
 * State (per sequence, opaque buffer of tdsa_policy_state_bytes; tdsa_policy_state_offsets
 *   gives the byte offsets of its arrays): topk and baseline_topk [batch][k] int32 (stable
 *   top-k order), last_max, ema, volatility [batch][max_blocks] float32, age, cold_streak
 *   [batch][max_blocks] int16, and the block count each sequence's arrays hold.
 * tdsa_policy_init -- initialize_state for `batch` rows of `length` scores.
 * tdsa_policy_step -- replay_step (rescue NULL) or verifier_step (rescue given, with the
 *   verifier scores): history_mode 0 = "own", 1 = "teacher"; full_refresh is the host's
 *   (policy.name == "full" or refresh_interval divides step or fallback) flag.  The new
 *   selection is left in the state's topk.  Outputs: evaluated_bits [batch][bits_stride]
 *   (bit j = key j read, after any rescue), block_flags [batch][max_blocks] (bit0 forced,
 *   bit1 read by the policy, bit2 rescued, bit3 holds a seed key, bit4 holds a cold key),
 *   ranking [batch][max_blocks] (rescue: cold blocks by verifier maximum; may be NULL),
 *   stats [batch][TDSA_POLICY_NSTATS] (TDSA_PST_*; TDSA_PST_ERROR = 1 when the seed is not
 *   k distinct keys below length: the state is then unchanged).
 * Limits: k <= 2048, block_size a power of two <= 128, ceil(length/block_size) <= max_blocks <= 4096,
 *   length <= 131072.  Scores are expected finite (a key whose score is -inf ties with the
 *   keys the policy did not read).  All device buffers; asynchronous on `stream`.
 */
enum tdsa_block_order {
  TDSA_ORDER_ADDRESS = 0,
  TDSA_ORDER_PREVIOUS_MAX = 1, /* also "predicted_risk" */
  TDSA_ORDER_BUCKET = 2,       /* "bucketN", N in tdsa_policy.buckets */
  TDSA_ORDER_ORACLE_CURRENT = 3
};
enum tdsa_risk_model { TDSA_RISK_LAST_MAX = 0, TDSA_RISK_EMA = 1 };

typedef struct tdsa_policy { /* approx.py:15-39 ApproxPolicy */
  double gamma;
  double ema_alpha;
  double volatility_lambda;
  double age_slope;
  int cold_streak;
  int dynamic_threshold;
  int order;  /* tdsa_block_order */
  int buckets;
  int age_cap; /* < 0: none */
  int recent_window;
  int risk_model; /* tdsa_risk_model */
} tdsa_policy;

typedef struct tdsa_rescue { /* verifier.py:15-43 VerifierConfig + promotion threshold */
  double rescue_fraction;
  double promotion_threshold;
  int use_threshold; /* 0: rescue ceil(rescue_fraction * cold blocks) best blocks */
} tdsa_rescue;

enum tdsa_policy_stat {
  TDSA_PST_ERROR = 0,
  TDSA_PST_TAU_SEED,
  TDSA_PST_TAU_FINAL,
  TDSA_PST_SCORED,     /* keys the temporal policy read (seed + refreshed blocks) */
  TDSA_PST_UNION,      /* keys read after the rescue */
  TDSA_PST_REFRESHED,
  TDSA_PST_SKIPPED,
  TDSA_PST_RESCUED,
  TDSA_PST_COLD_BLOCKS,
  TDSA_PST_SEED_BLOCKS,
  TDSA_PST_PHYS16, /* 16/32/64/128-key blocks holding a key read */
  TDSA_PST_PHYS32,
  TDSA_PST_PHYS64,
  TDSA_PST_PHYS128,
  TDSA_PST_TOP128, /* baseline[:N] members in the selection, N = 128 ... 2048 */
  TDSA_PST_TOP256,
  TDSA_PST_TOP512,
  TDSA_PST_TOP1024,
  TDSA_PST_TOP2048,
  TDSA_PST_MISSED,
  TDSA_PST_WORST_MISSED,
  TDSA_PST_NEWLY_HOT,
  TDSA_PST_NEWLY_HOT_MISSED,
  TDSA_PST_MASS_NUM, /* sum exp(score - max baseline score) over the selection */
  TDSA_PST_MASS_DEN, /* ... over the baseline */
  TDSA_PST_BLOCKS,
  TDSA_POLICY_NSTATS
};

size_t tdsa_policy_state_bytes(int batch, int k, int max_blocks);
int tdsa_policy_state_offsets(int batch, int k, int max_blocks, int64_t* offsets8);
size_t tdsa_policy_workspace_bytes(int batch, int max_length, int k, int max_blocks);
int tdsa_policy_init(void* state, size_t state_bytes, const float* scores, int64_t s_stride,
                     int batch, int length, int k, int block_size, int max_blocks,
                     void* workspace, size_t workspace_bytes, void* stream);
int tdsa_policy_step(void* state, size_t state_bytes, const float* scores, int64_t s_stride,
                     const float* verifier_scores, int64_t v_stride, int batch, int length,
                     int previous_length, int k, int block_size, int max_blocks,
                     const tdsa_policy* policy, int history_mode, int full_refresh,
                     const tdsa_rescue* rescue, void* workspace, size_t workspace_bytes,
                     uint32_t* evaluated_bits, int64_t bits_stride, uint8_t* block_flags,
                     int32_t* ranking, double* stats, void* stream);

/*
 * Failure-path self-test (no reference counterpart): one kernel waits on an mbarrier that
 * nothing arrives on, with the same bounded loop every in-kernel wait of this library
 * uses but a limit of `limit_cycles` SM cycles; when the limit runs out it raises
 * TDSA_ERR_TIMEOUT in the device status word (read it with tdsa_device_status) and
 * returns.  The context stays usable.  Asynchronous on `stream`.
 */
int tdsa_selftest_bounded_wait(long long limit_cycles, void* stream);

/* Library version string. */
const char* tdsa_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* tdsa_last_error(void);

/* Reads (and with reset != 0 clears) the device status word of the current device: the
 * OR of error bits kernels raised (TDSA_ERR_TIMEOUT when a bounded wait ran out,
 * TDSA_STATUS_RANGE when a device-side index was out of range, TDSA_STATUS_HIST when a key
 * histogram did not describe its row).
 * Synchronous. */
int tdsa_device_status(int* status_out, int reset);

/*
 * Dense indexer scores for a batch of independent sequences.
 * Replaces: full_scores_triton + _full_score_kernel (src/temporal_dsa/progressive_kernel.py:
 *   362-375, 195-215), torch_full_scores (:45-55) and the batched
 *   LightningIndexerSidecar.score_encoded (src/temporal_dsa/sidecar.py:89-107, Q = 1).
 * queries  [batch][64][128] of `dtype` (rows of one sequence contiguous), batch stride
 *          q_batch_stride (>= 8192);
 * weights  [batch][64] float32, batch stride w_batch_stride (>= 64);
 * keys     [batch][length][128] of `dtype`, rows k_row_stride apart (>= 128), sequences
 *          k_batch_stride apart;
 * scores   [batch][length] float32 out, batch stride s_batch_stride (>= length).
 * dtype TDSA_BF16 / TDSA_F16 run on the tcgen05 tensor cores (f32 accumulation).
 * TDSA_F32 runs on the tensor cores as error-compensated TF32 (q_hi.k_hi + q_lo.k_hi +
 * q_hi.k_lo, relative error ~2^-21 per product) when queries and keys have 16-byte aligned
 * bases and strides that are multiples of 4 floats, else an FP32 CUDA-core kernel.  16-bit
 * queries/keys need 16-byte aligned bases and strides that are multiples of 8 elements
 * (TMA).
 */
int tdsa_score_dense(const void* queries, int64_t q_batch_stride, const float* weights,
                     int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                     int64_t k_row_stride, int dtype, int batch, int length, float* scores,
                     int64_t s_batch_stride, void* stream);

/* Bytes of device workspace tdsa_topk needs for these sizes (0 if none).  For a batch of
 * rows of at most 32768 keys too small to fill the GPU one CTA per row, it also covers the
 * rows' key histograms: given at least this much (16-byte aligned), unsorted calls spread
 * each row over several SMs (a split histogram pass, then the cluster selection); with
 * less, they take the one-CTA-per-segment levels. */
size_t tdsa_topk_workspace_bytes(int batch, int length, int k);

/*
 * Row-wise exact top-k of a [batch][length] float32 score matrix.
 * Replaces: stable_topk (src/temporal_dsa/metrics.py:9-22) and the torch.topk calls that
 *   follow the score kernels (scripts/benchmark_progressive_dsa.py:117-169).
 * sorted != 0: each row in stable_topk order (score descending, ties by ascending index);
 * sorted == 0: the same index set in ascending index order.
 * out_indices [batch][k] of index_bytes (4 = int32, 8 = int64), row stride idx_batch_stride;
 * out_values  [batch][k] float32 or NULL, row stride val_batch_stride.
 * NaN ranks above +inf; -0.0 equals +0.0.  1 <= k <= length; k <= 8192 when sorted or
 * when length > 32768.
 */
int tdsa_topk(const float* scores, int64_t s_batch_stride, int batch, int length, int k,
              int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
              float* out_values, int64_t val_batch_stride, void* workspace,
              size_t workspace_bytes, void* stream);

/*
 * Merge candidate lists into a top-k per row (the second level of a sharded top-k: the
 * global top-k is contained in the union of the shards' local top-k).  New entry point,
 * no counterpart in the reference (which never shards).
 * cand_values [batch][count] float32 and cand_indices [batch][count] int32, row stride
 * cand_batch_stride; within a row the candidates must be in ascending index order (what
 * tdsa_topk with sorted == 0 produces, concatenated shard by shard).
 */
int tdsa_merge_topk(const float* cand_values, const int32_t* cand_indices,
                    int64_t cand_batch_stride, int batch, int count, int k, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* stream);

/*
 * Candidate exchange of an L-sharded top-k over peer memory (NVLink), in place of an
 * all-gather + tdsa_merge_topk.  New entry points, no counterpart in the reference (which
 * never shards).  One process per GPU, all ranks on one node.
 *
 * tdsa_exchange_create allocates this rank's exchange region (tdsa_exchange_bytes) and
 * writes its CUDA IPC handle (TDSA_IPC_HANDLE_BYTES bytes); the caller gathers every rank's
 * handle, rank-major, and passes them to tdsa_exchange_connect (synchronous).  Each step,
 * every rank calls tdsa_exchange_topk on its stream with its local top-k: values
 * [batch][k] float32 and indices [batch][k] int32 local to the shard (ascending index
 * order within a row, as tdsa_topk with sorted == 0 gives), row stride batch_stride, and
 * index_offset = the shard's first global index.  One launch publishes the rows into the
 * region, waits per row and bounded (about a second) for every rank's rows of the same
 * step, pulls them over NVLink and writes the global top-k (index_bytes 4 or 8).  A wait
 * that runs out raises TDSA_ERR_TIMEOUT in the device status word and leaves that row's
 * output undefined.  world * k <= 32768.  tdsa_exchange_destroy (synchronous) must run on
 * every rank only after all ranks' last step has finished (a barrier), since peers read
 * this rank's region.
 */
#define TDSA_IPC_HANDLE_BYTES 64
typedef struct tdsa_exchange tdsa_exchange;
size_t tdsa_exchange_bytes(int world, int batch, int k);
int tdsa_exchange_create(int world, int rank, int batch, int k, tdsa_exchange** out,
                         void* ipc_handle_out);
int tdsa_exchange_connect(tdsa_exchange* ex, const void* handles);
int tdsa_exchange_topk(tdsa_exchange* ex, const float* values, const int32_t* indices,
                       int64_t batch_stride, int32_t index_offset, int sorted,
                       void* out_indices, int index_bytes, int64_t idx_batch_stride,
                       float* out_values, int64_t val_batch_stride, void* stream);
int tdsa_exchange_destroy(tdsa_exchange* ex);

/* Bytes of device workspace tdsa_score_topk needs. */
size_t tdsa_score_topk_workspace_bytes(int batch, int length, int k);

/*
 * Dense scores followed by the row-wise top-k (tdsa_score_dense + tdsa_topk), the
 * "full_plus_topk" step of scripts/benchmark_progressive_dsa.py:117-123.  The scores live
 * in the caller's workspace.
 */
int tdsa_score_topk(const void* queries, int64_t q_batch_stride, const float* weights,
                    int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                    int64_t k_row_stride, int dtype, int batch, int length, int k, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * tdsa_score_topk without a workspace argument and without any device allocation.  No
 * counterpart in the reference: it is for callers that cannot allocate device memory at
 * call time -- C or C++ host code with no device allocator of its own, or a serving loop
 * that keeps its device footprint fixed after start-up -- and so cannot supply the
 * workspace tdsa_score_topk asks for.
 *
 * Scratch (scores, key histograms, top-k candidates) is one static 16 MiB buffer in the
 * library's device memory, one per device.  A call needing more than that
 * (tdsa_score_topk_workspace_bytes(batch, length, k) > 16 MiB, e.g. batch > 113 at length
 * 32768) returns TDSA_ERR_UNSUPPORTED before touching the device.  The first call on a
 * device does a one-time set-up (it looks up the buffer's device address, which may load
 * the library's module on that device): make that first call before any stream capture.
 * The looked-up address is kept for the life of the process: after a device reset (or a
 * reset of the primary context) the library must be reloaded before this entry point is
 * used again.  All calls on one device share the buffer, so calls that can overlap in time (different
 * streams, or host threads) race on it; calls issued in order on one stream do not.
 * Results are the same as tdsa_score_topk's.
 */
int tdsa_score_topk_noalloc(const void* queries, int64_t q_batch_stride, const float* weights,
                            int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                            int64_t k_row_stride, int dtype, int batch, int length, int k,
                            int sorted, void* out_indices, int index_bytes,
                            int64_t idx_batch_stride, float* out_values,
                            int64_t val_batch_stride, void* stream);

/*
 * The two halves of tdsa_score_topk for callers that keep their own buffers (a decode loop):
 * tdsa_score_dense_hist is tdsa_score_dense (16-bit keys) that also adds every score's key
 * histogram (order-preserving uint32 key >> 20, 4096 bins) to key_hist, one histogram per
 * 32768-key segment of each row: [batch][ceil(length / 32768)][4096]
 * (tdsa_key_hist_bytes), which must be zero on entry.  tdsa_topk_hist is tdsa_topk for
 * rows of at most 32768 keys that starts from that histogram instead of a full first pass,
 * and leaves key_hist zeroed again; tdsa_topk_hist_ws takes any length with the workspace
 * of tdsa_topk_workspace_bytes (every first-level segment starts from its histogram, and a
 * one-segment merge level from the bins the first level passes on).
 */
size_t tdsa_key_hist_bytes(int batch, int length);
/* Kernel launches (levels) of one top-k call.  with_key_hist: bit 0 -- tdsa_topk_hist_ws's
 * plan (key histograms given), bit 1 -- sorted output.  An unsorted call with histograms on
 * rows of up to 32768 + 4096 keys is one level. */
int tdsa_topk_levels(int batch, int length, int k, int with_key_hist);
int tdsa_topk_hist_ws(const float* scores, int64_t s_batch_stride, int batch, int length,
                      int k, int sorted, void* out_indices, int index_bytes,
                      int64_t idx_batch_stride, float* out_values, int64_t val_batch_stride,
                      uint32_t* key_hist, void* workspace, size_t workspace_bytes,
                      void* stream);
int tdsa_score_dense_hist(const void* queries, int64_t q_batch_stride, const float* weights,
                          int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                          int64_t k_row_stride, int dtype, int batch, int length, float* scores,
                          int64_t s_batch_stride, uint32_t* key_hist, void* stream);

/*
 * tdsa_score_dense_hist (key_hist may be null: no histogram) that also writes every score
 * rounded to float16 (round to nearest even) at trace[b * trace_batch_stride + s] for s <
 * length; nothing else of the trace is touched.  This emits one row of a score trace per
 * call from the score kernel itself: temporal_dsa/training.py:146-175 (evaluate_and_trace)
 * builds the same row on the host as score_encoded(...).float().cpu().numpy()
 * .astype(np.float16), padded with -inf to the trace width, and trace.py:34-61 saves it.
 */
int tdsa_score_dense_trace(const void* queries, int64_t q_batch_stride, const float* weights,
                           int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                           int64_t k_row_stride, int dtype, int batch, int length,
                           float* scores, int64_t s_batch_stride, uint32_t* key_hist,
                           uint16_t* trace, int64_t trace_batch_stride, void* stream);

int tdsa_topk_hist(const float* scores, int64_t s_batch_stride, int batch, int length, int k,
                   int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
                   float* out_values, int64_t val_batch_stride, uint32_t* key_hist,
                   void* stream);

/*
 * Block-structured kernels (block_size 16, 32, 64 or 128; 16-bit keys).  Keys of a block
 * that is not needed are never read.  Per-block arrays ([batch][bm_batch_stride], int8 or
 * float32) share one row stride >= ceil(length / block_size); per-key outputs have row
 * stride >= length.  selected_heads: 8 head ids (device int32), the same for every row.
 *
 * tdsa_h8_block_max -- replaces h8_block_max_triton + _h8_block_max_kernel
 *   (src/temporal_dsa/progressive_kernel.py:378-404, :218-246): partial = 8-head score of
 *   the keys of cold blocks, -inf elsewhere; block_max = per-block max of partial.
 */
int tdsa_h8_block_max(const void* queries, int64_t q_batch_stride, const float* weights,
                      int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                      int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                      const int32_t* selected_heads, const int8_t* cold_blocks,
                      float* partial, int64_t p_batch_stride, float* block_max,
                      int64_t bm_batch_stride, void* stream);

/* tdsa_masked_dense -- replaces masked_full_scores_triton + _masked_full_kernel
 *   (progressive_kernel.py:407-424, :249-274): dense scores of kept blocks, -inf elsewhere. */
int tdsa_masked_dense(const void* queries, int64_t q_batch_stride, const float* weights,
                      int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                      int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                      const int8_t* keep_blocks, int64_t keep_batch_stride, float* scores,
                      int64_t s_batch_stride, void* stream);

/* tdsa_two_pass -- replaces two_pass_scores_triton (progressive_kernel.py:478-497) in one
 *   call: block_max = the 8-head probe maximum of every cold block (direct_blocks[b] == 0;
 *   -inf for direct blocks), accepted[b] = direct or block_max >= *threshold (device float),
 *   scores = dense scores of the accepted blocks, -inf elsewhere.  Two launches; rejected
 *   blocks are read by the probe only, and the probe's partial scores are not stored. */
int tdsa_two_pass(const void* queries, int64_t q_batch_stride, const float* weights,
                  int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                  int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                  const int32_t* selected_heads, const int8_t* direct_blocks,
                  const float* threshold, float* scores, int64_t s_batch_stride,
                  int8_t* accepted, float* block_max, int64_t bm_batch_stride, void* stream);

/* tdsa_progressive_h8 -- replaces progressive_scores_triton + _progressive_kernel
 *   (progressive_kernel.py:427-475, :277-346), dense output: direct blocks score all 64
 *   heads (block_max -inf); cold blocks score the 8 selected heads, are promoted when their
 *   block max >= *threshold (device float) and then add the remaining heads
 *   (remaining_heads: 56 device ids, or NULL for the complement of selected_heads);
 *   rejected blocks score -inf; accepted[b] = 1 for direct or promoted blocks. */
int tdsa_progressive_h8(const void* queries, int64_t q_batch_stride, const float* weights,
                        int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                        int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                        const int32_t* selected_heads, const int32_t* remaining_heads,
                        const int8_t* direct_blocks, const float* threshold, float* scores,
                        int64_t s_batch_stride, int8_t* accepted, float* block_max,
                        int64_t bm_batch_stride, void* stream);

/* tdsa_compact_blocks -- the compact output of progressive_scores_triton (:335-340,
 *   :468-474): the scores and indices of every valid key of the accepted blocks, packed in
 *   ascending key order, and their count (device int32 per row). */
int tdsa_compact_blocks(const float* scores, int64_t s_batch_stride, const int8_t* accepted,
                        int64_t a_batch_stride, int batch, int length, int block_size,
                        float* out_scores, int32_t* out_indices, int64_t out_batch_stride,
                        int32_t* out_count, void* stream);

/*
 * Certified INT8 key sketch (no reference counterpart: the reference quantizes with one
 * symmetric scale per tensor and uses the result as an approximate verifier score,
 * fake_symmetric_quantize / score_dim_sparse in src/temporal_dsa/verifier_scoring.py:29-41,
 * :95-139; here the quantization is per key and comes with a certified error bound, so the
 * top-k it feeds stays exact).
 *
 * tdsa_sketch_keys -- sketches keys [first, length) of a 16-bit cache: sketch[b][key] =
 *   128 int8 values rint(k / s) (row stride 128 bytes, batch stride sketch_batch_stride
 *   bytes), scales[b][key] = s = max|k_i| / 127, bounds[b][key] = two float16 values
 *   (residual norm >= ||k - s k^||, norm >= ||s k^||), both rounded up; scales and bounds share
 *   scale_batch_stride (elements).  A key holding a non-finite value gets scale 0 and
 *   infinite bounds (always read in full).  136 bytes per key.
 *
 * tdsa_sketch_topk -- the exact top-k (as tdsa_topk of tdsa_score_dense's scores, ties
 *   included) that reads each key's sketch and the full 16-bit keys only of the 16-key blocks
 *   holding a key whose certified upper bound reaches tau, a lower bound of the k-th score
 *   (the k-th largest certified lower bound).  Five launches; workspace of
 *   tdsa_sketch_topk_workspace_bytes(batch, max_length, k) bytes, 256-byte aligned, any
 *   contents (max_length >= length sets its row strides).  stats (device, may be NULL):
 *   per row two uint64 counters the call adds to: keys read in full, 16-key blocks read.
 *   tdsa_sketch_workspace_offsets fills offsets[6] for checks of the last call: the byte
 *   offsets of the blocks' largest upper bounds (float32 [batch][block stride]), the keys'
 *   lower bounds and scores (float32 [batch][row stride] each) and tau (float32 [batch]),
 *   then the block stride and the row stride (elements).
 */
int tdsa_sketch_keys(const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                     int batch, int first, int length, int8_t* sketch,
                     int64_t sketch_batch_stride, float* scales, void* bounds,
                     int64_t scale_batch_stride, void* stream);
size_t tdsa_sketch_topk_workspace_bytes(int batch, int max_length, int k);
int tdsa_sketch_workspace_offsets(int batch, int max_length, int k, int64_t* offsets);
int tdsa_sketch_topk(const void* queries, int64_t q_batch_stride, const float* weights,
                     int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                     int64_t k_row_stride, int dtype, const int8_t* sketch,
                     int64_t sketch_batch_stride, const float* scales, const void* bounds,
                     int64_t scale_batch_stride, int batch, int length, int max_length, int k,
                     int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
                     float* out_values, int64_t val_batch_stride, uint64_t* stats,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Exact (certified) progressive top-k over a growing key cache (the schedule of
 * src/temporal_dsa/replay.py:172-222 with the bound of certified.py:18-48, which the
 * reference only replays on precomputed scores).  The caller owns `state`
 * (tdsa_exact_state_bytes bytes of device memory, any contents); tdsa_exact_init scores
 * densely and fills it, each tdsa_exact_step then seeds from the previous top-k, scores the
 * blocks holding those keys and the keys appended since the last call (prev_length ..
 * length), and skips every other block whose certified bound is below the running k-th
 * score.  The returned top-k equals dense scoring's.  16-bit keys; block_size 16/32/64/128;
 * batch, max_length, k and block_size must match the state's.  Outputs as tdsa_topk
 * (out_indices may be NULL).
 */
size_t tdsa_exact_state_bytes(int batch, int max_length, int k, int block_size);

int tdsa_exact_init(void* state, size_t state_bytes, const void* queries,
                    int64_t q_batch_stride, const float* weights, int64_t w_batch_stride,
                    const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                    int batch, int length, int max_length, int k, int block_size, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* stream);

int tdsa_exact_step(void* state, size_t state_bytes, const void* queries,
                    int64_t q_batch_stride, const float* weights, int64_t w_batch_stride,
                    const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                    int batch, int prev_length, int length, int max_length, int k,
                    int block_size, int sorted, void* out_indices, int index_bytes,
                    int64_t idx_batch_stride, float* out_values, int64_t val_batch_stride,
                    void* stream);

/* Accumulated counters per sequence, 8 x uint64 each: steps, blocks visited, blocks scored,
 * blocks pruned, keys scored, keys in the cache, first-wave blocks, second-wave blocks.
 * Synchronous (device to host copy). */
int tdsa_exact_stats(const void* state, size_t state_bytes, int batch, int max_length, int k,
                     int block_size, uint64_t* stats_out);

/*
 * Float64 certified-bound helpers, generic in heads and dims (src/temporal_dsa/
 * certified.py:6-61).  Device pointers to float64.
 * tdsa_block_key_norms: keys [tokens][heads][dim] -> out [ceil(tokens/bs)][heads], the max
 *   L2 norm per block and head (:51-61).
 * tdsa_temporal_radius: out[b] = sum_h block_key_norm[b][h] * (|w_now-w_prev|_h ||q_prev,h||
 *   + |w_now,h| ||q_now,h - q_prev,h||) (:18-48); coeff_workspace holds `heads` doubles.
 * tdsa_relu_index_score: out[t] = sum_h w[h] ReLU(q[h] . keys[t]) (:6-15).
 */
int tdsa_block_key_norms(const double* keys, int tokens, int heads, int dim, int block_size,
                         double* out, void* stream);
int tdsa_temporal_radius(const double* q_now, const double* q_prev, const double* w_now,
                         const double* w_prev, const double* block_key_norm, int heads, int dim,
                         int blocks, double* coeff_workspace, double* out, void* stream);
int tdsa_relu_index_score(const double* q, const double* keys, const double* w, int heads,
                          int dim, int tokens, double* out, void* stream);

/*
 * One-time re-layout of the W_q weight for tdsa_query_project (no reference counterpart:
 * a weight-packing step): w_q [8192][hidden_size] 16-bit (row stride wq_row_stride) ->
 * out [64 heads][ceil(hidden_size/64)][128][64], zero past hidden_size.  out holds
 * tdsa_packed_query_weights_bytes(hidden_size) bytes, 16-byte aligned.
 */
size_t tdsa_packed_query_weights_bytes(int hidden_size);
int tdsa_pack_query_weights(const void* w_q, int64_t wq_row_stride, int hidden_size,
                            void* out, void* stream);

/*
 * The whole decode-step query projection of the sidecar in one launch (replaces the
 * W_q GEMM + tdsa_query_prep pair): reference LightningIndexerSidecar.encode_queries,
 * src/temporal_dsa/sidecar.py:78-87.
 *   q[b]  = RoPE_noninterleaved(16-bit(hidden[b] @ w_q^T)) viewed [64][128], RoPE on the
 *           first rope_dim dims of each head (float32 math, one rounding);
 *   w[b]  = weight_scale * float(hidden[b]) @ w_proj^T  (float32, [64]).
 * hidden [batch][hidden_size] 16-bit, row stride hidden_stride; w_q [8192][hidden_size]
 * 16-bit (nn.Linear weight), row stride wq_row_stride; w_proj [64][hidden_size] float32
 * contiguous; positions [batch] int64.  q [batch][8192] (row stride q_stride), w [batch][64]
 * (row stride w_stride).  qraw: optional [batch][8192] output of the pre-RoPE projection
 * (NULL to skip).  hidden_size a multiple of 8; hidden, w_q, w_proj, q and qraw rows
 * 16-byte aligned.  wq_packed != 0: w_q is the output of tdsa_pack_query_weights
 * (wq_row_stride ignored) -- every tile the kernel streams is then one contiguous block,
 * which HBM serves at full bandwidth; the row-major layout works but reads 128-byte
 * pieces 4 KB apart.  The launch reads w_q and w_proj (constant weights) before it waits on
 * the previous kernel of the stream (programmatic dependent launch), so they must not be
 * written by the kernel issued right before it on the same stream; only hidden and
 * positions may come from that kernel.
 */
int tdsa_query_project(const void* hidden, int64_t hidden_stride, int hidden_size,
                       const void* w_q, int64_t wq_row_stride, int wq_packed,
                       const float* w_proj,
                       const int64_t* positions, void* q, int64_t q_stride, float* w,
                       int64_t w_stride, int dtype, int batch, int rope_dim, float rope_theta,
                       float weight_scale, void* qraw, int64_t qraw_stride, void* stream);

/*
 * Decode-step tail of the sidecar query projection, one launch: RoPE on the first rope_dim
 * dims of every head of the W_q GEMM output, and the float32 head weights
 * w = weight_scale * hidden @ w_proj^T.
 * Replaces: the tail of LightningIndexerSidecar.encode_queries (src/temporal_dsa/
 *   sidecar.py:78-87) with apply_noninterleaved_rope (:10-28).
 * qraw   [batch][64*128] (dtype TDSA_BF16 or TDSA_F16), row stride qraw_stride;
 * hidden [batch][hidden_size] (same dtype), w_proj [64][hidden_size] float32;
 * positions [batch] int64; q [batch][64][128] out (same dtype); w [batch][64] float32 out.
 */
int tdsa_query_prep(const void* qraw, int64_t qraw_stride, const void* hidden,
                    int64_t hidden_stride, int hidden_size, const float* w_proj,
                    const int64_t* positions, void* q, int64_t q_stride, float* w,
                    int64_t w_stride, int dtype, int batch, int rope_dim, float rope_theta,
                    float weight_scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TDSA_H_ */
