// extern "C" entry points of libtdsa: argument checks on the host, then the launchers.
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;

// Device status word.  Lives with the module on every device that loads the library.
__device__ int g_device_status = 0;

int* g_status_ptr[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};
std::mutex g_mutex;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

// Scratch of tdsa_score_topk_noalloc: scores, key histograms and top-k candidates of one
// call, in the module's static device memory (one copy per device that loads the library),
// so that call allocates nothing.  Every call on a device shares it.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u; }

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int device_sm_count(int device) {
  if (device < 0 || device >= kMaxDevices) return 148;
  if (g_sm_count[device] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    g_sm_count[device] = n > 0 ? n : 148;
  }
  return g_sm_count[device];
}

cudaError_t ensure_dynamic_smem(const void* kernel, int bytes) {
  // cudaFuncSetAttribute costs host time on every launch; remember, per device and kernel,
  // the largest dynamic shared memory size already set
  static std::mutex m;
  static std::vector<std::pair<const void*, int>> seen[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices)
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  std::lock_guard<std::mutex> lock(m);
  for (auto& e : seen[dev]) {
    if (e.first != kernel) continue;
    if (e.second >= bytes) return cudaSuccess;
    const cudaError_t rc =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (rc == cudaSuccess) e.second = bytes;
    return rc;
  }
  const cudaError_t rc =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (rc == cudaSuccess) seen[dev].emplace_back(kernel, bytes);
  return rc;
}

int* device_status_ptr() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

// Device address of the static scratch on the current device, looked up once per device
// (the set-up a first call does; it may load the module on that device).
void* noalloc_scratch() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("tdsa_score_topk_noalloc: no usable current device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error(std::string("tdsa_score_topk_noalloc: cudaGetSymbolAddress failed: ") +
                cudaGetErrorString(e));
      return nullptr;
    }
    g_noalloc_ptr[dev] = p;
  }
  return g_noalloc_ptr[dev];
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn)
        return fail(TDSA_ERR_CUDA, "cuTensorMapEncodeTiled entry point not available");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d,
                              s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TDSA_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return TDSA_OK;
}

namespace {

int check_score_args(const void* q, int64_t q_bs, const float* w, int64_t w_bs, const void* k,
                     int64_t k_bs, int64_t k_rs, int dtype, int batch, int length,
                     const float* out, int64_t o_bs, bool check_out = true) {
  if (dtype != TDSA_F32 && dtype != TDSA_F16 && dtype != TDSA_BF16)
    return fail(TDSA_ERR_INVALID, "dtype must be TDSA_F32, TDSA_F16 or TDSA_BF16");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (length < 0) return fail(TDSA_ERR_INVALID, "length must be >= 0");
  if (length == 0) return TDSA_OK;
  if (!q || !w || !k || (check_out && !out))
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (k_rs < kHeadDim) return fail(TDSA_ERR_INVALID, "key row stride must be >= 128");
  if (batch > 1 && (q_bs < kHeads * kHeadDim || w_bs < kHeads ||
                    k_bs < static_cast<int64_t>(length) * k_rs || (check_out && o_bs < length)))
    return fail(TDSA_ERR_INVALID, "batch strides overlap the rows of one sequence");
  if (dtype != TDSA_F32) {
    if (!aligned16(q) || !aligned16(k))
      return fail(TDSA_ERR_ALIGN, "16-bit queries/keys need 16-byte aligned base pointers");
    if (k_rs % 8 || (batch > 1 && (k_bs % 8 || q_bs % 8)))
      return fail(TDSA_ERR_ALIGN, "16-bit strides must be multiples of 8 elements");
  }
  return TDSA_OK;
}

int check_topk_out(void* out_idx, int index_bytes, int64_t idx_bs, const float* out_val,
                   int64_t val_bs, int batch, int k) {
  if (!out_idx) return fail(TDSA_ERR_INVALID, "out_indices is null");
  if (index_bytes != 4 && index_bytes != 8)
    return fail(TDSA_ERR_INVALID, "index_bytes must be 4 or 8");
  if (batch > 1 && (idx_bs < k || (out_val && val_bs < k)))
    return fail(TDSA_ERR_INVALID, "output row strides must be >= k");
  return TDSA_OK;
}

// Shared set-up of the block-structured entry points (16-bit keys only: tcgen05 path).
int block_setup(const void* q, int64_t q_bs, const float* w, int64_t w_bs, const void* k,
                int64_t k_bs, int64_t k_rs, int dtype, int batch, int length, int block_size,
                BlockArgs& a) {
  int rc = check_score_args(q, q_bs, w, w_bs, k, k_bs, k_rs, dtype, batch, length, nullptr, 0,
                            false);
  if (rc) return rc;
  if (dtype == TDSA_F32)
    return fail(TDSA_ERR_UNSUPPORTED, "block kernels take bf16/fp16 queries and keys");
  if (block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128)
    return fail(TDSA_ERR_UNSUPPORTED, "block_size must be 16, 32, 64 or 128");
  a.bs = block_size;
  a.bpt = 128 / block_size;
  a.length = length;
  a.nblocks = (length + block_size - 1) / block_size;
  a.tiles_per_seq = (a.nblocks + a.bpt - 1) / a.bpt;
  a.total_tiles = static_cast<int64_t>(a.tiles_per_seq) * batch;
  a.w = w;
  a.w_stride = w_bs;
  a.status = device_status_ptr();
  if (!a.status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return TDSA_OK;
}

int block_grid(const BlockArgs& a) {
  const int sms = device_sm_count(current_device());
  return static_cast<int>(a.total_tiles < sms ? a.total_tiles : sms);
}

}  // namespace
}  // namespace tdsa

using namespace tdsa;

extern "C" {

const char* tdsa_version(void) { return "tdsa-b200 0.1.0 sm_100a"; }

const char* tdsa_last_error(void) { return g_last_error.c_str(); }

int tdsa_device_status(int* status_out, int reset) {
  if (!status_out) return fail(TDSA_ERR_INVALID, "status_out is null");
  TDSA_CUDA_CHECK(cudaMemcpyFromSymbol(status_out, g_device_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    TDSA_CUDA_CHECK(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)));
  }
  return TDSA_OK;
}

int tdsa_score_dense(const void* queries, int64_t q_batch_stride, const float* weights,
                     int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                     int64_t k_row_stride, int dtype, int batch, int length, float* scores,
                     int64_t s_batch_stride, void* stream) {
  int rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                            k_batch_stride, k_row_stride, dtype, batch, length, scores,
                            s_batch_stride);
  if (rc || length == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  if (dtype == TDSA_F32) {
    const float* q = static_cast<const float*>(queries);
    const float* k = static_cast<const float*>(keys);
    // tensor cores (3 x TF32) when the layout admits TMA, else exact FP32 FMAs
    if (score_dense_tf32_supported(q, q_batch_stride, k, k_batch_stride, k_row_stride, batch))
      return launch_score_dense_tf32(q, q_batch_stride, weights, w_batch_stride, k,
                                     k_batch_stride, k_row_stride, batch, length, scores,
                                     s_batch_stride, st, status);
    return launch_score_dense_f32(q, q_batch_stride, weights, w_batch_stride, k,
                                  k_batch_stride, k_row_stride, batch, length, scores,
                                  s_batch_stride, st);
  }
  return launch_score_dense_tc(queries, q_batch_stride, weights, w_batch_stride, keys,
                               k_batch_stride, k_row_stride, dtype, batch, length, scores,
                               s_batch_stride, st, status);
}

// Bytes of the key histograms that let a few unsorted rows of one segment take the cluster
// top-k (several SMs per row) instead of one CTA per row segment; 0 when it does not apply.
static size_t topk_row_hist_bytes(int batch, int length) {
  return topk_cluster_rows(batch, length) > 1 ? static_cast<size_t>(batch) * kKeyHistBins * 4
                                              : 0;
}

size_t tdsa_topk_workspace_bytes(int batch, int length, int k) {
  if (batch < 1 || length < 1 || k < 1 || k > length) return 0;
  return std::max(topk_workspace_bytes(batch, length, k), topk_row_hist_bytes(batch, length));
}

int tdsa_topk(const float* scores, int64_t s_batch_stride, int batch, int length, int k,
              int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
              float* out_values, int64_t val_batch_stride, void* workspace,
              size_t workspace_bytes, void* stream) {
  if (!scores) return fail(TDSA_ERR_INVALID, "scores is null");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (batch > 1 && s_batch_stride < length)
    return fail(TDSA_ERR_INVALID, "score row stride must be >= length");
  int rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values,
                          val_batch_stride, batch, k);
  if (rc) return rc;
  const size_t hist_bytes = topk_row_hist_bytes(batch, length);
  if (!sorted && hist_bytes && workspace && workspace_bytes >= hist_bytes &&
      (reinterpret_cast<uintptr_t>(workspace) & 15u) == 0 && topk_check(length, k, 0) == 0) {
    // few unsorted rows: histogram each row over several CTAs, then the cluster top-k
    uint32_t* hist = static_cast<uint32_t*>(workspace);
    rc = launch_row_hist_parts(scores, batch > 1 ? s_batch_stride : length, batch, length, hist,
                               static_cast<cudaStream_t>(stream));
    if (rc) return rc;
    return launch_topk(scores, s_batch_stride, nullptr, 0, batch, length, k, 0, out_indices,
                       index_bytes, idx_batch_stride, out_values, val_batch_stride, nullptr, 0,
                       static_cast<cudaStream_t>(stream), nullptr, hist);
  }
  return launch_topk(scores, s_batch_stride, nullptr, 0, batch, length, k, sorted ? 1 : 0,
                     out_indices, index_bytes, idx_batch_stride, out_values, val_batch_stride,
                     workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int tdsa_merge_topk(const float* cand_values, const int32_t* cand_indices,
                    int64_t cand_batch_stride, int batch, int count, int k, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* stream) {
  if (!cand_values || !cand_indices) return fail(TDSA_ERR_INVALID, "null candidate pointer");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (count > kTopkSegment)
    return fail(TDSA_ERR_UNSUPPORTED, "merge takes at most 32768 candidates per row");
  if (batch > 1 && cand_batch_stride < count)
    return fail(TDSA_ERR_INVALID, "candidate row stride must be >= count");
  int rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values,
                          val_batch_stride, batch, k);
  if (rc) return rc;
  return launch_topk(cand_values, cand_batch_stride, cand_indices, cand_batch_stride, batch,
                     count, k, sorted ? 1 : 0, out_indices, index_bytes, idx_batch_stride,
                     out_values, val_batch_stride, nullptr, 0,
                     static_cast<cudaStream_t>(stream));
}

int tdsa_topk_levels(int batch, int length, int k, int with_key_hist) {
  if (batch < 1 || length < 1 || k < 1 || k > length) return 0;
  return topk_levels(batch, length, k, with_key_hist);
}

size_t tdsa_key_hist_bytes(int batch, int length) {
  if (batch < 1 || length < 1) return 0;
  const size_t segs = (static_cast<size_t>(length) + kTopkSegment - 1) / kTopkSegment;
  return static_cast<size_t>(batch) * segs * kKeyHistBins * 4;
}

size_t tdsa_score_topk_workspace_bytes(int batch, int length, int k) {
  if (batch < 1 || length < 1 || k < 1 || k > length) return 0;
  const size_t scores = (static_cast<size_t>(batch) * length * 4 + 255) & ~size_t(255);
  return scores + tdsa_key_hist_bytes(batch, length) + topk_workspace_bytes(batch, length, k);
}

int tdsa_score_topk(const void* queries, int64_t q_batch_stride, const float* weights,
                    int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                    int64_t k_row_stride, int dtype, int batch, int length, int k, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (length < 1) return fail(TDSA_ERR_INVALID, "length must be >= 1");
  int rc = topk_check(length, k, sorted);
  if (rc) return rc;
  rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values, val_batch_stride,
                      batch, k);
  if (rc) return rc;
  const size_t need = tdsa_score_topk_workspace_bytes(batch, length, k);
  if (!workspace || workspace_bytes < need)
    return fail(TDSA_ERR_WORKSPACE, "score_topk workspace missing or too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* scores = reinterpret_cast<float*>(ws);
  const size_t score_bytes = (static_cast<size_t>(batch) * length * 4 + 255) & ~size_t(255);
  const size_t hist_bytes = tdsa_key_hist_bytes(batch, length);
  uint32_t* hist = reinterpret_cast<uint32_t*>(ws + score_bytes);
  // the score kernel's key histograms (one per 32768-key segment) let the top-k skip its
  // first passes (16-bit keys)
  const bool use_hist = dtype != TDSA_F32;
  if (use_hist) {
    TDSA_CUDA_CHECK(cudaMemsetAsync(hist, 0, hist_bytes, st));
    rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                          k_batch_stride, k_row_stride, dtype, batch, length, scores, length);
    if (rc) return rc;
    int* status = device_status_ptr();
    if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
    rc = launch_score_dense_tc(queries, q_batch_stride, weights, w_batch_stride, keys,
                               k_batch_stride, k_row_stride, dtype, batch, length, scores,
                               length, st, status, hist);
  } else {
    rc = tdsa_score_dense(queries, q_batch_stride, weights, w_batch_stride, keys,
                          k_batch_stride, k_row_stride, dtype, batch, length, scores, length,
                          stream);
  }
  if (rc) return rc;
  return launch_topk(scores, length, nullptr, 0, batch, length, k, sorted ? 1 : 0, out_indices,
                     index_bytes, idx_batch_stride, out_values, val_batch_stride,
                     ws + score_bytes + hist_bytes, workspace_bytes - score_bytes - hist_bytes,
                     st, nullptr, use_hist ? hist : nullptr);
}

int tdsa_score_topk_noalloc(const void* queries, int64_t q_batch_stride, const float* weights,
                            int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                            int64_t k_row_stride, int dtype, int batch, int length, int k,
                            int sorted, void* out_indices, int index_bytes,
                            int64_t idx_batch_stride, float* out_values,
                            int64_t val_batch_stride, void* stream) {
  // Sizes are checked before anything touches the device.
  if (batch < 1 || length < 1 || k < 1 || k > length)
    return fail(TDSA_ERR_INVALID, "tdsa_score_topk_noalloc: needs batch >= 1 and 1 <= k <= length");
  const size_t need = tdsa_score_topk_workspace_bytes(batch, length, k);
  if (need > kNoAllocScratchBytes)
    return fail(TDSA_ERR_UNSUPPORTED,
                "tdsa_score_topk_noalloc: this call needs " + std::to_string(need) +
                    " bytes of scratch; the static scratch holds " +
                    std::to_string(kNoAllocScratchBytes) +
                    " (tdsa_score_topk_workspace_bytes(batch, length, k) must not exceed it)");
  void* scratch = noalloc_scratch();
  if (!scratch) return TDSA_ERR_CUDA;
  // The existing path, with the static scratch as its workspace; it zeroes the key
  // histogram region itself (cudaMemsetAsync) before the score kernel adds to it.
  return tdsa_score_topk(queries, q_batch_stride, weights, w_batch_stride, keys,
                         k_batch_stride, k_row_stride, dtype, batch, length, k, sorted,
                         out_indices, index_bytes, idx_batch_stride, out_values,
                         val_batch_stride, scratch, kNoAllocScratchBytes, stream);
}

int tdsa_score_dense_hist(const void* queries, int64_t q_batch_stride, const float* weights,
                          int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                          int64_t k_row_stride, int dtype, int batch, int length, float* scores,
                          int64_t s_batch_stride, uint32_t* key_hist, void* stream) {
  int rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                            k_batch_stride, k_row_stride, dtype, batch, length, scores,
                            s_batch_stride);
  if (rc || length == 0) return rc;
  if (dtype == TDSA_F32) return fail(TDSA_ERR_UNSUPPORTED, "key histograms need 16-bit keys");
  if (!key_hist) return fail(TDSA_ERR_INVALID, "key_hist is null");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return launch_score_dense_tc(queries, q_batch_stride, weights, w_batch_stride, keys,
                               k_batch_stride, k_row_stride, dtype, batch, length, scores,
                               s_batch_stride, static_cast<cudaStream_t>(stream), status,
                               key_hist);
}

int tdsa_score_dense_trace(const void* queries, int64_t q_batch_stride, const float* weights,
                           int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                           int64_t k_row_stride, int dtype, int batch, int length,
                           float* scores, int64_t s_batch_stride, uint32_t* key_hist,
                           uint16_t* trace, int64_t trace_batch_stride, void* stream) {
  int rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                            k_batch_stride, k_row_stride, dtype, batch, length, scores,
                            s_batch_stride);
  if (rc || length == 0) return rc;
  if (dtype == TDSA_F32) return fail(TDSA_ERR_UNSUPPORTED, "score traces need 16-bit keys");
  if (!trace) return fail(TDSA_ERR_INVALID, "trace is null");
  if (batch > 1 && trace_batch_stride < length)
    return fail(TDSA_ERR_INVALID, "trace batch stride must be >= length");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return launch_score_dense_tc(queries, q_batch_stride, weights, w_batch_stride, keys,
                               k_batch_stride, k_row_stride, dtype, batch, length, scores,
                               s_batch_stride, static_cast<cudaStream_t>(stream), status,
                               key_hist, trace, trace_batch_stride);
}

int tdsa_topk_hist(const float* scores, int64_t s_batch_stride, int batch, int length, int k,
                   int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
                   float* out_values, int64_t val_batch_stride, uint32_t* key_hist,
                   void* stream) {
  if (!scores || !key_hist) return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (batch > 1 && s_batch_stride < length)
    return fail(TDSA_ERR_INVALID, "score row stride must be >= length");
  if (length > kTopkSegment)
    return fail(TDSA_ERR_UNSUPPORTED, "tdsa_topk_hist takes rows of at most 32768 keys");
  int rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values,
                          val_batch_stride, batch, k);
  if (rc) return rc;
  return launch_topk(scores, s_batch_stride, nullptr, 0, batch, length, k, sorted ? 1 : 0,
                     out_indices, index_bytes, idx_batch_stride, out_values, val_batch_stride,
                     nullptr, 0, static_cast<cudaStream_t>(stream), nullptr, key_hist);
}

int tdsa_topk_hist_ws(const float* scores, int64_t s_batch_stride, int batch, int length,
                      int k, int sorted, void* out_indices, int index_bytes,
                      int64_t idx_batch_stride, float* out_values, int64_t val_batch_stride,
                      uint32_t* key_hist, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!scores || !key_hist) return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (batch > 1 && s_batch_stride < length)
    return fail(TDSA_ERR_INVALID, "score row stride must be >= length");
  int rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values,
                          val_batch_stride, batch, k);
  if (rc) return rc;
  return launch_topk(scores, s_batch_stride, nullptr, 0, batch, length, k, sorted ? 1 : 0,
                     out_indices, index_bytes, idx_batch_stride, out_values, val_batch_stride,
                     workspace, workspace_bytes, static_cast<cudaStream_t>(stream), nullptr,
                     key_hist);
}

int tdsa_query_prep(const void* qraw, int64_t qraw_stride, const void* hidden,
                    int64_t hidden_stride, int hidden_size, const float* w_proj,
                    const int64_t* positions, void* q, int64_t q_stride, float* w,
                    int64_t w_stride, int dtype, int batch, int rope_dim, float rope_theta,
                    float weight_scale, void* stream) {
  if (!qraw || !hidden || !w_proj || !positions || !q || !w)
    return fail(TDSA_ERR_INVALID, "null pointer");
  if (dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_INVALID, "query_prep takes TDSA_BF16 or TDSA_F16");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (hidden_size < 1 || hidden_size > 16384)
    return fail(TDSA_ERR_UNSUPPORTED, "hidden_size must be in [1, 16384]");
  if (rope_dim < 0 || rope_dim > kHeadDim || rope_dim % 2)
    return fail(TDSA_ERR_INVALID, "rope_dim must be even and <= 128");
  if (batch > 1 && (qraw_stride < kHeads * kHeadDim || q_stride < kHeads * kHeadDim ||
                    hidden_stride < hidden_size || w_stride < kHeads))
    return fail(TDSA_ERR_INVALID, "row strides overlap");
  return launch_qprep(qraw, qraw_stride, hidden, hidden_stride, hidden_size, w_proj, positions,
                      q, q_stride, w, w_stride, dtype, batch, rope_dim, rope_theta,
                      weight_scale, static_cast<cudaStream_t>(stream));
}

int tdsa_hadamard128(const void* in, int64_t in_row_stride, int64_t rows, int dtype, void* out,
                     int64_t out_row_stride, void* stream) {
  if (rows < 0) return fail(TDSA_ERR_INVALID, "rows must be >= 0");
  if (rows == 0) return TDSA_OK;
  if (!in || !out) return fail(TDSA_ERR_INVALID, "null pointer");
  if (dtype != TDSA_F32 && dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_INVALID, "unknown dtype");
  if (rows > 1 && (in_row_stride < 128 || out_row_stride < 128))
    return fail(TDSA_ERR_INVALID, "row strides must be >= 128");
  return launch_hadamard128(in, in_row_stride, rows, dtype, out, out_row_stride,
                            static_cast<cudaStream_t>(stream));
}

int tdsa_select_quantize(const void* in, int64_t in_row_stride, int64_t rows, int width,
                         int dtype, const int8_t* keep, int bits, double scale,
                         uint32_t* absmax_word, void* out, int64_t out_row_stride,
                         void* stream) {
  if (rows < 0 || width < 1) return fail(TDSA_ERR_INVALID, "rows >= 0 and width >= 1");
  if (rows == 0) return TDSA_OK;
  if (!in || !out) return fail(TDSA_ERR_INVALID, "null pointer");
  if (dtype != TDSA_F32 && dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_INVALID, "unknown dtype");
  if (bits != 0 && bits != 2 && bits != 4 && bits != 8)
    return fail(TDSA_ERR_INVALID, "bits must be one of 2, 4, 8 (or 0: no quantization)");
  if (bits && scale <= 0.0 && !absmax_word)
    return fail(TDSA_ERR_INVALID, "a computed scale needs absmax_word");
  if (rows > 1 && (in_row_stride < width || out_row_stride < width))
    return fail(TDSA_ERR_INVALID, "row strides must be >= width");
  return launch_select_quantize(in, in_row_stride, rows, width, dtype, keep, bits, scale,
                                absmax_word, out, out_row_stride,
                                static_cast<cudaStream_t>(stream));
}

int tdsa_selftest_bounded_wait(long long limit_cycles, void* stream) {
  if (limit_cycles < 0 || limit_cycles > 4000000000LL)
    return fail(TDSA_ERR_INVALID, "limit_cycles must be in [0, 4e9]");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return launch_bounded_wait_selftest(limit_cycles, static_cast<cudaStream_t>(stream), status);
}

size_t tdsa_packed_query_weights_bytes(int hidden_size) {
  if (hidden_size < 8 || hidden_size > 65536 || hidden_size % 8) return 0;
  return packed_wq_bytes(hidden_size);
}

int tdsa_pack_query_weights(const void* w_q, int64_t wq_row_stride, int hidden_size,
                            void* out, void* stream) {
  if (!w_q || !out) return fail(TDSA_ERR_INVALID, "null pointer");
  if (hidden_size < 8 || hidden_size > 65536 || hidden_size % 8)
    return fail(TDSA_ERR_UNSUPPORTED, "hidden_size must be a multiple of 8 in [8, 65536]");
  if (wq_row_stride < hidden_size) return fail(TDSA_ERR_INVALID, "row stride < hidden_size");
  if (!aligned16(out)) return fail(TDSA_ERR_ALIGN, "out must be 16-byte aligned");
  return launch_pack_wq(w_q, wq_row_stride, hidden_size, out, static_cast<cudaStream_t>(stream));
}

size_t tdsa_policy_state_bytes(int batch, int k, int max_blocks) {
  if (batch < 1 || k < 1 || max_blocks < 1) return 0;
  return policy_state_bytes(batch, k, max_blocks, nullptr);
}

int tdsa_policy_state_offsets(int batch, int k, int max_blocks, int64_t* offsets8) {
  if (!offsets8 || batch < 1 || k < 1 || max_blocks < 1)
    return fail(TDSA_ERR_INVALID, "bad policy state shape");
  policy_state_bytes(batch, k, max_blocks, offsets8);
  return TDSA_OK;
}

namespace {
struct PolicyWs {
  size_t masked, cmax, base_new, approx, topk, total;
};
PolicyWs policy_ws(int batch, int length, int k, int nbc) {
  const size_t B = static_cast<size_t>(batch);
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  PolicyWs w;
  size_t o = 0;
  w.masked = o;   o = up(o + B * length * 4);
  w.cmax = o;     o = up(o + B * nbc * 4);
  w.base_new = o; o = up(o + B * k * 4);
  w.approx = o;   o = up(o + B * k * 4);
  w.topk = o;     o = up(o + topk_workspace_bytes(batch, length, k));
  w.total = o;
  return w;
}

int policy_checks(const void* state, size_t state_bytes, const float* scores, int64_t s_stride,
                  int batch, int length, int k, int block_size, int max_blocks) {
  if (!state || !scores) return fail(TDSA_ERR_INVALID, "null pointer");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (block_size < 1 || block_size > 128 || (block_size & (block_size - 1)))
    return fail(TDSA_ERR_UNSUPPORTED, "the policy takes power-of-two block sizes up to 128");
  if (k < 1 || k > length) return fail(TDSA_ERR_INVALID, "K cannot exceed the current length");
  if (k > 2048) return fail(TDSA_ERR_UNSUPPORTED, "the policy takes k <= 2048");
  if (length > 131072) return fail(TDSA_ERR_UNSUPPORTED, "the policy takes length <= 131072");
  const int nb = (length + block_size - 1) / block_size;
  if (max_blocks < nb || max_blocks > 4096)
    return fail(TDSA_ERR_INVALID, "need ceil(length/block_size) <= max_blocks <= 4096");
  if (batch > 1 && s_stride < length)
    return fail(TDSA_ERR_INVALID, "score row stride must be >= length");
  if (state_bytes < policy_state_bytes(batch, k, max_blocks, nullptr))
    return fail(TDSA_ERR_WORKSPACE, "policy state buffer too small");
  return TDSA_OK;
}
}  // namespace

size_t tdsa_policy_workspace_bytes(int batch, int max_length, int k, int max_blocks) {
  if (batch < 1 || max_length < 1 || k < 1 || k > max_length || max_blocks < 1) return 0;
  return policy_ws(batch, max_length, k, max_blocks).total;
}

int tdsa_policy_init(void* state, size_t state_bytes, const float* scores, int64_t s_stride,
                     int batch, int length, int k, int block_size, int max_blocks,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = policy_checks(state, state_bytes, scores, s_stride, batch, length, k, block_size,
                         max_blocks);
  if (rc) return rc;
  const PolicyWs w = policy_ws(batch, length, k, max_blocks);
  if (!workspace || workspace_bytes < w.total)
    return fail(TDSA_ERR_WORKSPACE, "policy workspace missing or too small");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  return launch_policy(1, static_cast<uint8_t*>(state), batch, k, max_blocks, scores,
                       batch > 1 ? s_stride : length, nullptr, 0, length, length, block_size,
                       nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0,
                       reinterpret_cast<int32_t*>(ws + w.base_new), nullptr, ws + w.topk,
                       w.total - w.topk, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}

int tdsa_policy_step(void* state, size_t state_bytes, const float* scores, int64_t s_stride,
                     const float* verifier_scores, int64_t v_stride, int batch, int length,
                     int previous_length, int k, int block_size, int max_blocks,
                     const tdsa_policy* policy, int history_mode, int full_refresh,
                     const tdsa_rescue* rescue, void* workspace, size_t workspace_bytes,
                     uint32_t* evaluated_bits, int64_t bits_stride, uint8_t* block_flags,
                     int32_t* ranking, double* stats, void* stream) {
  int rc = policy_checks(state, state_bytes, scores, s_stride, batch, length, k, block_size,
                         max_blocks);
  if (rc) return rc;
  if (!policy || !evaluated_bits || !block_flags || !stats)
    return fail(TDSA_ERR_INVALID, "null policy, evaluated_bits, block_flags or stats");
  if (history_mode != 0 && history_mode != 1)
    return fail(TDSA_ERR_INVALID, "history_mode must be 0 (own) or 1 (teacher)");
  if (policy->order < TDSA_ORDER_ADDRESS || policy->order > TDSA_ORDER_ORACLE_CURRENT)
    return fail(TDSA_ERR_INVALID, "unknown block order");
  if (policy->order == TDSA_ORDER_BUCKET && policy->buckets < 1)
    return fail(TDSA_ERR_INVALID, "bucket order needs buckets >= 1");
  if (policy->risk_model != TDSA_RISK_LAST_MAX && policy->risk_model != TDSA_RISK_EMA)
    return fail(TDSA_ERR_INVALID, "unknown risk model");
  if (rescue) {
    if (!verifier_scores) return fail(TDSA_ERR_INVALID, "a rescue step needs verifier scores");
    if (history_mode != 0) return fail(TDSA_ERR_INVALID, "the verifier step runs in own mode");
    if (!rescue->use_threshold && !(rescue->rescue_fraction >= 0 && rescue->rescue_fraction <= 1))
      return fail(TDSA_ERR_INVALID, "rescue_fraction must be in [0, 1]");
    if (batch > 1 && v_stride < length)
      return fail(TDSA_ERR_INVALID, "verifier score row stride must be >= length");
  }
  if (previous_length < 0) return fail(TDSA_ERR_INVALID, "previous_length must be >= 0");
  if (bits_stride < (length + 31) / 32 && batch > 1)
    return fail(TDSA_ERR_INVALID, "bits_stride must be >= ceil(length / 32)");
  if (policy_decide_smem_bytes(length, block_size, k) > 227 * 1024)
    return fail(TDSA_ERR_UNSUPPORTED, "this length / block size / k needs too much shared memory");
  const PolicyWs w = policy_ws(batch, length, k, max_blocks);
  if (!workspace || workspace_bytes < w.total)
    return fail(TDSA_ERR_WORKSPACE, "policy workspace missing or too small");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  return launch_policy(
      0, static_cast<uint8_t*>(state), batch, k, max_blocks, scores,
      batch > 1 ? s_stride : length, rescue ? verifier_scores : nullptr,
      batch > 1 ? v_stride : length, length, previous_length, block_size, policy, history_mode,
      full_refresh, rescue, reinterpret_cast<float*>(ws + w.masked),
      reinterpret_cast<float*>(ws + w.cmax), block_flags, ranking, evaluated_bits,
      batch > 1 ? bits_stride : (length + 31) / 32, reinterpret_cast<int32_t*>(ws + w.base_new),
      reinterpret_cast<int32_t*>(ws + w.approx), ws + w.topk, w.total - w.topk, stats, status,
      static_cast<cudaStream_t>(stream));
}

int tdsa_key_append(const void* hidden, int64_t hidden_stride, int hidden_size,
                    const void* w_k, int64_t wk_row_stride, const float* ln_weight,
                    const float* ln_bias, float eps, const int64_t* positions,
                    const int64_t* slots, void* cache, int64_t cache_batch_stride,
                    int64_t cache_row_stride, int64_t cache_rows, int dtype, int batch,
                    int rope_dim, float rope_theta, void* stream) {
  if (!hidden || !w_k || !positions || !cache) return fail(TDSA_ERR_INVALID, "null pointer");
  if (dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_INVALID, "key_append takes TDSA_BF16 or TDSA_F16");
  if (batch < 1 || batch > (1 << 20)) return fail(TDSA_ERR_INVALID, "batch must be in [1, 2^20]");
  if (hidden_size < 8 || hidden_size % 8)
    return fail(TDSA_ERR_UNSUPPORTED, "hidden_size must be a positive multiple of 8");
  if (rope_dim < 0 || rope_dim > kHeadDim || rope_dim % 2)
    return fail(TDSA_ERR_INVALID, "rope_dim must be even and in [0, 128]");
  if (!(eps >= 0.f)) return fail(TDSA_ERR_INVALID, "eps must be >= 0");
  if (wk_row_stride < hidden_size || (batch > 1 && hidden_stride < hidden_size))
    return fail(TDSA_ERR_INVALID, "row strides must be >= hidden_size");
  if (cache_rows < 1 || cache_row_stride < kHeadDim ||
      (batch > 1 && cache_batch_stride < cache_rows * cache_row_stride))
    return fail(TDSA_ERR_INVALID, "cache strides do not hold [batch][cache_rows][128]");
  if (!aligned16(hidden) || !aligned16(w_k) || wk_row_stride % 8 ||
      (batch > 1 && hidden_stride % 8))
    return fail(TDSA_ERR_ALIGN, "hidden and w_k need 16-byte aligned rows");
  if (reinterpret_cast<uintptr_t>(cache) % 2)
    return fail(TDSA_ERR_ALIGN, "cache must be 2-byte aligned");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return launch_key_append(hidden, hidden_stride, hidden_size, w_k, wk_row_stride, ln_weight,
                           ln_bias, eps, positions, slots, cache, cache_batch_stride,
                           cache_row_stride, cache_rows, dtype, batch, rope_dim, rope_theta,
                           status, static_cast<cudaStream_t>(stream));
}

int tdsa_query_project(const void* hidden, int64_t hidden_stride, int hidden_size,
                       const void* w_q, int64_t wq_row_stride, int wq_packed,
                       const float* w_proj,
                       const int64_t* positions, void* q, int64_t q_stride, float* w,
                       int64_t w_stride, int dtype, int batch, int rope_dim, float rope_theta,
                       float weight_scale, void* qraw, int64_t qraw_stride, void* stream) {
  if (!hidden || !w_q || !w_proj || !positions || !q || !w)
    return fail(TDSA_ERR_INVALID, "null pointer");
  if (dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_INVALID, "query_project takes TDSA_BF16 or TDSA_F16");
  if (batch < 1 || batch > 65535 * 256)
    return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535 * 256]");
  if (hidden_size < 8 || hidden_size > 65536 || hidden_size % 8)
    return fail(TDSA_ERR_UNSUPPORTED, "hidden_size must be a multiple of 8 in [8, 65536]");
  if (rope_dim < 0 || rope_dim > kHeadDim || rope_dim % 2)
    return fail(TDSA_ERR_INVALID, "rope_dim must be even and <= 128");
  if ((!wq_packed && wq_row_stride < hidden_size) ||
      (batch > 1 && hidden_stride < hidden_size))
    return fail(TDSA_ERR_INVALID, "row strides overlap");
  if (batch > 1 && (q_stride < kHeads * kHeadDim || w_stride < kHeads ||
                    (qraw && qraw_stride < kHeads * kHeadDim)))
    return fail(TDSA_ERR_INVALID, "row strides overlap");
  if (!aligned16(hidden) || !aligned16(w_q) || !aligned16(w_proj) ||
      (!wq_packed && wq_row_stride % 8) ||
      (batch > 1 && hidden_stride % 8))
    return fail(TDSA_ERR_ALIGN, "hidden, w_q and w_proj need 16-byte aligned rows (TMA)");
  if (!aligned16(q) || (qraw && !aligned16(qraw)) ||
      (batch > 1 && (q_stride % 8 || (qraw && qraw_stride % 8))))
    return fail(TDSA_ERR_ALIGN, "q and qraw need 16-byte aligned rows");
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "device status word not available");
  return launch_query_project(hidden, hidden_stride, hidden_size, w_q, wq_row_stride,
                              wq_packed ? 1 : 0, w_proj,
                              positions, q, q_stride, w, w_stride, dtype, batch, rope_dim,
                              rope_theta, weight_scale, qraw, qraw_stride,
                              static_cast<cudaStream_t>(stream), status);
}

int tdsa_h8_block_max(const void* queries, int64_t q_batch_stride, const float* weights,
                      int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                      int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                      const int32_t* selected_heads, const int8_t* cold_blocks,
                      float* partial, int64_t p_batch_stride, float* block_max,
                      int64_t bm_batch_stride, void* stream) {
  if (length < 1) return fail(TDSA_ERR_INVALID, "length must be >= 1");
  BlockArgs a;
  int rc = block_setup(queries, q_batch_stride, weights, w_batch_stride, keys, k_batch_stride,
                       k_row_stride, dtype, batch, length, block_size, a);
  if (rc) return rc;
  if (!selected_heads || !cold_blocks || !partial || !block_max)
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch > 1 && (p_batch_stride < length || bm_batch_stride < a.nblocks))
    return fail(TDSA_ERR_INVALID, "output row strides too small");
  a.mask = cold_blocks;
  a.mask_stride = bm_batch_stride;
  a.selected = selected_heads;
  a.out = partial;
  a.out_stride = p_batch_stride;
  a.block_max = block_max;
  a.bm_stride = bm_batch_stride;
  return launch_score_blocks(kModeH8, queries, q_batch_stride, keys, k_batch_stride,
                             k_row_stride, dtype, batch, a, block_grid(a),
                             static_cast<cudaStream_t>(stream));
}

int tdsa_masked_dense(const void* queries, int64_t q_batch_stride, const float* weights,
                      int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                      int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                      const int8_t* keep_blocks, int64_t keep_batch_stride, float* scores,
                      int64_t s_batch_stride, void* stream) {
  if (length < 1) return fail(TDSA_ERR_INVALID, "length must be >= 1");
  BlockArgs a;
  int rc = block_setup(queries, q_batch_stride, weights, w_batch_stride, keys, k_batch_stride,
                       k_row_stride, dtype, batch, length, block_size, a);
  if (rc) return rc;
  if (!keep_blocks || !scores) return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch > 1 && (s_batch_stride < length || keep_batch_stride < a.nblocks))
    return fail(TDSA_ERR_INVALID, "row strides too small");
  a.mask = keep_blocks;
  a.mask_stride = keep_batch_stride;
  a.out = scores;
  a.out_stride = s_batch_stride;
  return launch_score_blocks(kModeMasked, queries, q_batch_stride, keys, k_batch_stride,
                             k_row_stride, dtype, batch, a, block_grid(a),
                             static_cast<cudaStream_t>(stream));
}

int tdsa_two_pass(const void* queries, int64_t q_batch_stride, const float* weights,
                  int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                  int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                  const int32_t* selected_heads, const int8_t* direct_blocks,
                  const float* threshold, float* scores, int64_t s_batch_stride,
                  int8_t* accepted, float* block_max, int64_t bm_batch_stride, void* stream) {
  if (length < 1) return fail(TDSA_ERR_INVALID, "length must be >= 1");
  BlockArgs a;
  int rc = block_setup(queries, q_batch_stride, weights, w_batch_stride, keys, k_batch_stride,
                       k_row_stride, dtype, batch, length, block_size, a);
  if (rc) return rc;
  if (!selected_heads || !direct_blocks || !threshold || !scores || !accepted || !block_max)
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch > 1 && (s_batch_stride < length || bm_batch_stride < a.nblocks))
    return fail(TDSA_ERR_INVALID, "row strides too small");
  // 1. the 8-head probe maximum of every cold (non-direct) block; no partial scores kept
  a.mask = direct_blocks;
  a.mask_stride = bm_batch_stride;
  a.mask_invert = 1;
  a.selected = selected_heads;
  a.block_max = block_max;
  a.bm_stride = bm_batch_stride;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = launch_score_blocks(kModeH8, queries, q_batch_stride, keys, k_batch_stride, k_row_stride,
                           dtype, batch, a, block_grid(a), st);
  if (rc) return rc;
  // 2. dense scores of the accepted blocks (direct, or probe max >= threshold), the
  // acceptance written per block; rejected blocks are not read
  BlockArgs m = a;
  m.mask_invert = 0;
  m.selected = nullptr;
  m.block_max = nullptr;
  m.accept_max = block_max;
  m.threshold = threshold;
  m.accepted = accepted;
  m.out = scores;
  m.out_stride = s_batch_stride;
  return launch_score_blocks(kModeMasked, queries, q_batch_stride, keys, k_batch_stride,
                             k_row_stride, dtype, batch, m, block_grid(m), st);
}

int tdsa_progressive_h8(const void* queries, int64_t q_batch_stride, const float* weights,
                        int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                        int64_t k_row_stride, int dtype, int batch, int length, int block_size,
                        const int32_t* selected_heads, const int32_t* remaining_heads,
                        const int8_t* direct_blocks, const float* threshold, float* scores,
                        int64_t s_batch_stride, int8_t* accepted, float* block_max,
                        int64_t bm_batch_stride, void* stream) {
  if (length < 1) return fail(TDSA_ERR_INVALID, "length must be >= 1");
  BlockArgs a;
  int rc = block_setup(queries, q_batch_stride, weights, w_batch_stride, keys, k_batch_stride,
                       k_row_stride, dtype, batch, length, block_size, a);
  if (rc) return rc;
  if (!selected_heads || !direct_blocks || !threshold || !scores || !accepted || !block_max)
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch > 1 && (s_batch_stride < length || bm_batch_stride < a.nblocks))
    return fail(TDSA_ERR_INVALID, "row strides too small");
  a.mask = direct_blocks;
  a.mask_stride = bm_batch_stride;
  a.selected = selected_heads;
  a.remaining = remaining_heads;
  a.threshold = threshold;
  a.out = scores;
  a.out_stride = s_batch_stride;
  a.block_max = block_max;
  a.accepted = accepted;
  a.bm_stride = bm_batch_stride;
  return launch_score_blocks(kModeProgressive, queries, q_batch_stride, keys, k_batch_stride,
                             k_row_stride, dtype, batch, a, block_grid(a),
                             static_cast<cudaStream_t>(stream));
}

int tdsa_compact_blocks(const float* scores, int64_t s_batch_stride, const int8_t* accepted,
                        int64_t a_batch_stride, int batch, int length, int block_size,
                        float* out_scores, int32_t* out_indices, int64_t out_batch_stride,
                        int32_t* out_count, void* stream) {
  if (!scores || !accepted || !out_scores || !out_indices || !out_count)
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (batch < 1 || batch > 65535 || length < 1 || block_size < 1)
    return fail(TDSA_ERR_INVALID, "bad batch, length or block size");
  if (batch > 1 && (s_batch_stride < length || out_batch_stride < length ||
                    a_batch_stride < (length + block_size - 1) / block_size))
    return fail(TDSA_ERR_INVALID, "row strides too small");
  return launch_compact_blocks(scores, s_batch_stride, accepted, a_batch_stride, batch, length,
                               block_size, out_scores, out_indices, out_batch_stride, out_count,
                               static_cast<cudaStream_t>(stream));
}

int tdsa_sketch_keys(const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                     int batch, int first, int length, int8_t* sketch,
                     int64_t sketch_batch_stride, float* scales, void* bounds,
                     int64_t scale_batch_stride, void* stream) {
  if (!keys || !sketch || !scales || !bounds) return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (dtype != TDSA_BF16 && dtype != TDSA_F16)
    return fail(TDSA_ERR_UNSUPPORTED, "the key sketch takes bf16/fp16 keys");
  if (batch < 1 || batch > 65535 || first < 0 || first > length)
    return fail(TDSA_ERR_INVALID, "need batch in [1, 65535] and 0 <= first <= length");
  if (k_row_stride < kHeadDim || (batch > 1 && (k_batch_stride < static_cast<int64_t>(length) * k_row_stride ||
                                                sketch_batch_stride < static_cast<int64_t>(length) * kHeadDim ||
                                                scale_batch_stride < length)))
    return fail(TDSA_ERR_INVALID, "strides overlap the rows of one sequence");
  if (!aligned16(keys) || k_row_stride % 8 || (batch > 1 && k_batch_stride % 8) ||
      !aligned16(sketch) || (batch > 1 && sketch_batch_stride % 16) ||
      (reinterpret_cast<uintptr_t>(scales) & 3u) || (reinterpret_cast<uintptr_t>(bounds) & 3u))
    return fail(TDSA_ERR_ALIGN, "keys and the sketch need 16-byte aligned rows (TMA)");
  return launch_sketch_keys(keys, k_batch_stride, k_row_stride, dtype, batch, first, length,
                            sketch, sketch_batch_stride, scales, bounds, scale_batch_stride,
                            static_cast<cudaStream_t>(stream));
}

size_t tdsa_sketch_topk_workspace_bytes(int batch, int max_length, int k) {
  if (batch < 1 || max_length < 1 || k < 1 || k > max_length) return 0;
  return sketch_workspace_bytes(batch, max_length, k);
}

int tdsa_sketch_workspace_offsets(int batch, int max_length, int k, int64_t* offsets) {
  if (!offsets || batch < 1 || max_length < 1 || k < 1 || k > max_length)
    return fail(TDSA_ERR_INVALID, "bad geometry");
  sketch_workspace_offsets(batch, max_length, k, offsets);
  return TDSA_OK;
}

int tdsa_sketch_topk(const void* queries, int64_t q_batch_stride, const float* weights,
                     int64_t w_batch_stride, const void* keys, int64_t k_batch_stride,
                     int64_t k_row_stride, int dtype, const int8_t* sketch,
                     int64_t sketch_batch_stride, const float* scales, const void* bounds,
                     int64_t scale_batch_stride, int batch, int length, int max_length, int k,
                     int sorted, void* out_indices, int index_bytes, int64_t idx_batch_stride,
                     float* out_values, int64_t val_batch_stride, uint64_t* stats,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                            k_batch_stride, k_row_stride, dtype, batch, length, nullptr, 0,
                            false);
  if (rc) return rc;
  if (dtype == TDSA_F32) return fail(TDSA_ERR_UNSUPPORTED, "the key sketch takes bf16/fp16 keys");
  if (length < k || length > max_length)
    return fail(TDSA_ERR_INVALID, "need k <= length <= max_length");
  rc = topk_check(length, k, sorted);
  if (rc) return rc;
  rc = check_topk_out(out_indices, index_bytes, idx_batch_stride, out_values, val_batch_stride,
                      batch, k);
  if (rc) return rc;
  if (!out_indices) return fail(TDSA_ERR_INVALID, "out_indices is null");
  if (!sketch || !scales || !bounds) return fail(TDSA_ERR_INVALID, "null sketch argument");
  if (!aligned16(sketch) || (batch > 1 && sketch_batch_stride % 16) ||
      (reinterpret_cast<uintptr_t>(scales) & 3u) || (reinterpret_cast<uintptr_t>(bounds) & 3u))
    return fail(TDSA_ERR_ALIGN, "the sketch needs 16-byte aligned rows (TMA)");
  if (batch > 1 && (sketch_batch_stride < static_cast<int64_t>(length) * kHeadDim ||
                    scale_batch_stride < length))
    return fail(TDSA_ERR_INVALID, "sketch strides overlap the rows of one sequence");
  const size_t need = sketch_workspace_bytes(batch, max_length, k);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(TDSA_ERR_WORKSPACE,
                "workspace missing, unaligned (256 B) or smaller than tdsa_sketch_topk_workspace_bytes");
  return run_sketch_topk(queries, q_batch_stride, weights, w_batch_stride, keys, k_batch_stride,
                         k_row_stride, dtype, sketch, sketch_batch_stride, scales, bounds,
                         scale_batch_stride, batch, length, max_length, k, sorted ? 1 : 0,
                         out_indices, index_bytes, idx_batch_stride, out_values,
                         val_batch_stride, reinterpret_cast<unsigned long long*>(stats),
                         workspace, static_cast<cudaStream_t>(stream));
}

size_t tdsa_exact_state_bytes(int batch, int max_length, int k, int block_size) {
  if (batch < 1 || max_length < 1 || k < 1 || k > max_length ||
      (block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128))
    return 0;
  return exact_layout(batch, max_length, k, block_size).total;
}

static int exact_common(int init, void* state, size_t state_bytes, const void* queries,
                        int64_t q_batch_stride, const float* weights, int64_t w_batch_stride,
                        const void* keys, int64_t k_batch_stride, int64_t k_row_stride,
                        int dtype, int batch, int prev_length, int length, int max_length,
                        int k, int block_size, int sorted, void* out_indices, int index_bytes,
                        int64_t idx_batch_stride, float* out_values, int64_t val_batch_stride,
                        void* stream) {
  int rc = check_score_args(queries, q_batch_stride, weights, w_batch_stride, keys,
                            k_batch_stride, k_row_stride, dtype, batch, length, nullptr, 0,
                            false);
  if (rc) return rc;
  if (dtype == TDSA_F32)
    return fail(TDSA_ERR_UNSUPPORTED, "the exact progressive path takes bf16/fp16 keys");
  if (length < 1 || length > max_length)
    return fail(TDSA_ERR_INVALID, "need 1 <= length <= max_length");
  if (!init && (prev_length < k || prev_length > length))
    return fail(TDSA_ERR_INVALID, "need k <= prev_length <= length (the cache only grows)");
  rc = topk_check(length, k, sorted);
  if (rc) return rc;
  if (out_indices && index_bytes != 4 && index_bytes != 8)
    return fail(TDSA_ERR_INVALID, "index_bytes must be 4 or 8");
  if (batch > 1 && ((out_indices && idx_batch_stride < k) || (out_values && val_batch_stride < k)))
    return fail(TDSA_ERR_INVALID, "output row strides must be >= k");
  const size_t need = tdsa_exact_state_bytes(batch, max_length, k, block_size);
  if (need == 0) return fail(TDSA_ERR_INVALID, "bad state geometry (block_size 16/32/64/128)");
  if (!state || state_bytes < need)
    return fail(TDSA_ERR_WORKSPACE, "exact state missing or smaller than tdsa_exact_state_bytes");
  const ExactLayout L = exact_layout(batch, max_length, k, block_size);
  return run_exact(init, static_cast<uint8_t*>(state), L, queries, q_batch_stride, weights,
                   w_batch_stride, keys, k_batch_stride, k_row_stride, dtype, batch,
                   prev_length, length, max_length, k, block_size, sorted ? 1 : 0, out_indices,
                   index_bytes, idx_batch_stride, out_values, val_batch_stride,
                   static_cast<cudaStream_t>(stream));
}

int tdsa_exact_init(void* state, size_t state_bytes, const void* queries,
                    int64_t q_batch_stride, const float* weights, int64_t w_batch_stride,
                    const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                    int batch, int length, int max_length, int k, int block_size, int sorted,
                    void* out_indices, int index_bytes, int64_t idx_batch_stride,
                    float* out_values, int64_t val_batch_stride, void* stream) {
  return exact_common(1, state, state_bytes, queries, q_batch_stride, weights, w_batch_stride,
                      keys, k_batch_stride, k_row_stride, dtype, batch, 0, length, max_length,
                      k, block_size, sorted, out_indices, index_bytes, idx_batch_stride,
                      out_values, val_batch_stride, stream);
}

int tdsa_exact_step(void* state, size_t state_bytes, const void* queries,
                    int64_t q_batch_stride, const float* weights, int64_t w_batch_stride,
                    const void* keys, int64_t k_batch_stride, int64_t k_row_stride, int dtype,
                    int batch, int prev_length, int length, int max_length, int k,
                    int block_size, int sorted, void* out_indices, int index_bytes,
                    int64_t idx_batch_stride, float* out_values, int64_t val_batch_stride,
                    void* stream) {
  return exact_common(0, state, state_bytes, queries, q_batch_stride, weights, w_batch_stride,
                      keys, k_batch_stride, k_row_stride, dtype, batch, prev_length, length,
                      max_length, k, block_size, sorted, out_indices, index_bytes,
                      idx_batch_stride, out_values, val_batch_stride, stream);
}

int tdsa_exact_stats(const void* state, size_t state_bytes, int batch, int max_length, int k,
                     int block_size, uint64_t* stats_out) {
  const size_t need = tdsa_exact_state_bytes(batch, max_length, k, block_size);
  if (!state || !stats_out || need == 0 || state_bytes < need)
    return fail(TDSA_ERR_INVALID, "bad state or geometry");
  const ExactLayout L = exact_layout(batch, max_length, k, block_size);
  TDSA_CUDA_CHECK(cudaMemcpy(stats_out, static_cast<const uint8_t*>(state) + L.stats,
                             static_cast<size_t>(batch) * 64, cudaMemcpyDeviceToHost));
  return TDSA_OK;
}

int tdsa_block_key_norms(const double* keys, int tokens, int heads, int dim, int block_size,
                         double* out, void* stream) {
  if (!keys || !out) return fail(TDSA_ERR_INVALID, "null pointer");
  if (tokens < 1 || heads < 1 || dim < 1 || block_size < 1)
    return fail(TDSA_ERR_INVALID, "tokens, heads, dim and block_size must be positive");
  return launch_block_key_norms(keys, tokens, heads, dim, block_size, out,
                                static_cast<cudaStream_t>(stream));
}

int tdsa_temporal_radius(const double* q_now, const double* q_prev, const double* w_now,
                         const double* w_prev, const double* block_key_norm, int heads, int dim,
                         int blocks, double* coeff_workspace, double* out, void* stream) {
  if (!q_now || !q_prev || !w_now || !w_prev || !block_key_norm || !coeff_workspace || !out)
    return fail(TDSA_ERR_INVALID, "null pointer");
  if (heads < 1 || dim < 1 || blocks < 0) return fail(TDSA_ERR_INVALID, "bad sizes");
  if (blocks == 0) return TDSA_OK;
  return launch_temporal_radius(q_now, q_prev, w_now, w_prev, block_key_norm, heads, dim,
                                blocks, coeff_workspace, out, static_cast<cudaStream_t>(stream));
}

int tdsa_relu_index_score(const double* q, const double* keys, const double* w, int heads,
                          int dim, int tokens, double* out, void* stream) {
  if (!q || !keys || !w || !out) return fail(TDSA_ERR_INVALID, "null pointer");
  if (heads < 1 || dim < 1 || tokens < 0) return fail(TDSA_ERR_INVALID, "bad sizes");
  if (tokens == 0) return TDSA_OK;
  return launch_relu_index_score(q, keys, w, heads, dim, tokens, out,
                                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
