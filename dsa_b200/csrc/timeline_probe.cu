// Read-stream probe of timeline builds (TDSA_TIMELINE only; the product library holds none
// of this): the dense score kernel's key stream with no arithmetic, to measure the read
// ceiling that kernel streams against.  One CTA per SM walks a contiguous range of 32 KB
// key tiles ([batch][length][128] bf16, as the score kernel numbers them) through a 4-stage
// shared-memory ring, loading each tile either as the score kernel does (two 64-column
// boxes with the 128-byte swizzle, mode 0) or as one plain bulk copy (mode 1), and refills a
// stage as soon as its previous tile has landed.
#ifdef TDSA_TIMELINE
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace tdsa {

namespace {

constexpr int kRingStages = 4;
constexpr int kRingTile = 32768;

__global__ void __launch_bounds__(32, 1)
    read_stream_kernel(const __grid_constant__ CUtensorMap kmap, const uint8_t* keys,
                       int64_t total_tiles, int tiles_per_seq, int mode, int* status) {
  extern __shared__ uint8_t raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[kRingStages];
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  for (int s = 0; s < kRingStages; ++s) mbar_init(&bars[s], 1);
  fence_mbar_init();
  const int64_t t0 = total_tiles * blockIdx.x / gridDim.x;
  const int64_t t1 = total_tiles * (blockIdx.x + 1) / gridDim.x;
  const uint64_t pol = policy_evict_first();
  int i = 0;
  for (int64_t t = t0; t < t1; ++t, ++i) {
    const int s = i % kRingStages;
    if (i >= kRingStages && !mbar_wait(&bars[s], ((i / kRingStages) - 1) & 1u, &abort_flag))
      break;
    mbar_arrive_expect_tx(&bars[s], kRingTile);
    uint8_t* dst = ring + s * kRingTile;
    if (mode == 0) {
      const int b = static_cast<int>(t / tiles_per_seq);
      const int tt = static_cast<int>(t - static_cast<int64_t>(b) * tiles_per_seq);
      tma_load_3d(dst, &kmap, &bars[s], 0, tt * 128, b, pol);
      tma_load_3d(dst + kRingTile / 2, &kmap, &bars[s], 64, tt * 128, b, pol);
    } else {
      bulk_load(dst, keys + t * kRingTile, kRingTile, &bars[s]);
    }
  }
  volatile int no_abort = 0;  // every issued copy lands before the CTA exits
  for (int s = 0; s < kRingStages && s < i; ++s) {
    const int n = (i - s + kRingStages - 1) / kRingStages;
    mbar_wait(&bars[s], (n - 1) & 1u, &no_abort);
  }
  if (abort_flag) atomicOr(status, TDSA_ERR_TIMEOUT);
}

}  // namespace

}  // namespace tdsa

// keys: [batch][length][128] bf16, contiguous, length a multiple of 128.
extern "C" int tdsa_timeline_read_stream(const void* keys, int batch, int length, int mode,
                                         void* stream) {
  using namespace tdsa;
  if (!keys || batch < 1 || length < 128 || length % 128 || (mode != 0 && mode != 1))
    return fail(TDSA_ERR_INVALID, "read stream: bad arguments");
  CUtensorMap kmap;
  const uint64_t dims[3] = {128, static_cast<uint64_t>(length), static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {256, static_cast<uint64_t>(length) * 256};
  const uint32_t box[3] = {64, 128, 1};
  int rc = encode_tmap(&kmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, keys, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int tps = length / 128;
  const int64_t total = static_cast<int64_t>(tps) * batch;
  const int sms = device_sm_count(current_device());
  const int grid = total < sms ? static_cast<int>(total) : sms;
  const int smem = kRingStages * kRingTile + 1024;
  int* status = device_status_ptr();
  if (!status) return fail(TDSA_ERR_CUDA, "read stream: no device status word");
  TDSA_CUDA_CHECK(ensure_dynamic_smem(reinterpret_cast<const void*>(read_stream_kernel), smem));
  read_stream_kernel<<<grid, 32, smem, static_cast<cudaStream_t>(stream)>>>(
      kmap, static_cast<const uint8_t*>(keys), total, tps, mode, status);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}
#endif
