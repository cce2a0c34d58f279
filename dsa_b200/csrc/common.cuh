// Shared definitions of the indexer library: status codes, the device status word,
// order-preserving float keys and host helpers (tensor maps, device properties).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/tdsa.h"

namespace tdsa {

constexpr int kHeads = 64;     // indexer heads (reference progressive_kernel.py:18)
constexpr int kHeadDim = 128;  // indexer head dim (reference progressive_kernel.py:19)
constexpr int kVerifierHeads = 8;

// Order-preserving map float -> uint32: larger float => larger key.  -0.0 and +0.0 map to
// the same key (they compare equal, as in numpy), every NaN maps above +inf.
__device__ __forceinline__ uint32_t float_to_key(float x) {
  uint32_t b = __float_as_uint(x);
  if ((b & 0x7FFFFFFFu) == 0u) b = 0u;               // -0.0 -> +0.0
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu)) return 0xFFFFFFFFu;  // NaN
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}

// One histogram increment per lane with `in` set, made by the whole warp: the lanes whose
// bin equals the first active lane's add together with one atomic (clustered scores hit
// one bin from most lanes), the others add alone.
__device__ __forceinline__ void add_to_bin(uint32_t* hist, bool in, uint32_t bin) {
  const unsigned act = __ballot_sync(0xffffffffu, in);
  if (!act) return;
  const int lead = __ffs(act) - 1;
  const uint32_t b0 = __shfl_sync(0xffffffffu, bin, lead);
  const unsigned same = __ballot_sync(0xffffffffu, in && bin == b0);
  if ((threadIdx.x & 31) == lead) atomicAdd(&hist[b0], __popc(same));
  else if (in && bin != b0) atomicAdd(&hist[bin], 1u);
}

// ------------------------------------------------------------------ host helpers
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

int device_sm_count(int device);
int current_device();

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes), called only when the
// kernel has not had at least `bytes` set on the current device yet.
cudaError_t ensure_dynamic_smem(const void* kernel, int bytes);

// Encodes a tiled tensor map (driver entry point fetched through the runtime).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

inline int elem_bytes(int dtype) { return dtype == TDSA_F32 ? 4 : 2; }

// Launch with programmatic stream serialization: the kernel may start while its
// predecessor on the stream drains, and synchronises itself with pdl_wait (ptx.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

#define TDSA_CUDA_CHECK(expr)                                                          \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess)                                                             \
      return ::tdsa::fail(TDSA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

}  // namespace tdsa
