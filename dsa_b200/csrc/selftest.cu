// Self-test of the kernels' failure path: a wait that can never complete must give up after
// its cycle limit, raise TDSA_ERR_TIMEOUT in the device status word and leave the context
// usable.  The kernel waits on an mbarrier nobody arrives on (the same bounded try_wait
// loop the real kernels use, with a caller-chosen limit instead of ~1 s), so no GPU fault,
// trap or hang is involved.
#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace tdsa {

namespace {

__global__ void bounded_wait_kernel(long long limit_cycles, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    fence_mbar_init();
  }
  __syncthreads();
  bool done = mbar_test(&bar, 0);
  const long long start = clock64();
  while (!done && clock64() - start <= limit_cycles) done = mbar_test(&bar, 0);
  if (!done && threadIdx.x == 0) atomicOr(status, TDSA_ERR_TIMEOUT);
}

}  // namespace

int launch_bounded_wait_selftest(long long limit_cycles, cudaStream_t stream, int* status) {
  bounded_wait_kernel<<<1, 32, 0, stream>>>(limit_cycles, status);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
