// Optional device timeline of the decode step's kernels (query projection, dense score,
// top-k): with TDSA_TIMELINE defined (python -m dsa_b200.build --timeline, which writes
// libtdsa_timeline.so beside the library) one thread per CTA records %globaltimer at fixed
// points of its kernel; without it every macro below is empty and the kernels are unchanged.
//
// Each instrumented kernel owns a record array of 8 launches x ncta CTAs x nslot points.  A
// CTA takes a ticket from the kernel's launch counter at entry; ticket / (CTAs per launch)
// is the launch number, kept modulo 8, so the last 8 launches of a kernel stay readable as
// long as its launches do not overlap (a dependent launch on the same stream enters only
// after the previous launch of the same kernel, two kernels back, has completed).
// tdsa_timeline_<name>(dst, launches) copies the array and the counter out (host; after a
// synchronize).  Timeline builds are for measurement only; the product library never
// defines TDSA_TIMELINE.
#pragma once

#ifdef TDSA_TIMELINE
#include <cuda_runtime.h>

__device__ __forceinline__ unsigned long long tdsa_tl_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

#define TDSA_TL_DECL(name, ncta, nslot)                                                  \
  __device__ unsigned long long tdsa_tl_##name[8 * (ncta) * (nslot)];                  \
  __device__ unsigned int tdsa_tl_##name##_tickets;                                     \
  extern "C" int tdsa_timeline_##name(unsigned long long* dst, unsigned int* tickets) { \
    if (cudaMemcpyFromSymbol(tickets, tdsa_tl_##name##_tickets, sizeof(unsigned int)) != \
        cudaSuccess)                                                                    \
      return 1;                                                                         \
    return cudaMemcpyFromSymbol(dst, tdsa_tl_##name, sizeof(tdsa_tl_##name)) ==         \
                   cudaSuccess                                                          \
               ? 0                                                                      \
               : 1;                                                                     \
  }
// the launch number of this CTA's kernel (one call per CTA)
#define TDSA_TL_TICKET(name) \
  ((atomicAdd(&tdsa_tl_##name##_tickets, 1u) / (gridDim.x * gridDim.y)) & 7u)
#define TDSA_TL_REC(name, ncta, nslot, launch, cta, slot)                             \
  do {                                                                               \
    if ((cta) < (ncta))                                                              \
      tdsa_tl_##name[((launch) * (ncta) + (cta)) * (nslot) + (slot)] = tdsa_tl_now(); \
  } while (0)
#else
#define TDSA_TL_DECL(name, ncta, nslot)
#define TDSA_TL_TICKET(name) 0u
#define TDSA_TL_REC(name, ncta, nslot, launch, cta, slot) \
  do {                                                    \
  } while (0)
#endif
