// Candidate exchange of an L-sharded top-k over peer memory (NVLink / NVSwitch), in place
// of an all-gather + merge.  New: the reference never shards (its scoring runs on one GPU).
//
// Every rank allocates one exchange region (layout in kernels.cuh, PeerGather) and shares
// it with the node's other ranks through CUDA IPC.  A step is ONE launch per rank
// (launch_exchange_topk, topk.cu): each CTA publishes its row of the rank's local top-k into
// the region, raises that row's flag in every rank's region with a system-scope release
// store (a plain store over NVLink for a peer), waits (bounded) for the row's flag from
// every rank, pulls the ranks' rows from their regions and selects the global top-k -- the
// collective and the selection in one kernel.  Loads and stores only; no multicast.
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

struct tdsa_exchange {
  int world = 0, rank = 0, rows = 0, k = 0, device = -1;
  uint8_t* base = nullptr;  // this rank's region
  size_t bytes = 0;
  uint8_t* peers[tdsa::kMaxExchangeWorld] = {nullptr};  // every rank's region, mapped here
  bool opened[tdsa::kMaxExchangeWorld] = {false};
  uint8_t** d_peers = nullptr;                          // device copy of `peers`
  bool connected = false;
  tdsa::PeerGather g = {};
};

namespace tdsa {

namespace {

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Byte offsets of the region's parts; returns the region size.
size_t exchange_layout(int world, int rows, int k, PeerGather& g) {
  const size_t cand = static_cast<size_t>(2) * rows * k * 4;
  size_t off = 0;
  g.vals_off = 0;
  off = align_up(cand, 256);
  g.idx_off = static_cast<int64_t>(off);
  off = align_up(off + cand, 256);
  g.flags_off = static_cast<int64_t>(off);
  off = align_up(off + static_cast<size_t>(2) * world * rows * 4, 256);
  g.ctr_off = static_cast<int64_t>(off);
  off = align_up(off + 16, 256);
  const size_t scratch = static_cast<size_t>(rows) * world * k * 4;
  g.scratch_v_off = static_cast<int64_t>(off);
  off = align_up(off + scratch, 256);
  g.scratch_i_off = static_cast<int64_t>(off);
  off = align_up(off + scratch, 256);
  return off;
}

}  // namespace

}  // namespace tdsa

using tdsa::fail;

extern "C" {

size_t tdsa_exchange_bytes(int world, int batch, int k) {
  if (world < 1 || world > tdsa::kMaxExchangeWorld || batch < 1 || k < 1) return 0;
  tdsa::PeerGather g = {};
  return tdsa::exchange_layout(world, batch, k, g);
}

int tdsa_exchange_create(int world, int rank, int batch, int k, tdsa_exchange** out,
                         void* ipc_handle_out) {
  if (!out || !ipc_handle_out) return fail(TDSA_ERR_INVALID, "null pointer argument");
  *out = nullptr;
  if (world < 1 || world > tdsa::kMaxExchangeWorld)
    return fail(TDSA_ERR_INVALID, "world must be in [1, 16]");
  if (rank < 0 || rank >= world) return fail(TDSA_ERR_INVALID, "rank outside [0, world)");
  if (batch < 1 || batch > 65535) return fail(TDSA_ERR_INVALID, "batch must be in [1, 65535]");
  if (k < 1 || static_cast<int64_t>(world) * k > tdsa::kTopkSegment)
    return fail(TDSA_ERR_UNSUPPORTED, "an exchange merges at most 32768 candidates per row");
  auto* ex = new tdsa_exchange();
  ex->world = world;
  ex->rank = rank;
  ex->rows = batch;
  ex->k = k;
  ex->device = tdsa::current_device();
  ex->bytes = tdsa::exchange_layout(world, batch, k, ex->g);
  auto undo = [&](const char* what, cudaError_t e) {
    if (ex->d_peers) cudaFree(ex->d_peers);
    if (ex->base) cudaFree(ex->base);
    delete ex;
    return fail(TDSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  };
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&ex->base), ex->bytes);
  if (e != cudaSuccess) return undo("cudaMalloc", e);
  e = cudaMemset(ex->base, 0, ex->bytes);
  if (e != cudaSuccess) return undo("cudaMemset", e);
  e = cudaMalloc(reinterpret_cast<void**>(&ex->d_peers), sizeof(uint8_t*) * world);
  if (e != cudaSuccess) return undo("cudaMalloc", e);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, ex->base);
  if (e != cudaSuccess) return undo("cudaIpcGetMemHandle", e);
  static_assert(sizeof(cudaIpcMemHandle_t) == TDSA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *out = ex;
  return TDSA_OK;
}

int tdsa_exchange_connect(tdsa_exchange* ex, const void* handles) {
  if (!ex || !handles) return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (ex->connected) return fail(TDSA_ERR_INVALID, "exchange already connected");
  const auto* hs = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < ex->world; ++r) {
    if (r == ex->rank) {
      ex->peers[r] = ex->base;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + static_cast<size_t>(r) * TDSA_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (ex->opened[q]) {
          cudaIpcCloseMemHandle(ex->peers[q]);
          ex->opened[q] = false;
        }
      return fail(TDSA_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    }
    ex->peers[r] = static_cast<uint8_t*>(p);
    ex->opened[r] = true;
  }
  TDSA_CUDA_CHECK(cudaMemcpy(ex->d_peers, ex->peers, sizeof(uint8_t*) * ex->world,
                             cudaMemcpyHostToDevice));
  ex->g.peer_base = ex->d_peers;
  ex->g.own = ex->base;
  ex->g.world = ex->world;
  ex->g.rank = ex->rank;
  ex->g.rows = ex->rows;
  ex->g.k = ex->k;
  ex->connected = true;
  return TDSA_OK;
}

int tdsa_exchange_topk(tdsa_exchange* ex, const float* values, const int32_t* indices,
                       int64_t batch_stride, int32_t index_offset, int sorted,
                       void* out_indices, int index_bytes, int64_t idx_batch_stride,
                       float* out_values, int64_t val_batch_stride, void* stream) {
  if (!ex || !values || !indices || !out_indices)
    return fail(TDSA_ERR_INVALID, "null pointer argument");
  if (!ex->connected) return fail(TDSA_ERR_INVALID, "exchange not connected");
  if (index_bytes != 4 && index_bytes != 8) return fail(TDSA_ERR_INVALID, "index_bytes: 4 or 8");
  if (ex->rows > 1 && batch_stride < ex->k)
    return fail(TDSA_ERR_INVALID, "candidate row stride must be >= k");
  if (ex->rows > 1 && (idx_batch_stride < ex->k || (out_values && val_batch_stride < ex->k)))
    return fail(TDSA_ERR_INVALID, "output row stride must be >= k");
  tdsa::PeerGather g = ex->g;
  g.local_vals = values;
  g.local_idx = indices;
  g.local_stride = batch_stride;
  g.offset = index_offset;
  return tdsa::launch_exchange_topk(g, sorted ? 1 : 0, out_indices, index_bytes,
                                    idx_batch_stride, out_values, val_batch_stride,
                                    static_cast<cudaStream_t>(stream));
}

int tdsa_exchange_destroy(tdsa_exchange* ex) {
  if (!ex) return TDSA_OK;
  int rc = TDSA_OK;
  for (int r = 0; r < ex->world; ++r)
    if (ex->opened[r] && cudaIpcCloseMemHandle(ex->peers[r]) != cudaSuccess) rc = TDSA_ERR_CUDA;
  if (ex->d_peers && cudaFree(ex->d_peers) != cudaSuccess) rc = TDSA_ERR_CUDA;
  if (ex->base && cudaFree(ex->base) != cudaSuccess) rc = TDSA_ERR_CUDA;
  delete ex;
  return rc ? fail(rc, "tdsa_exchange_destroy: a CUDA free failed") : TDSA_OK;
}

}  // extern "C"
