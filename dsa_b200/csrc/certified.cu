// Float64 device versions of the reference's certified-bound helpers
// (src/temporal_dsa/certified.py:6-61), generic in heads and dims:
//   relu_index_score      I_s = sum_j w_j ReLU(q_j . k_s)                    (:6-15)
//   temporal_score_radius R_b = sum_h block_key_norm[b,h] * coefficient_h     (:18-48)
//                         coefficient_h = |w_t,h - w_p,h| ||q_p,h|| + |w_t,h| ||q_t,h - q_p,h||
//   block_key_norms       max_{s in block} ||k_s,h||  for keys [tokens, heads, dim] (:51-61)
#include "common.cuh"
#include "kernels.cuh"

namespace tdsa {

namespace {

// One warp per (block, head): max over the block's tokens of the L2 norm.
__global__ void block_key_norms_kernel(const double* __restrict__ keys, int tokens, int heads,
                                       int dim, int bs, double* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nb = (tokens + bs - 1) / bs;
  if (warp >= nb * heads) return;
  const int b = warp / heads, h = warp % heads;
  double best = 0.0;
  for (int t = b * bs; t < min(tokens, (b + 1) * bs); ++t) {
    const double* row = keys + (static_cast<int64_t>(t) * heads + h) * dim;
    double s = 0.0;
    for (int d = lane; d < dim; d += 32) s += row[d] * row[d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    best = fmax(best, sqrt(s));
  }
  if (lane == 0) out[static_cast<int64_t>(b) * heads + h] = best;
}

// coefficient_h, one warp per head.
__global__ void radius_coeff_kernel(const double* __restrict__ qn, const double* __restrict__ qp,
                                    const double* __restrict__ wn, const double* __restrict__ wp,
                                    int heads, int dim, double* __restrict__ coeff) {
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (h >= heads) return;
  double dd = 0.0, pp = 0.0;
  for (int d = lane; d < dim; d += 32) {
    const double a = qn[static_cast<int64_t>(h) * dim + d], b = qp[static_cast<int64_t>(h) * dim + d];
    dd += (a - b) * (a - b);
    pp += b * b;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    dd += __shfl_xor_sync(0xffffffffu, dd, o);
    pp += __shfl_xor_sync(0xffffffffu, pp, o);
  }
  if (lane == 0) coeff[h] = fabs(wn[h] - wp[h]) * sqrt(pp) + fabs(wn[h]) * sqrt(dd);
}

// R_b = block_key_norm[b,:] . coeff, one thread per block.
__global__ void radius_kernel(const double* __restrict__ norms, const double* __restrict__ coeff,
                              int nb, int heads, double* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  double r = 0.0;
  for (int h = 0; h < heads; ++h) r += norms[static_cast<int64_t>(b) * heads + h] * coeff[h];
  out[b] = r;
}

// I_s, one thread per token; q [heads, dim] staged in shared memory when it fits.
__global__ void relu_index_kernel(const double* __restrict__ q, const double* __restrict__ keys,
                                  const double* __restrict__ w, int heads, int dim, int tokens,
                                  double* __restrict__ out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  const double* k = keys + static_cast<int64_t>(t) * dim;
  double s = 0.0;
  for (int h = 0; h < heads; ++h) {
    double dot = 0.0;
    for (int d = 0; d < dim; ++d) dot += q[static_cast<int64_t>(h) * dim + d] * k[d];
    s += fmax(dot, 0.0) * w[h];
  }
  out[t] = s;
}

}  // namespace

int launch_block_key_norms(const double* keys, int tokens, int heads, int dim, int bs,
                           double* out, cudaStream_t stream) {
  const int nb = (tokens + bs - 1) / bs;
  const int64_t warps = static_cast<int64_t>(nb) * heads;
  const int blocks = static_cast<int>((warps * 32 + 255) / 256);
  block_key_norms_kernel<<<blocks, 256, 0, stream>>>(keys, tokens, heads, dim, bs, out);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

int launch_temporal_radius(const double* qn, const double* qp, const double* wn,
                           const double* wp, const double* norms, int heads, int dim, int nb,
                           double* coeff_ws, double* out, cudaStream_t stream) {
  radius_coeff_kernel<<<(heads * 32 + 255) / 256, 256, 0, stream>>>(qn, qp, wn, wp, heads, dim,
                                                                    coeff_ws);
  TDSA_CUDA_CHECK(cudaGetLastError());
  radius_kernel<<<(nb + 255) / 256, 256, 0, stream>>>(norms, coeff_ws, nb, heads, out);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

int launch_relu_index_score(const double* q, const double* keys, const double* w, int heads,
                            int dim, int tokens, double* out, cudaStream_t stream) {
  relu_index_kernel<<<(tokens + 127) / 128, 128, 0, stream>>>(q, keys, w, heads, dim, tokens,
                                                             out);
  TDSA_CUDA_CHECK(cudaGetLastError());
  return TDSA_OK;
}

}  // namespace tdsa
