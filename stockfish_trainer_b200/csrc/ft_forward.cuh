// Sparse feature-transformer FORWARD (sm_100a).
//
// Semantics (reference src/model/modules/feature_transformer/kernel.py:89-103):
//   out[b, c] = bias[c] + sum over k ascending, idx[b, k] != -1, of W[idx[b, k], c]
// in fp32, one add per active feature in ascending k -- the same order as the
// reference, so the result is bit-identical.
//
// Mapping: one warp per (perspective, position) item and column chunk.  The
// warp reads 32 indices with one coalesced load, ballots the valid ones and
// walks them in ascending k, U rows at a time: all U x V 128-bit row loads
// are issued before the U x V adds, so each lane keeps U*V loads in flight.
// Lanes own fixed column vectors, which keeps the per-column add order.
#pragma once

#include "common.cuh"

namespace nnue {

struct FwdParams {
  const int32_t* idx[2];  // [B, K] per perspective (int32, -1 padded)
  float* out[2];          // [B, C] per perspective
  const float* W;         // [T, C]
  const float* bias;      // [C]
  int64_t B;
  int32_t K;
  int32_t T;
  int32_t P;               // perspectives in this launch (1 or 2)
  int32_t items_per_warp;  // consecutive (perspective, position) items per warp
  int32_t chunk0;          // first column chunk of this launch (blockIdx.y offset)
  Geom g;
};

template <typename VT, int V, int U>
__global__ void __launch_bounds__(kBlock) ft_forward_kernel(const FwdParams p) {
  using Ops = Vec<VT>;
  const int lane = threadIdx.x & 31;
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);

  bool ok[V];
  VT bias_r[V];
  const VT* __restrict__ bvec = reinterpret_cast<const VT*>(p.bias) + c0 + lane;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    ok[v] = lane + 32 * v < width;
    bias_r[v] = ok[v] ? bvec[32 * v] : Ops::zero();
  }
  const VT* __restrict__ Wv = reinterpret_cast<const VT*>(p.W) + c0 + lane;
  const int64_t row_vec = p.g.n_vec;

  const int64_t n_items = (int64_t)p.P * p.B;
  int64_t item = ((int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5)) * p.items_per_warp;
  const int64_t item_end = item + p.items_per_warp < n_items ? item + p.items_per_warp : n_items;

  for (; item < item_end; ++item) {
    const int persp = item >= p.B ? 1 : 0;
    const int64_t b = item - (int64_t)persp * p.B;
    const int32_t* __restrict__ irow = (persp ? p.idx[1] : p.idx[0]) + b * p.K;

    VT acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = bias_r[v];

    for (int k0 = 0; k0 < p.K; k0 += 32) {
      const int kk = k0 + lane;
      const int f = kk < p.K ? __ldcs(irow + kk) : -1;
      const bool valid = (unsigned)f < (unsigned)p.T;
      if (!valid && f != -1) flag_error(kErrBadIndex);
      unsigned mask = __ballot_sync(kFull, valid);
      while (mask) {
        int rows[U];
        bool has[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          has[u] = mask != 0;
          const int src = has[u] ? __ffs(mask) - 1 : 0;
          rows[u] = __shfl_sync(kFull, f, src);
          mask &= mask - 1;
        }
        VT w[U][V];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (has[u] && ok[v]) w[u][v] = Ops::ldg(Wv + (int64_t)rows[u] * row_vec + 32 * v);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (has[u] && ok[v]) Ops::add(acc[v], w[u][v]);
      }
    }
    VT* o = reinterpret_cast<VT*>(persp ? p.out[1] : p.out[0]) + b * row_vec + c0 + lane;
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (ok[v]) Ops::st_stream(o + 32 * v, acc[v]);
  }
}

}  // namespace nnue
