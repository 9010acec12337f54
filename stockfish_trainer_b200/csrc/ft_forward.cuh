// Sparse feature-transformer FORWARD (sm_100a).
//
// Semantics (reference src/model/modules/feature_transformer/kernel.py:89-103):
//   out[b, c] = bias[c] + sum over k ascending, idx[b, k] != -1, of W[idx[b, k], c]
// in fp32, one add per active feature in ascending k -- the same order as the
// reference, so the result is bit-identical.
//
// Mapping: one warp per (perspective, position) item and column chunk, a few
// consecutive items per warp.  The warp reads all index slots of an item at
// once (8 coalesced loads of 32), compacts the valid ones into a per-warp
// shared-memory list (ascending k) and streams the rows through a register
// queue (below).  The next item's indices are loaded while the current
// item's rows are in flight, so the index latency is hidden.  Lanes own fixed
// column vectors, which keeps the per-column add order.
#pragma once

#include <type_traits>

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
  TableSet tabs;           // MULTI kernels: W split over separately allocated row blocks
};

constexpr int kIdxGroups = 8;  // index slots read per item in one go: 8 x 32 = 256 (at most)

// Loads slots [32 * g0, 32 * (g0 + IG)) of one index row, one group of 32 per
// register, all loads in flight together.
template <int IG>
__device__ __forceinline__ void load_index_groups(const int32_t* __restrict__ irow, int K, int g0, int lane,
                                                  int (&f)[IG]) {
#pragma unroll
  for (int g = 0; g < IG; ++g) {
    const int k = (g0 + g) * 32 + lane;
    f[g] = k < K ? __ldcs(irow + k) : -1;
  }
}

// Writes the valid indices of f[] (ascending slot order), times `scale`, to
// `list`; returns how many.  Indices outside [-1, T) are flagged and dropped.
template <int IG>
__device__ __forceinline__ int compact_valid(const int (&f)[IG], int T, int* list, int lane, int scale = 1) {
  const unsigned lt = lanemask_lt();
  int n = 0;
#pragma unroll
  for (int g = 0; g < IG; ++g) {
    const bool valid = (unsigned)f[g] < (unsigned)T;
    if (!valid && f[g] != -1) flag_error(kErrBadIndex);
    const unsigned m = __ballot_sync(kFull, valid);
    if (valid) list[n + __popc(m & lt)] = f[g] * scale;
    n += __popc(m);
  }
  __syncwarp();
  return n;
}

// Table-set form of compact_valid: the list holds each valid row's address
// in its own block (lane-independent: block base + local row + chunk start).
template <typename VT, int IG>
__device__ __forceinline__ int compact_rows(const int (&f)[IG], int T, const TableSet& tabs, int row_vec,
                                            int c0, const VT** list, int lane) {
  const unsigned lt = lanemask_lt();
  int n = 0;
#pragma unroll
  for (int g = 0; g < IG; ++g) {
    const bool valid = (unsigned)f[g] < (unsigned)T;
    if (!valid && f[g] != -1) flag_error(kErrBadIndex);
    const unsigned m = __ballot_sync(kFull, valid);
    if (valid) {
      const int t = tabs.find(f[g]);
      list[n + __popc(m & lt)] =
          reinterpret_cast<const VT*>(tabs.base[t]) + (f[g] - tabs.start(t)) * (int64_t)row_vec + c0;
    }
    n += __popc(m);
  }
  __syncwarp();
  return n;
}

// The rows of an item stream through a D-slot register queue: consuming
// slot d immediately re-issues it with the row D further on, so D rows stay
// in flight for the whole item.  The compacted list holds row OFFSETS (index
// x row vectors, int32) and the bias is re-read from L1 per item.  The
// kernel is latency-bound: bytes in flight per SM are resident warps x D x
// one row slice, so MINB (resident blocks the register budget is sized for)
// matters as much as D.
// IG: index groups of 32 slots read per item in one go (IG * 32 >= K keeps
// every item to one pass; fewer groups, fewer registers).
template <typename VT, int V, int D, int MINB = 1, bool MULTI = false, int BLOCK = kBlock, int IG = kIdxGroups>
__global__ void __launch_bounds__(BLOCK, MINB) ft_forward_kernel(const FwdParams p) {
  using Ops = Vec<VT>;
  // one table: 32-bit row offsets; table set: row addresses
  using Entry = std::conditional_t<MULTI, const VT*, int>;
  __shared__ Entry s_list[BLOCK / 32][32 * IG];
  const int lane = threadIdx.x & 31;
  Entry* list = s_list[threadIdx.x >> 5];
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);
  bool ok[V];
#pragma unroll
  for (int v = 0; v < V; ++v) ok[v] = lane + 32 * v < width;
  const VT* __restrict__ bvec = reinterpret_cast<const VT*>(p.bias) + c0 + lane;
  const VT* __restrict__ Wv = reinterpret_cast<const VT*>(p.W) + c0 + lane;
  const int row_vec = p.g.n_vec;

  const int64_t n_items = (int64_t)p.P * p.B;
  int64_t item = ((int64_t)blockIdx.x * (BLOCK / 32) + (threadIdx.x >> 5)) * p.items_per_warp;
  const int64_t item_end = item + p.items_per_warp < n_items ? item + p.items_per_warp : n_items;
  if (item >= item_end) return;
  auto index_row = [&](int64_t it) {
    const int q = it >= p.B ? 1 : 0;
    return (q ? p.idx[1] : p.idx[0]) + (it - (int64_t)q * p.B) * p.K;
  };
  const int n_super = (p.K + 32 * IG - 1) / (32 * IG);
  int f[IG];
  load_index_groups<IG>(index_row(item), p.K, 0, lane, f);

  for (; item < item_end; ++item) {
    const int persp = item >= p.B ? 1 : 0;
    const int64_t b = item - (int64_t)persp * p.B;
    const int32_t* __restrict__ irow = index_row(item);
    VT acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = ok[v] ? Ops::ldg(bvec + 32 * v) : Ops::zero();
    for (int sg = 0; sg < n_super; ++sg) {
      if (sg > 0) load_index_groups<IG>(irow, p.K, sg * IG, lane, f);
      int n;
      if constexpr (MULTI) n = compact_rows<VT, IG>(f, p.T, p.tabs, row_vec, c0, list, lane);
      else n = compact_valid<IG>(f, p.T, list, lane, row_vec);
      // the next item's indices load while this item's rows are in flight
      if (sg == n_super - 1 && item + 1 < item_end) load_index_groups<IG>(index_row(item + 1), p.K, 0, lane, f);
      VT w[D][V];
      auto row_ptr = [&](const Entry e) -> const VT* {
        if constexpr (MULTI) return e + lane;
        else return Wv + e;
      };
      auto issue = [&](int slot, int j) {
        if (j < n) {
          const VT* a = row_ptr(list[j]);
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (ok[v]) w[slot][v] = Ops::ldg(a + 32 * v);
        }
      };
#pragma unroll
      for (int d = 0; d < D; ++d) issue(d, d);
      int j0 = 0;
      // steady state: every slot consumed and re-issued in range, no checks
      for (; j0 + 2 * D <= n; j0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (ok[v]) Ops::add(acc[v], w[d][v]);
          const VT* a = row_ptr(list[j0 + d + D]);
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (ok[v]) w[d][v] = Ops::ldg(a + 32 * v);
        }
      }
      for (; j0 < n; j0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
          if (j0 + d < n) {
#pragma unroll
            for (int v = 0; v < V; ++v)
              if (ok[v]) Ops::add(acc[v], w[d][v]);
          }
          issue(d, j0 + d + D);
        }
      }
      __syncwarp();  // every lane has read `list` before it is rewritten
    }
    VT* o = reinterpret_cast<VT*>(persp ? p.out[1] : p.out[0]) + b * row_vec + c0 + lane;
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (ok[v]) Ops::st_stream(o + 32 * v, acc[v]);
  }
}

// The narrow last column chunk (W <= 16 vectors; 6 for C = 1048), packed:
// G = 32 / W items at once per warp, lane group g (lanes g*W .. g*W + W - 1)
// owning item `base + g` and the chunk's W columns.  A full-width warp on this
// chunk would keep 32 - W lanes idle through a whole item walk -- one ninth
// of the kernel's warp time for a fiftieth of its bytes.  The G items'
// valid indices are compacted one item at a time (whole-warp ballots) into
// per-group shared-memory lists, then every group walks its own list
// through a D-slot register queue, all groups in lockstep up to the longest
// list.  Each lane still sums its column bias-first then in ascending k, so
// the outputs equal ft_forward_kernel's bit for bit.  Needs K <= 32 * IG
// (one index pass per item).
template <int W, int D, int IG, int MINB, int BLOCK>
__global__ void __launch_bounds__(BLOCK, MINB) ft_forward_tail_kernel(const FwdParams p) {
  using Ops = Vec<float4>;
  constexpr int G = 32 / W;
  constexpr int kStride = 32 * IG + 1;  // +1: the groups' lists start in different banks
  __shared__ int s_list[BLOCK / 32][G * kStride];
  const int lane = threadIdx.x & 31;
  int* lists = s_list[threadIdx.x >> 5];
  const int g = lane / W, sub = lane - g * W;
  const bool live = g < G;
  const int chunk = p.g.n_chunks - 1;
  const int c0 = p.g.begin(chunk);
  const int row_vec = p.g.n_vec;
  const float4* __restrict__ Wv = reinterpret_cast<const float4*>(p.W) + c0 + sub;
  const float4 bvec = live ? Ops::ldg(reinterpret_cast<const float4*>(p.bias) + c0 + sub) : Ops::zero();
  int* my_list = lists + (live ? g : 0) * kStride;

  const int64_t n_items = (int64_t)p.P * p.B;
  int64_t item = ((int64_t)blockIdx.x * (BLOCK / 32) + (threadIdx.x >> 5)) * (int64_t)p.items_per_warp * G;
  const int64_t item_end =
      item + (int64_t)p.items_per_warp * G < n_items ? item + (int64_t)p.items_per_warp * G : n_items;
  auto index_row = [&](int64_t it) {
    const int q = it >= p.B ? 1 : 0;
    return (q ? p.idx[1] : p.idx[0]) + (it - (int64_t)q * p.B) * p.K;
  };
  for (; item < item_end; item += G) {
    // compaction: item base + t into list t
    int n_mine = 0, n_max = 0;
#pragma unroll 1
    for (int t = 0; t < G; ++t) {
      int n_t = 0;
      if (item + t < item_end) {
        int f[IG];
        load_index_groups<IG>(index_row(item + t), p.K, 0, lane, f);
        n_t = compact_valid<IG>(f, p.T, lists + t * kStride, lane, row_vec);
      }
      if (t == g) n_mine = n_t;
      n_max = n_t > n_max ? n_t : n_max;
    }
    if (!live) n_mine = 0;
    float4 acc = bvec;
    float4 w[D];
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (d < n_mine) w[d] = Ops::ldg(Wv + my_list[d]);
    for (int j0 = 0; j0 < n_max; j0 += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int j = j0 + d;
        if (j < n_mine) {
          Ops::add(acc, w[d]);
          if (j + D < n_mine) w[d] = Ops::ldg(Wv + my_list[j + D]);
        }
      }
    }
    const int64_t it = item + g;
    if (live && it < item_end) {
      const int persp = it >= p.B ? 1 : 0;
      const int64_t b = it - (int64_t)persp * p.B;
      Ops::st_stream(reinterpret_cast<float4*>(persp ? p.out[1] : p.out[0]) + b * row_vec + c0 + sub, acc);
    }
    __syncwarp();  // every lane has read the lists before they are rewritten
  }
}

// out[r] = weight[r] + virtual_weight[r % period], one fp32 add per element:
// HalfKav2Hm.merged_weight (halfka_v2_hm.py:69-70, weight +
// virtual_weight.repeat(NUM_BUCKETS, 1)) without materialising the repeat.
template <typename VT>
__global__ void __launch_bounds__(256) merge_virtual_kernel(const VT* __restrict__ w, const VT* __restrict__ vw,
                                                            int64_t n, int64_t row_vec, int64_t period,
                                                            VT* __restrict__ out) {
  using Ops = Vec<VT>;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / row_vec, c = i - r * row_vec;
    VT x = __ldcs(w + i);
    Ops::add(x, __ldg(vw + (r % period) * row_vec + c));
    out[i] = x;
  }
}

}  // namespace nnue
