// Sparse feature-transformer BACKWARD (sm_100a).
//
// Reference semantics (src/model/modules/feature_transformer/kernel.py):
//   prep  :108-138  flatten idx, drop -1, STABLE sort by feature -> for every
//                   feature f the list of positions b that use it, ascending b
//   kernel:167-186  acc = 0; for b in that list: acc += dOut[b];
//                   weight_grad[f] = weight_grad[f] + acc
//   bias  :269      bias_grad += dOut.sum(0)
// The module-level caller (src/model/modules/features/composed.py:49-54)
// runs this once per perspective on one shared table; autograd then adds the
// two dense gradients.  The pair path here produces that sum directly:
//   dW[f] = acc_white(f) + acc_black(f)
// with each acc summed in ascending b, which is bit-identical to the
// reference's two zero-initialised gradients added once.
//
// Pipeline (no host synchronisation anywhere, so it is graph-capturable):
//   1. key = f * P + perspective.  A least-significant-digit radix sort of the
//      (key, b) pairs, <= 10-bit digits.  Each digit pass is
//        hist    : per warp tile, digit histogram  -> tile_hist[digit][tile]
//        scan    : exclusive scan of tile_hist (digit-major) -> tile offsets
//        scatter : each warp re-walks its tile in order; __match_any_sync
//                  ranks equal digits within 32 lanes, a per-warp running
//                  count in shared memory carries the rank across rounds.
//      Tiles are walked in input order, so every pass is stable and the
//      result is ordered by key with ties in original (ascending b) order.
//      The first pass reads the raw [B, K] index arrays directly and also
//      builds the full per-key histogram (-> segment offsets seg_start).
//   2. classify: rows with more than `heavy_threshold` entries go to a heavy
//      list (bounded); their work is split finer and scheduled first.
//   3. segsum: one warp per (row, column chunk); heavy rows one warp per
//      (row, 32-vector piece).  Every row of dW is written exactly once
//      (rows no position touches get 0), which replaces torch.zeros + RMW.
//   4. bias: deterministic column sum (per-part partials, fixed-order combine).
#pragma once

#include "common.cuh"

namespace nnue {

// ----------------------------------------------------------------------------
// Exclusive scan (int32), reduce-then-scan in three launches.  The length is
// either host-known or derived on the device from a count (so passes after the
// first can size themselves from the number of valid entries without a sync).
// ----------------------------------------------------------------------------
struct ScanLen {
  int64_t n;            // host length when `count` is null
  const int32_t* count; // device entry count -> length = bins * ceil(count / tile)
  int32_t tile;
  int32_t bins;
};

__device__ __forceinline__ int64_t scan_length(const ScanLen& L) {
  if (!L.count) return L.n;
  const int64_t tiles = ((int64_t)*L.count + L.tile - 1) / L.tile;
  return tiles * L.bins;
}

constexpr int kScanItems = 16;
constexpr int kScanTile = kBlock * kScanItems;

__global__ void __launch_bounds__(kBlock) scan_reduce_kernel(const int32_t* __restrict__ in, ScanLen L,
                                                             int32_t* __restrict__ block_sums) {
  __shared__ int red[32];
  const int64_t n = scan_length(L);
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  int s = 0;
  if (base < n) {
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
      const int64_t j = base + i * kBlock + threadIdx.x;
      if (j < n) s += in[j];
    }
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    int t = threadIdx.x < kWarpsPerBlock ? red[threadIdx.x] : 0;
    t = warp_sum(t);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = t;
  }
}

// Single block: exclusive scan of nb block sums, in place.
__global__ void __launch_bounds__(1024) scan_top_kernel(int32_t* __restrict__ block_sums, int64_t nb) {
  __shared__ int scratch[33];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < nb; base += blockDim.x) {
    const int64_t j = base + threadIdx.x;
    const int v = j < nb ? block_sums[j] : 0;
    const int incl = block_inclusive_scan(v, scratch);
    const int c = carry;
    if (j < nb) block_sums[j] = c + incl - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = c + incl;
    __syncthreads();
  }
}

// out[i] = block offset + exclusive prefix inside the block.  In place is fine.
__global__ void __launch_bounds__(kBlock) scan_down_kernel(const int32_t* in, int32_t* out, ScanLen L,
                                                           const int32_t* __restrict__ block_sums) {
  __shared__ int scratch[33];
  const int64_t n = scan_length(L);
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  if (base >= n) return;  // uniform per block
  const int64_t t0 = base + (int64_t)threadIdx.x * kScanItems;
  int v[kScanItems];
  int tsum = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    v[i] = t0 + i < n ? in[t0 + i] : 0;
    tsum += v[i];
  }
  const int incl = block_inclusive_scan(tsum, scratch);
  int run = block_sums[blockIdx.x] + incl - tsum;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    if (t0 + i < n) out[t0 + i] = run;
    run += v[i];
  }
}

// ----------------------------------------------------------------------------
// Radix passes
// ----------------------------------------------------------------------------
struct RawSrc {
  const int32_t* idx[2];  // [B, K] per perspective
  int64_t n_raw;          // B * K
  int32_t K;
  int32_t T;
  int32_t P;
};

struct PassParams {
  RawSrc raw;                // first pass: read the raw index arrays
  const int32_t* in_keys;    // later passes
  const int32_t* in_vals;
  const int32_t* count;      // later passes: device count of valid entries
  int32_t tile;              // first pass: index rows per warp; later: entries per warp (multiple of 32*kSortBatch)
  int32_t shift;             // digit = (key >> shift) & (bins - 1)
  int32_t bits;
  int32_t* tile_hist;        // [bins][n_tiles]
  int32_t* key_count;        // first pass: full histogram over keys (may be null)
  int32_t* out_keys;         // null on the last pass
  int32_t* out_vals;
  int64_t out_cap;           // capacity of out_keys / out_vals
};

constexpr int kSortBatch = 16;  // 32-slot chunks loaded before they are processed

// ---- first pass: walk the raw [P][B][K] index arrays row by row ------------
// A warp tile is `tile` consecutive index rows (perspective-major, then
// position).  Each row is read in chunks of 32 slots, kSortBatch chunks per
// batch of loads; a chunk with no valid slot (the -1 tail) costs one ballot.
// Entries are visited in (perspective, position, slot) order, so ranks are
// stable.
struct RowWalk {
  int64_t row;  // global row = perspective * B + position
  int kc;       // 32-slot chunk inside the row
};

__device__ __forceinline__ void raw_load_batch(const PassParams& p, RowWalk w, int64_t r_end, int KC, int lane,
                                               int (&f)[kSortBatch], int (&persp)[kSortBatch],
                                               int (&b)[kSortBatch]) {
  const int64_t B = p.raw.n_raw / (p.raw.K > 0 ? p.raw.K : 1);
#pragma unroll
  for (int r = 0; r < kSortBatch; ++r) {
    f[r] = -1;
    persp[r] = 0;
    b[r] = 0;
    if (w.row < r_end) {
      const int q = w.row >= B ? 1 : 0;
      const int64_t pos = w.row - q * B;
      const int k = w.kc * 32 + lane;
      persp[r] = q;
      b[r] = (int)pos;
      if (k < p.raw.K) f[r] = __ldcs((q ? p.raw.idx[1] : p.raw.idx[0]) + pos * p.raw.K + k);
      if (++w.kc == KC) {
        w.kc = 0;
        ++w.row;
      }
    }
  }
}

__device__ __forceinline__ RowWalk advance(RowWalk w, int KC, int n) {
  const int64_t t = (int64_t)w.kc + n;
  w.row += t / KC;
  w.kc = (int)(t % KC);
  return w;
}

__global__ void __launch_bounds__(kBlock) sort_hist_rows_kernel(const PassParams p) {
  extern __shared__ int32_t sh[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bins = 1 << p.bits;
  int32_t* h = sh + warp * bins;
  for (int i = lane; i < bins; i += 32) h[i] = 0;
  __syncwarp();
  const int64_t rows = (int64_t)p.raw.P * (p.raw.n_raw / (p.raw.K > 0 ? p.raw.K : 1));
  const int64_t n_tiles = (rows + p.tile - 1) / p.tile;
  const int64_t tile = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (tile >= n_tiles) return;
  const int KC = (p.raw.K + 31) / 32;
  const int64_t r0 = tile * p.tile;
  const int64_t r1 = r0 + p.tile < rows ? r0 + p.tile : rows;
  for (RowWalk w{r0, 0}; w.row < r1; w = advance(w, KC, kSortBatch)) {
    int f[kSortBatch], persp[kSortBatch], b[kSortBatch];
    raw_load_batch(p, w, r1, KC, lane, f, persp, b);
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r) {
      const bool valid = (unsigned)f[r] < (unsigned)p.raw.T;
      if (!valid && f[r] != -1) flag_error(kErrBadIndex);
      if (__ballot_sync(kFull, valid) == 0) continue;
      if (valid) {
        const int key = f[r] * p.raw.P + persp[r];
        atomicAdd(&h[(key >> p.shift) & (bins - 1)], 1);
        if (p.key_count) atomicAdd(&p.key_count[key], 1);
      }
    }
  }
  __syncwarp();
  for (int i = lane; i < bins; i += 32) p.tile_hist[(int64_t)i * n_tiles + tile] = h[i];
}

// Appends one 32-wide round of (key, value) pairs to the per-digit runs.
__device__ __forceinline__ void scatter_round(const PassParams& p, int32_t* h, int bins, bool valid, int key, int val,
                                              unsigned lt) {
  const int digit = valid ? ((key >> p.shift) & (bins - 1)) : bins;  // `bins` = no digit
  const unsigned peers = __match_any_sync(kFull, digit);
  const int rank = __popc(peers & lt);
  const int dst0 = valid ? h[digit] : 0;
  __syncwarp();
  if (valid) {
    const int dst = dst0 + rank;
    if ((unsigned long long)(unsigned)dst < (unsigned long long)p.out_cap) {
      if (p.out_keys) p.out_keys[dst] = key;
      p.out_vals[dst] = val;
    } else {
      flag_error(kErrBadSegment);
    }
    if (rank == 0) h[digit] = dst0 + __popc(peers);
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kBlock) sort_scatter_rows_kernel(const PassParams p) {
  extern __shared__ int32_t sh[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bins = 1 << p.bits;
  int32_t* h = sh + warp * bins;  // running destination per digit
  const int64_t rows = (int64_t)p.raw.P * (p.raw.n_raw / (p.raw.K > 0 ? p.raw.K : 1));
  const int64_t n_tiles = (rows + p.tile - 1) / p.tile;
  const int64_t tile = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (tile >= n_tiles) return;
  // tile_hist now holds the scanned offsets: start of (digit, tile).
  for (int i = lane; i < bins; i += 32) h[i] = p.tile_hist[(int64_t)i * n_tiles + tile];
  __syncwarp();
  const int KC = (p.raw.K + 31) / 32;
  const int64_t r0 = tile * p.tile;
  const int64_t r1 = r0 + p.tile < rows ? r0 + p.tile : rows;
  const unsigned lt = lanemask_lt();
  for (RowWalk w{r0, 0}; w.row < r1; w = advance(w, KC, kSortBatch)) {
    int f[kSortBatch], persp[kSortBatch], b[kSortBatch];
    raw_load_batch(p, w, r1, KC, lane, f, persp, b);
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r) {
      const bool valid = (unsigned)f[r] < (unsigned)p.raw.T;
      if (__ballot_sync(kFull, valid) == 0) continue;
      const int64_t B = p.raw.n_raw / p.raw.K;
      scatter_round(p, h, bins, valid, f[r] * p.raw.P + persp[r], (int)(persp[r] * B + b[r]), lt);
    }
  }
}

// ---- later passes: flat (key, value) arrays of device-known length ---------
__global__ void __launch_bounds__(kBlock) sort_hist_kernel(const PassParams p) {
  extern __shared__ int32_t sh[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bins = 1 << p.bits;
  int32_t* h = sh + warp * bins;
  for (int i = lane; i < bins; i += 32) h[i] = 0;
  __syncwarp();
  const int64_t n_src = *p.count;
  const int64_t n_tiles = (n_src + p.tile - 1) / p.tile;
  const int64_t tile = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (tile >= n_tiles) return;  // whole warp
  const int64_t e0 = tile * p.tile;
  const int64_t e1 = e0 + p.tile < n_src ? e0 + p.tile : n_src;
  for (int64_t base = e0; base < e1; base += 32 * kSortBatch) {
    int key[kSortBatch];
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r) {
      const int64_t e = base + r * 32 + lane;
      key[r] = e < e1 ? __ldg(p.in_keys + e) : -1;
    }
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r)
      if (key[r] >= 0) atomicAdd(&h[(key[r] >> p.shift) & (bins - 1)], 1);
  }
  __syncwarp();
  for (int i = lane; i < bins; i += 32) p.tile_hist[(int64_t)i * n_tiles + tile] = h[i];
}

__global__ void __launch_bounds__(kBlock) sort_scatter_kernel(const PassParams p) {
  extern __shared__ int32_t sh[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bins = 1 << p.bits;
  int32_t* h = sh + warp * bins;  // running destination per digit
  const int64_t n_src = *p.count;
  const int64_t n_tiles = (n_src + p.tile - 1) / p.tile;
  const int64_t tile = (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (tile >= n_tiles) return;
  for (int i = lane; i < bins; i += 32) h[i] = p.tile_hist[(int64_t)i * n_tiles + tile];
  __syncwarp();
  const int64_t e0 = tile * p.tile;
  const int64_t e1 = e0 + p.tile < n_src ? e0 + p.tile : n_src;
  const unsigned lt = lanemask_lt();
  for (int64_t base = e0; base < e1; base += 32 * kSortBatch) {
    int key[kSortBatch], val[kSortBatch];
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r) {
      const int64_t e = base + r * 32 + lane;
      key[r] = -1;
      val[r] = 0;
      if (e < e1) {
        key[r] = __ldg(p.in_keys + e);
        val[r] = __ldg(p.in_vals + e);
      }
    }
#pragma unroll
    for (int r = 0; r < kSortBatch; ++r) {
      if (base + r * 32 >= e1) break;  // uniform
      scatter_round(p, h, bins, key[r] >= 0, key[r], val[r], lt);
    }
  }
}

// Rows with more than `threshold` entries (both perspectives) are heavy
// (used by the fallback walk path only).
__global__ void classify_rows_kernel(const int32_t* __restrict__ seg_start, int32_t T, int32_t P,
                                     int32_t threshold, int32_t cap, int32_t* __restrict__ n_heavy,
                                     int32_t* __restrict__ heavy_list, uint8_t* __restrict__ row_kind) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= T) return;
  const int n = seg_start[(f + 1) * P] - seg_start[f * P];
  uint8_t kind = 0;
  if (n > threshold) {
    const int s = atomicAdd(n_heavy, 1);
    if (s < cap) {
      heavy_list[s] = (int32_t)f;
      kind = 1;
    }
  }
  row_kind[f] = kind;
}

// Streaming work split: warp w owns the rows whose first entry lies in
// [w * epw, (w + 1) * epw), i.e. rows [first_row[w], first_row[w + 1]).
// Row f is the first row of every w with seg(f - 1) < w * epw <= seg(f), so
// each first_row entry has exactly one writer.  n_warps is the grid's
// capacity; warps past the last entry get empty ranges (first_row = T).
__global__ void warp_ranges_kernel(const int32_t* __restrict__ seg_start, int32_t T, int32_t P, int32_t epw,
                                   int32_t n_warps, int32_t* __restrict__ first_row) {
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f > T) return;
  const int64_t prev = f == 0 ? -1 : seg_start[(f - 1) * P];
  const int64_t lo = f == 0 ? 0 : prev / epw + 1;
  const int64_t hi = f == T ? n_warps : seg_start[f * P] / epw;
  for (int64_t w = lo; w <= hi && w <= n_warps; ++w) first_row[w] = (int32_t)f;
}

// ----------------------------------------------------------------------------
// Segment sums.  Sorted values encode (perspective, position) as
// perspective * B + b, so a load can be issued from the value alone.
// ----------------------------------------------------------------------------
struct SegParams {
  const float* dout[2];       // [B, C] per perspective
  const int32_t* sorted_b;    // perspective * B + position, grouped by key, ascending within a key
  const int32_t* seg_start;   // [T * P + 1]
  const int32_t* heavy_list;  // walk path only
  const int32_t* n_heavy;
  const uint8_t* row_kind;
  const int32_t* first_row;   // stream path: [n_stream_warps + 1]
  float* dW;                  // [T, C]
  int64_t B;                  // positions per perspective
  int32_t T;
  int32_t P;
  int32_t accumulate;         // 0: dW[f] = sum (all rows written); 1: dW[f] += sum (touched rows)
  int32_t heavy_cap;
  int32_t chunk0;             // first column chunk of this launch (blockIdx.y offset)
  int32_t n_stream_warps;
  int32_t row_begin;          // rows [row_begin, row_end) of dW are produced by this call
  int32_t row_end;
  Geom g;
};

// Decodes a sorted value of perspective q; out-of-range values (a corrupt
// workspace) are flagged and returned as -1, never dereferenced.
__device__ __forceinline__ int decode_position(int v, int q, int64_t B) {
  const int64_t b = (int64_t)v - (int64_t)q * B;
  if ((unsigned long long)b >= (unsigned long long)B) {
    flag_error(kErrBadSegment);
    return -1;
  }
  return (int)b;
}

template <typename VT, int V>
__device__ __forceinline__ void seg_write(const SegParams& p, int64_t f, int col, const VT (&tot)[V],
                                          const bool (&ok)[V], bool touched) {
  using Ops = Vec<VT>;
  VT* dst = reinterpret_cast<VT*>(p.dW) + f * (int64_t)p.g.n_vec + col;
  if (p.accumulate) {
    if (!touched) return;
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (ok[v]) {
        VT cur = dst[32 * v];
        Ops::add(cur, tot[v]);
        dst[32 * v] = cur;
      }
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (ok[v]) dst[32 * v] = tot[v];
  }
}

// acc[v] += dOut_q[b, cols] for the entries of sorted_b[s, e) (perspective q),
// ascending, where `my` already holds the decoded first 32 positions
// (lane i: entry s + i).  Later groups of 32 are loaded as needed.
template <typename VT, int V, int U>
__device__ __forceinline__ void seg_sum(VT (&acc)[V], const VT* __restrict__ src, int64_t row_vec,
                                                  const int32_t* __restrict__ sb, int s, int e, int q, int64_t B,
                                                  int my, const bool (&ok)[V], int lane) {
  using Ops = Vec<VT>;
  for (int j0 = s; j0 < e; j0 += 32) {
    const int cnt = e - j0 < 32 ? e - j0 : 32;
    if (j0 != s) my = lane < cnt ? decode_position(__ldg(sb + j0 + lane), q, B) : -1;
    for (int u0 = 0; u0 < cnt; u0 += U) {
      int rows[U];
      bool has[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        rows[u] = __shfl_sync(kFull, my, (u0 + u) & 31);
        has[u] = u0 + u < cnt && rows[u] >= 0;
      }
      VT w[U][V];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (has[u] && ok[v]) w[u][v] = Ops::ldg(src + (int64_t)rows[u] * row_vec + 32 * v);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (has[u] && ok[v]) Ops::add(acc[v], w[u][v]);
    }
  }
}

// Light rows: one warp per (row, column chunk), U dOut rows in flight per
// batch, positions broadcast from registers with __shfl_sync.  The row's
// segment bounds (both perspectives) and its heavy flag arrive in ONE round
// trip and the first 32 positions of both perspectives in a second, so a
// row costs two dependent round trips before its data batches start.  The
// kernel is latency-bound: the bytes in flight per SM are resident warps x U
// x one 512-byte row slice, so MINB (resident blocks the register budget is
// sized for) matters as much as U.  Heavy rows are left to
// ft_segsum_heavy_kernel.
template <typename VT, int V, int U, int MINB = 1>
__global__ void __launch_bounds__(kBlock, MINB) ft_segsum_light_kernel(const SegParams p) {
  using Ops = Vec<VT>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);
  const int64_t row_vec = p.g.n_vec;
  const int64_t f = p.row_begin + (int64_t)blockIdx.x * kWarpsPerBlock + warp;
  if (f >= p.row_end) return;
  const int P = p.P;
  const int bnd = lane <= P ? p.seg_start[f * P + lane] : 0;
  const int kind = p.row_kind[f];
  const int s0 = __shfl_sync(kFull, bnd, 0);
  const int s1 = __shfl_sync(kFull, bnd, 1);
  const int e1 = __shfl_sync(kFull, bnd, P);
  if (kind) return;
  const int g0 = s0 + lane < s1 ? decode_position(__ldg(p.sorted_b + s0 + lane), 0, p.B) : -1;
  const int g1 = (P == 2 && s1 + lane < e1) ? decode_position(__ldg(p.sorted_b + s1 + lane), 1, p.B) : -1;
  bool ok[V];
#pragma unroll
  for (int v = 0; v < V; ++v) ok[v] = lane + 32 * v < width;
  VT tot[V];
#pragma unroll
  for (int v = 0; v < V; ++v) tot[v] = Ops::zero();
  seg_sum<VT, V, U>(tot, reinterpret_cast<const VT*>(p.dout[0]) + c0 + lane, row_vec, p.sorted_b, s0, s1,
                              0, p.B, g0, ok, lane);
  if (P == 2) {
    VT acc1[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc1[v] = Ops::zero();
    seg_sum<VT, V, U>(acc1, reinterpret_cast<const VT*>(p.dout[1]) + c0 + lane, row_vec, p.sorted_b, s1,
                                e1, 1, p.B, g1, ok, lane);
#pragma unroll
    for (int v = 0; v < V; ++v) Ops::add(tot[v], acc1[v]);
  }
  seg_write<VT, V>(p, f, c0 + lane, tot, ok, e1 > s0);
}

// Heavy rows of the fallback path: one warp per 32-vector piece of a column
// chunk streams the row's dOut slices through a kHeavyStages-deep ring.
constexpr int kHeavyWarps = 2;
constexpr int kHeavyStages = 48;

template <typename VT>
__global__ void __launch_bounds__(32 * kHeavyWarps) ft_segsum_heavy_kernel(const SegParams p) {
  using Ops = Vec<VT>;
  extern __shared__ __align__(16) unsigned char heavy_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  VT* ring = reinterpret_cast<VT*>(heavy_smem) + warp * kHeavyStages * 32 + lane;
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);
  const int pieces = (width + 31) / 32;
  const int wi = blockIdx.x * kHeavyWarps + warp;
  const int slot = wi / pieces, piece = wi - slot * pieces;
  const int nh = *p.n_heavy < p.heavy_cap ? *p.n_heavy : p.heavy_cap;
  if (slot >= nh) return;
  const int64_t f = p.heavy_list[slot];
  if (f < p.row_begin || f >= p.row_end) return;
  const int col = c0 + piece * 32 + lane;
  const bool ok1 = piece * 32 + lane < width;
  const int64_t row_vec = p.g.n_vec;

  VT tot = Ops::zero();
  for (int q = 0; q < p.P; ++q) {
    const int s = p.seg_start[f * p.P + q], e = p.seg_start[f * p.P + q + 1];
    const VT* src = reinterpret_cast<const VT*>(q ? p.dout[1] : p.dout[0]) + (ok1 ? col : 0);
    VT acc = Ops::zero();
    int t = s;  // issue pointer, kHeavyStages entries ahead of the consume pointer
    int idx_base = -1, my_b = -1;
    auto issue = [&](int slot_i) {
      if (t < e) {
        const int base = t & ~31;
        if (base != idx_base) {
          idx_base = base;
          my_b = base + lane < e && base + lane >= s ? decode_position(__ldg(p.sorted_b + base + lane), q, p.B) : -1;
        }
        const int b = __shfl_sync(kFull, my_b, t & 31);
        cp_async_vec<VT>(ring + slot_i * 32, src + (b >= 0 ? (int64_t)b * row_vec : 0), ok1 && b >= 0);
      }
      cp_async_commit();  // empty groups keep the pending count constant
      ++t;
    };
    for (int i = 0; i < kHeavyStages; ++i) issue(i);
    for (int j = s, stage = 0; j < e; ++j) {
      cp_async_wait<kHeavyStages - 1>();
      Ops::add(acc, ring[stage * 32]);
      __syncwarp();
      issue(stage);
      stage = stage + 1 == kHeavyStages ? 0 : stage + 1;
    }
    cp_async_wait<0>();
    if (q == 0) tot = acc;
    else Ops::add(tot, acc);
  }
  const bool ok[1] = {ok1};
  const VT t1[1] = {tot};
  seg_write<VT, 1>(p, f, col, t1, ok, true);
}

// ---------------------------------------------------------------------------
// Streaming segment sums (fast path: 16-byte vectors, chunks of <= 32 x SV
// vectors).  Each warp owns a contiguous range of rows holding about
// `entries per warp` entries; because rows are in key order, their entries
// are one contiguous run of the sorted list.  The warp streams that run
// through a lane-private cp.async ring kStreamStages entries deep (SV
// vectors per lane per entry), adding each arriving dOut slice to the
// current (row, perspective) accumulator and finishing a row when its last
// segment ends -- the pipeline never drains between rows, and hot rows need
// no special path.  Values decode to (perspective, position) at issue time;
// the consume side walks the segment table, 32 boundaries per load.
// ---------------------------------------------------------------------------
// 16-byte cp.async, skipped entirely when !pred (the destination keeps its
// old bytes; callers never use them).
__device__ __forceinline__ void cp_async16_if(float4* smem_dst, const float4* gsrc, bool pred) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p cp.async.cg.shared.global [%0], [%1], 16;\n}\n" ::"r"(d),
      "l"(gsrc), "r"((int)pred)
      : "memory");
}

// S: ring stages per warp, G: entries per commit group, WPB: warps per block.
template <int SV, int S, int G, int WPB>
__global__ void __launch_bounds__(32 * WPB) ft_segsum_stream_kernel(const SegParams p) {
  using Ops = Vec<float4>;
  static_assert(S % G == 0, "stages must be a multiple of the group size");
  extern __shared__ __align__(16) unsigned char stream_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4* ring = reinterpret_cast<float4*>(stream_smem) + (warp * S * SV) * 32 + lane;
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);
  bool ok[SV];
#pragma unroll
  for (int v = 0; v < SV; ++v) ok[v] = lane + 32 * v < width;
  const int w = blockIdx.x * WPB + warp;
  if (w >= p.n_stream_warps) return;
  const int f_begin = p.first_row[w], f_end = p.first_row[w + 1];
  if (f_begin >= f_end) return;
  const int64_t row_vec = p.g.n_vec;
  const int P = p.P;
  const int Bi = (int)p.B;
  const float4* __restrict__ d0 = reinterpret_cast<const float4*>(p.dout[0]) + c0 + lane;
  const float4* __restrict__ d1 = reinterpret_cast<const float4*>(P == 2 ? p.dout[1] : p.dout[0]) + c0 + lane;
  const int E0 = p.seg_start[(int64_t)f_begin * P];
  const int E1 = p.seg_start[(int64_t)f_end * P];

  // ---- issue side: entry t -> ring slot (t - E0) % S, G entries per group
  int t = E0, idx_base = -1, my_v = 0;
  auto issue = [&](int slot_i) {
    if (t < E1) {
      const int base = t & ~31;
      if (base != idx_base) {
        idx_base = base;
        my_v = base + lane < E1 ? __ldg(p.sorted_b + base + lane) : 0;
      }
      const int v = __shfl_sync(kFull, my_v, t & 31);
      const int q = v >= Bi ? 1 : 0;
      const int b = v - q * Bi;
      const bool good = (unsigned)b < (unsigned)Bi;
      if (!good) flag_error(kErrBadSegment);
      const float4* src = (q ? d1 : d0) + (good ? (int64_t)b * row_vec : 0);
#pragma unroll
      for (int s = 0; s < SV; ++s) cp_async16_if(ring + (slot_i * SV + s) * 32, src + 32 * s, ok[s] && good);
    }
    ++t;
  };
#pragma unroll 1
  for (int i = 0; i < S; i += G) {
#pragma unroll
    for (int e = 0; e < G; ++e) issue(i + e);
    cp_async_commit();
  }

  // ---- consume side: segment boundaries of keys [f_begin * P, f_end * P]
  int key = f_begin * P;
  int bnd_base = -1, my_bnd = 0;
  auto seg_end = [&](int k) {  // end of segment k = seg_start[k + 1]
    const int idx = k + 1;
    const int base = idx & ~31;
    if (base != bnd_base) {
      bnd_base = base;
      my_bnd = p.seg_start[base + lane < p.T * P + 1 ? base + lane : p.T * P];
    }
    return __shfl_sync(kFull, my_bnd, idx & 31);
  };
  float4 acc[SV], tot[SV];
#pragma unroll
  for (int s = 0; s < SV; ++s) acc[s] = tot[s] = Ops::zero();
  int end = seg_end(key);
  int row_first = E0;
  int j = E0, stage = 0;
  bool done = false;
  while (!done) {
    cp_async_wait<S / G - 1>();  // the oldest group (G entries) has landed
#pragma unroll
    for (int e = 0; e < G; ++e) {
      // close every segment that ends at j (empty segments and rows included)
      while (!done && end == j) {
        const int q = key - (key / P) * P;
        if (q == 0) {
#pragma unroll
          for (int s = 0; s < SV; ++s) tot[s] = acc[s];
        } else {
#pragma unroll
          for (int s = 0; s < SV; ++s) Ops::add(tot[s], acc[s]);
        }
#pragma unroll
        for (int s = 0; s < SV; ++s) acc[s] = Ops::zero();
        if (q == P - 1) {
          const int64_t f = key / P;
          seg_write<float4, SV>(p, f, c0 + lane, tot, ok, j > row_first);
          row_first = j;
          if (f + 1 >= f_end) done = true;
        }
        if (!done) {
          ++key;
          end = seg_end(key);
        }
      }
      // a segment table that is not monotone (corrupt workspace) ends the walk
      if (!done && (end < j || (j >= E1 && end != j))) {
        flag_error(kErrBadSegment);
        done = true;
      }
      if (!done && j < E1) {
#pragma unroll
        for (int s = 0; s < SV; ++s) Ops::add(acc[s], ring[((stage + e) * SV + s) * 32]);
        ++j;
      }
    }
    if (done) break;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < G; ++e) issue(stage + e);
    cp_async_commit();
    stage = stage + G == S ? 0 : stage + G;
  }
  cp_async_wait<0>();
}

// ----------------------------------------------------------------------------
// Bias gradient: deterministic column sum over positions, both perspectives.
// Accumulated in float64 (partials over position ranges, then a fixed-order
// warp tree), so each perspective's sum is within half an fp32 ulp of the
// exact value; the two perspectives are then rounded and added in fp32, the
// way autograd adds the reference's two bias gradients (kernel.py:269).
// torch's own reduction order cannot be reproduced, so this is the closest
// any implementation can get to it.
// ----------------------------------------------------------------------------
struct ColParams {
  const float* dout[2];
  int64_t B;
  int32_t P;
  int32_t C;         // floats per row
  int32_t parts;
  int32_t vec4;      // rows are float4-loadable
  double* partial;   // [P][parts][C]
};

__global__ void __launch_bounds__(kBlock) colsum_partial_kernel(const ColParams p) {
  const int part = blockIdx.x, q = blockIdx.y;
  const int64_t r0 = p.B * part / p.parts, r1 = p.B * (part + 1) / p.parts;
  const float* __restrict__ src = q ? p.dout[1] : p.dout[0];
  double* dst = p.partial + ((int64_t)q * p.parts + part) * p.C;
  if (p.vec4) {
    const int n4 = p.C / 4;
    for (int c4 = threadIdx.x; c4 < n4; c4 += blockDim.x) {
      double a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      int64_t r = r0;
      for (; r + 4 <= r1; r += 4) {
        float4 t[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) t[i] = __ldg(reinterpret_cast<const float4*>(src + (r + i) * p.C) + c4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a0 += t[i].x;
          a1 += t[i].y;
          a2 += t[i].z;
          a3 += t[i].w;
        }
      }
      for (; r < r1; ++r) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(src + r * p.C) + c4);
        a0 += t.x;
        a1 += t.y;
        a2 += t.z;
        a3 += t.w;
      }
      dst[4 * c4 + 0] = a0;
      dst[4 * c4 + 1] = a1;
      dst[4 * c4 + 2] = a2;
      dst[4 * c4 + 3] = a3;
    }
  } else {
    for (int c = threadIdx.x; c < p.C; c += blockDim.x) {
      double a = 0;
      for (int64_t r = r0; r < r1; ++r) a += __ldg(src + r * p.C + c);
      dst[c] = a;
    }
  }
}

// One warp per column: lanes take parts lane, lane+32, ... in order, then a
// fixed xor-tree; the result is deterministic.
__global__ void __launch_bounds__(kBlock) colsum_final_kernel(const double* __restrict__ partial, int32_t P,
                                                              int32_t parts, int32_t C, float* dB,
                                                              int32_t accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t c = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (c >= C) return;
  float tot = 0.f;
  for (int q = 0; q < P; ++q) {
    double s = 0;
    for (int i = lane; i < parts; i += 32) s += partial[((int64_t)q * parts + i) * C + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
    const float sf = (float)s;
    tot = q == 0 ? sf : tot + sf;
  }
  if (lane == 0) dB[c] = accumulate ? dB[c] + tot : tot;
}

}  // namespace nnue
