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
//   1. index phase: key = f * P + perspective, value = perspective * B + b.
//      A counting placement builds, for every key, the list of its positions
//      in ascending b (the stable sort's order) plus the segment offsets
//      seg_start (below: count, scan, place, order).
//   2. classify: rows with more than `heavy_threshold` entries go to a heavy
//      list (bounded); their work is split finer and runs beside the rest.
//   3. segsum: one warp per (row, column chunk); heavy rows one warp per
//      (row, 32-vector piece, perspective).  Every row of dW is written
//      exactly once (rows no position touches get 0), which replaces
//      torch.zeros + read-modify-write.
//   4. bias: deterministic column sum (per-part partials, fixed-order combine).
#pragma once

#include "common.cuh"

namespace nnue {

// ----------------------------------------------------------------------------
// Exclusive scan (int32), reduce-then-scan in three launches.
// ----------------------------------------------------------------------------
struct ScanLen {
  int64_t n;  // elements
};

__device__ __forceinline__ int64_t scan_length(const ScanLen& L) { return L.n; }

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
// The raw [B, K] index arrays of both perspectives
// ----------------------------------------------------------------------------
struct RawSrc {
  const int32_t* idx[2];  // [B, K] per perspective
  int64_t n_raw;          // B * K
  int32_t K;
  int32_t T;
  int32_t P;
};

// ----------------------------------------------------------------------------
// Counting placement: per key, the list of its positions in ascending b (the
// order of the reference's stable sort), built as a sparse transpose.
//   count : one pass over the raw index arrays, seg[key] += 1 per valid slot
//   scan  : exclusive scan -> seg_start; cursor = copy of seg_start
//   place : second pass; slot = atomicAdd(cursor[key], 1), values land in
//           their key's segment in arbitrary order
//   order : every segment is sorted ascending (values of one key share the
//           perspective, so ascending value = ascending b).  Equal values are
//           the same position twice, so the order among them cannot change
//           any sum; the result equals the stable sort.
//           n <= 256: one warp, bitonic network in registers;
//           n <= kSegSmem: one block, bitonic network in shared memory;
//           larger: one block counts positions in shared-memory windows.
// ----------------------------------------------------------------------------
// The raw slots of perspective q, four at a time when aligned.
struct RawCursor {
  const int32_t* base;
  int64_t n;
  bool vec4;
};

__device__ __forceinline__ RawCursor raw_cursor(const RawSrc& r, int q) {
  const int32_t* b = q ? r.idx[1] : r.idx[0];
  return RawCursor{b, r.n_raw, (reinterpret_cast<uintptr_t>(b) & 15) == 0};
}

// Calls fn(e, f) for every slot e of perspective q in this thread's share.
template <typename Fn>
__device__ __forceinline__ void for_raw_slots(const RawCursor& c, int64_t tid, int64_t nthreads, Fn&& fn) {
  if (c.vec4) {
    const int64_t n4 = c.n >> 2;
    const int4* b4 = reinterpret_cast<const int4*>(c.base);
    for (int64_t i = tid; i < n4; i += nthreads) {
      const int4 v = __ldcs(b4 + i);
      fn(4 * i, v.x);
      fn(4 * i + 1, v.y);
      fn(4 * i + 2, v.z);
      fn(4 * i + 3, v.w);
    }
    for (int64_t e = 4 * n4 + tid; e < c.n; e += nthreads) fn(e, __ldcs(c.base + e));
  } else {
    for (int64_t e = tid; e < c.n; e += nthreads) fn(e, __ldcs(c.base + e));
  }
}

__global__ void __launch_bounds__(kBlock) count_keys_kernel(const RawSrc r, int32_t* __restrict__ seg) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int q = 0; q < r.P; ++q) {
    const RawCursor c = raw_cursor(r, q);
    for_raw_slots(c, tid, nthreads, [&](int64_t, int f) {
      if ((unsigned)f < (unsigned)r.T) atomicAdd(seg + (int64_t)f * r.P + q, 1);
      else if (f != -1) flag_error(kErrBadIndex);
    });
  }
}

__global__ void __launch_bounds__(kBlock) place_keys_kernel(const RawSrc r, int32_t* __restrict__ cursor,
                                                           int32_t* __restrict__ vals, int64_t cap) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t B = r.K > 0 ? r.n_raw / r.K : 0;
  for (int q = 0; q < r.P; ++q) {
    const RawCursor c = raw_cursor(r, q);
    for_raw_slots(c, tid, nthreads, [&](int64_t e, int f) {
      if ((unsigned)f >= (unsigned)r.T) return;
      const int pos = atomicAdd(cursor + (int64_t)f * r.P + q, 1);
      if ((unsigned long long)(unsigned)pos < (unsigned long long)cap) vals[pos] = (int)(q * B + e / r.K);
      else flag_error(kErrBadSegment);
    });
  }
}

// Ascending bitonic sort of the n <= 32 * E values at data[0, n), one warp,
// blocked layout (lane l holds elements l * E .. l * E + E - 1).
template <int E>
__device__ __forceinline__ void warp_sort_segment(int32_t* __restrict__ data, int n, int lane) {
  constexpr int N = 32 * E;
  int v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    v[e] = i < n ? data[i] : INT32_MAX;
  }
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= E) {  // partner element in lane ^ (j / E), same slot
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = lane * E + e;
          const int other = __shfl_xor_sync(kFull, v[e], j / E);
          const bool up = (i & k) == 0, lower = (i & j) == 0;
          v[e] = (lower == up) ? min(v[e], other) : max(v[e], other);
        }
      } else {  // partner slot e ^ j in this lane
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if (e & j) continue;
          const bool up = ((lane * E + e) & k) == 0;
          const int a = v[e], b = v[e ^ j];
          v[e] = up ? min(a, b) : max(a, b);
          v[e ^ j] = up ? max(a, b) : min(a, b);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    if (i < n) data[i] = v[e];
  }
}

// One warp per key: segments of <= 256 values are sorted here, longer ones
// are listed for order_big_segments_kernel (big[0] = count, big[1..] = keys).
__global__ void __launch_bounds__(kBlock) order_segments_kernel(const int32_t* __restrict__ seg, int64_t NK,
                                                               int32_t* __restrict__ vals, int32_t* __restrict__ big) {
  const int lane = threadIdx.x & 31;
  const int64_t key = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (key >= NK) return;
  const int s = seg[key], n = seg[key + 1] - s;
  if (n <= 1) return;
  if (n <= 32) {
    // placement often leaves short segments in order already
    const int v = lane < n ? vals[s + lane] : INT32_MAX;
    const int next = __shfl_down_sync(kFull, v, 1);
    if (__all_sync(kFull, lane >= n - 1 || v <= next)) return;
  }
  if (n <= 32) warp_sort_segment<1>(vals + s, n, lane);
  else if (n <= 64) warp_sort_segment<2>(vals + s, n, lane);
  else if (n <= 128) warp_sort_segment<4>(vals + s, n, lane);
  else if (n <= 256) warp_sort_segment<8>(vals + s, n, lane);
  else if (lane == 0) big[1 + atomicAdd(big, 1)] = (int32_t)key;
}

constexpr int kSegSmem = 8192;      // values sorted in shared memory by one block
constexpr int kSegWindow = 16384;   // positions counted per window (16-bit counters, two per word)
constexpr int kBigThreads = 512;

// One block per long segment.  Either a bitonic network over the values in
// shared memory, or a counting sort by position, kSegWindow positions per
// window (the values of one key lie in [v0, v0 + B)); the cheaper one by
// operation count is taken.  The count reads a copy of the segment in
// `spare` (an int array as long as `vals`).  Counters are 16-bit: the host
// only selects this path when max_active < 65536, so no (key, position)
// pair can repeat more often.
__global__ void __launch_bounds__(kBigThreads) order_big_segments_kernel(const int32_t* __restrict__ seg,
                                                                        int32_t P, int64_t B,
                                                                        int32_t* __restrict__ vals,
                                                                        int32_t* __restrict__ spare,
                                                                        const int32_t* __restrict__ big) {
  __shared__ uint32_t sm[kSegSmem > kSegWindow / 2 ? kSegSmem : kSegWindow / 2];
  __shared__ int scratch[33];
  const int n_big = big[0];
  const int64_t windows = (B + kSegWindow - 1) / kSegWindow;
  for (int bi = blockIdx.x; bi < n_big; bi += gridDim.x) {
    const int64_t key = big[1 + bi];
    const int s = seg[key], n = seg[key + 1] - s;
    int32_t* d = vals + s;
    int N = 1, lg = 0;
    while (N < n) {
      N <<= 1;
      ++lg;
    }
    const bool network = n <= kSegSmem && (int64_t)lg * (lg + 1) / 2 * N < windows * ((int64_t)n + kSegWindow);
    if (network) {
      int32_t* si = reinterpret_cast<int32_t*>(sm);
      for (int i = threadIdx.x; i < N; i += blockDim.x) si[i] = i < n ? d[i] : INT32_MAX;
      __syncthreads();
      for (int k = 2; k <= N; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
          for (int i = threadIdx.x; i < N; i += blockDim.x) {
            const int x = i ^ j;
            if (x > i) {
              const int a = si[i], b = si[x];
              const bool up = (i & k) == 0;
              if ((a > b) == up) {
                si[i] = b;
                si[x] = a;
              }
            }
          }
          __syncthreads();
        }
      for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = si[i];
    } else {
      int32_t* src = spare + s;
      for (int i = threadIdx.x; i < n; i += blockDim.x) src[i] = d[i];
      __syncthreads();
      const int64_t v0 = (key % P) * B;
      int out = 0;
      for (int64_t w0 = 0; w0 < B; w0 += kSegWindow) {
        for (int i = threadIdx.x; i < kSegWindow / 2; i += blockDim.x) sm[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
          const int64_t b = (int64_t)src[i] - v0 - w0;
          if (b >= 0 && b < kSegWindow) atomicAdd(&sm[b >> 1], 1u << (16 * (int)(b & 1)));
        }
        __syncthreads();
        constexpr int kWords = kSegWindow / 2 / kBigThreads;  // counter words per thread
        uint32_t c[kWords];
        int tsum = 0;
#pragma unroll
        for (int t = 0; t < kWords; ++t) {
          c[t] = sm[threadIdx.x * kWords + t];
          tsum += (int)(c[t] & 0xffffu) + (int)(c[t] >> 16);
        }
        const int incl = block_inclusive_scan(tsum, scratch);
        const int total = scratch[32];
        int o = out + incl - tsum;
#pragma unroll
        for (int t = 0; t < kWords; ++t) {
          const int value = (int)(v0 + w0 + 2 * (threadIdx.x * kWords + t));
          const int c0 = (int)(c[t] & 0xffffu), c1 = (int)(c[t] >> 16);
          for (int r = 0; r < c0; ++r)
            if (o + r < n) d[o + r] = value;
          o += c0;
          for (int r = 0; r < c1; ++r)
            if (o + r < n) d[o + r] = value + 1;
          o += c1;
        }
        out += total;
        __syncthreads();
      }
      if (out != n && threadIdx.x == 0) flag_error(kErrBadSegment);
    }
    __syncthreads();
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
  float* dW;                  // [T, C]
  int64_t B;                  // positions per perspective
  int32_t T;
  int32_t P;
  int32_t accumulate;         // 0: dW[f] = sum (all rows written); 1: dW[f] += sum (touched rows)
  int32_t heavy_cap;
  int32_t chunk0;             // first column chunk of this launch (blockIdx.y offset)
  int32_t row_begin;          // rows [row_begin, row_end) of dW are produced by this call
  int32_t row_end;
  Geom g;
  TableSet dws;               // n > 1: dW split over separately allocated row blocks (dW unused)
  float* heavy_part;          // [heavy_cap, 2, n_vec] vectors: per-perspective sums of heavy rows
  unsigned* heavy_ticket;     // [heavy_cap, heavy_ticket_stride]: pair tickets (one per piece), zeroed per call
  int32_t heavy_ticket_stride;
  int32_t persp_delta;        // queued light rows: dout[1] - dout[0] in vectors (the host checked the range)
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
  VT* dst;
  if (p.dws.n > 1) {
    const int t = p.dws.find(f);
    dst = reinterpret_cast<VT*>(p.dws.base[t]) + (f - p.dws.start(t)) * (int64_t)p.g.n_vec + col;
  } else {
    dst = reinterpret_cast<VT*>(p.dW) + f * (int64_t)p.g.n_vec + col;
  }
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

// Row offset (in vectors) of the position stored in a sorted value of
// perspective q: (v - q * B) * row_vec.  Values outside the perspective's
// range (a corrupt workspace) are flagged and read row 0 instead, so every
// load stays in bounds.  The host guarantees B * row_vec < 2^31.
__device__ __forceinline__ int position_offset(int v, int q, int64_t B, int row_vec) {
  int b = v - q * (int)B;
  if ((unsigned)b >= (unsigned)B) {
    flag_error(kErrBadSegment);
    b = 0;
  }
  return b * row_vec;
}

// acc[v] += dOut_q[b, cols] for the entries of sorted_b[s, e) (perspective q),
// ascending, where `my` already holds the row offsets of the first 32
// entries (lane i: entry s + i).  Later groups of 32 are loaded as needed.
// Full batches of U entries run without per-entry checks; only the last
// batch of a group is predicated.
template <typename VT, int V, int U>
__device__ __forceinline__ void seg_sum(VT (&acc)[V], const VT* __restrict__ src, int row_vec,
                                        const int32_t* __restrict__ sb, int s, int e, int q, int64_t B, int my,
                                        const bool (&ok)[V], int lane) {
  using Ops = Vec<VT>;
  for (int j0 = s; j0 < e; j0 += 32) {
    const int cnt = e - j0 < 32 ? e - j0 : 32;
    if (j0 != s) my = lane < cnt ? position_offset(__ldg(sb + j0 + lane), q, B, row_vec) : 0;
    int u0 = 0;
#pragma unroll 1
    for (; u0 + U <= cnt; u0 += U) {
      VT w[U][V];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = __shfl_sync(kFull, my, u0 + u);
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (ok[v]) w[u][v] = Ops::ldg(src + o + 32 * v);
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (ok[v]) Ops::add(acc[v], w[u][v]);
    }
    if (u0 < cnt) {
      VT w[U][V];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int o = __shfl_sync(kFull, my, (u0 + u) & 31);
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (u0 + u < cnt && ok[v]) w[u][v] = Ops::ldg(src + o + 32 * v);
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int v = 0; v < V; ++v)
          if (u0 + u < cnt && ok[v]) Ops::add(acc[v], w[u][v]);
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
template <typename VT, int V, int U, int MINB = 1, int BLOCK = kBlock>
__global__ void __launch_bounds__(BLOCK, MINB) ft_segsum_light_kernel(const SegParams p) {
  using Ops = Vec<VT>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const int width = p.g.width(chunk);
  const int row_vec = p.g.n_vec;
  const int64_t f = p.row_begin + (int64_t)blockIdx.x * (BLOCK / 32) + warp;
  if (f >= p.row_end) return;
  const int P = p.P;
  const int bnd = lane <= P ? p.seg_start[f * P + lane] : 0;
  const int kind = p.row_kind[f];
  const int s0 = __shfl_sync(kFull, bnd, 0);
  const int s1 = __shfl_sync(kFull, bnd, 1);
  const int e1 = __shfl_sync(kFull, bnd, P);
  if (kind) return;
  const int g0 = s0 + lane < s1 ? position_offset(__ldg(p.sorted_b + s0 + lane), 0, p.B, row_vec) : 0;
  const int g1 = (P == 2 && s1 + lane < e1) ? position_offset(__ldg(p.sorted_b + s1 + lane), 1, p.B, row_vec) : 0;
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

// Light rows, queued: one warp per (row, column chunk of <= 32 vectors), the
// form used when each lane owns one 16-byte vector.  A row's entries of both
// perspectives are contiguous in sorted_b ([s0, s1) perspective 0, [s1, e1)
// perspective 1).  Up to kQueueList of them are loaded in one round trip and
// turned into 32-bit row offsets from dout[0] (perspective 1 adds
// persp_delta, the distance to dout[1] in vectors -- the host checked every
// such offset fits in int32) in a per-warp shared-memory list; each lane
// adds them to its own column pointer.  Each perspective's rows then stream through a D-slot register
// queue, as in the forward: consuming slot d re-issues it with the entry D
// further on, so D row slices stay in flight during the walk.  Perspective
// 0's sum is parked in shared memory while perspective 1 is walked with the
// same registers.  Each perspective is summed from zero in ascending b and
// dW = acc0 + acc1 is written once: the same adds, in the same order, as
// ft_segsum_light_kernel.
constexpr int kQueueList = 256;

// Offsets of entries [first, first + m) (m <= kQueueList) of the row starting
// at s0 into list[0, m).  Entries at or past n0 belong to perspective 1.
__device__ __forceinline__ void queue_offsets(const SegParams& p, int* list, int s0, int first, int m, int n0,
                                              int lane) {
  const int B = (int)p.B;  // the host guarantees B * row_vec < 2^31
  const int row_vec = p.g.n_vec;
  int v[kQueueList / 32];
  const int32_t* __restrict__ sbp = p.sorted_b + (s0 + first) + lane;
#pragma unroll
  for (int g = 0; g < kQueueList / 32; ++g) v[g] = g * 32 + lane < m ? __ldg(sbp + g * 32) : 0;
#pragma unroll
  for (int g = 0; g < kQueueList / 32; ++g) {
    const int j = g * 32 + lane;
    if (j < m) {
      const bool q = first + j >= n0;
      int b = v[g] - (q ? B : 0);
      if ((unsigned)b >= (unsigned)B) {  // corrupt workspace: flag, read row 0
        flag_error(kErrBadSegment);
        b = 0;
      }
      list[j] = b * row_vec + (q ? p.persp_delta : 0);
    }
  }
  __syncwarp();
}

// acc + the rows at src + list[lo, hi), added one by one in list order.
template <int D>
__device__ __forceinline__ float4 queue_sum(const float4* __restrict__ src, const int* list, int lo, int hi,
                                            bool ok, float4 acc) {
  using Ops = Vec<float4>;
  float4 w[D];
#pragma unroll
  for (int d = 0; d < D; ++d)
    if (lo + d < hi && ok) w[d] = Ops::ldg(src + list[lo + d]);
  int j = lo;
  for (; j + 2 * D <= hi; j += D) {  // every slot consumed and re-issued in range
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (ok) {
        Ops::add(acc, w[d]);
        w[d] = Ops::ldg(src + list[j + d + D]);
      }
  }
  for (; j < hi; j += D) {
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (ok) {
        if (j + d < hi) Ops::add(acc, w[d]);
        if (j + d + D < hi) w[d] = Ops::ldg(src + list[j + d + D]);
      }
  }
  return acc;
}

// Sum (from zero, in order) of entries [lo, hi) of a row longer than the
// list -- only when rows past the heavy-row cap stay light, or with a raised
// heavy-row threshold -- one entry at a time, straight from sorted_b (few
// registers, so this path does not set the kernel's register budget).
__device__ __forceinline__ float4 queue_sum_long(const int32_t* __restrict__ sorted_b, int B, int row_vec,
                                              int persp_delta, const float4* __restrict__ src, int s0, int lo,
                                              int hi, int n0, bool ok, int lane) {
  using Ops = Vec<float4>;
  float4 acc = Ops::zero();
  for (int j0 = lo; j0 < hi; j0 += 32) {
    const int cnt = hi - j0 < 32 ? hi - j0 : 32;
    int o = 0;
    if (lane < cnt) {
      const bool q = j0 + lane >= n0;
      int b = __ldg(sorted_b + s0 + j0 + lane) - (q ? B : 0);
      if ((unsigned)b >= (unsigned)B) {
        flag_error(kErrBadSegment);
        b = 0;
      }
      o = b * row_vec + (q ? persp_delta : 0);
    }
    for (int u = 0; u < cnt; ++u) {
      const int ou = __shfl_sync(kFull, o, u);
      if (ok) Ops::add(acc, Ops::ldg(src + ou));
    }
  }
  return acc;
}

// acc + the rows at src + (lane u's `g`) for u in [0, n), n <= 32: the same
// queue fed from a register group of offsets by shuffles (short rows: no
// shared-memory round trip before the first row load).
template <int D>
__device__ __forceinline__ float4 queue_sum_regs(const float4* __restrict__ src, int g, int n, bool ok,
                                                 float4 acc) {
  using Ops = Vec<float4>;
  float4 w[D];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    const int o = __shfl_sync(kFull, g, d);
    if (d < n && ok) w[d] = Ops::ldg(src + o);
  }
  int j = 0;
  for (; j + 2 * D <= n; j += D) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int o = __shfl_sync(kFull, g, j + d + D);
      if (ok) {
        Ops::add(acc, w[d]);
        w[d] = Ops::ldg(src + o);
      }
    }
  }
  for (; j < n; j += D) {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      const int o = __shfl_sync(kFull, g, (j + d + D) & 31);
      if (ok) {
        if (j + d < n) Ops::add(acc, w[d]);
        if (j + d + D < n) w[d] = Ops::ldg(src + o);
      }
    }
  }
  return acc;
}

template <int D, int MINB, int BLOCK>
__global__ void __launch_bounds__(BLOCK, MINB) ft_segsum_lightq_kernel(const SegParams p) {
  __shared__ int s_list[BLOCK / 32][kQueueList];
  __shared__ float4 s_park[BLOCK / 32][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* list = s_list[warp];
  const int chunk = p.chunk0 + blockIdx.y;
  const int c0 = p.g.begin(chunk);
  const bool ok = lane < p.g.width(chunk);
  int64_t f = p.row_begin + (int64_t)blockIdx.x * (BLOCK / 32) + warp;
  if (f >= p.row_end) return;
  const int P = p.P;
  const int bnd = lane <= P ? p.seg_start[f * P + lane] : 0;
  const int kind = p.row_kind[f];
  const int s0 = __shfl_sync(kFull, bnd, 0);
  const int s1 = __shfl_sync(kFull, bnd, 1);
  const int e1 = __shfl_sync(kFull, bnd, P);
  if (kind) return;
  const int col = c0 + lane;
  const float4* __restrict__ src = reinterpret_cast<const float4*>(p.dout[0]) + col;
  const int n = e1 - s0, n0 = s1 - s0;
  float4 acc;
  if (n0 <= 32 && n - n0 <= 32) {
    // short row: each perspective's offsets in one register, both loaded in one round trip
    const int B = (int)p.B, row_vec = p.g.n_vec;
    int b0 = lane < n0 ? __ldg(p.sorted_b + s0 + lane) : 0;
    int b1 = lane < n - n0 ? __ldg(p.sorted_b + s1 + lane) - B : 0;
    if ((unsigned)b0 >= (unsigned)B || (unsigned)b1 >= (unsigned)B) {  // corrupt workspace: flag, read row 0
      flag_error(kErrBadSegment);
      b0 = (unsigned)b0 < (unsigned)B ? b0 : 0;
      b1 = (unsigned)b1 < (unsigned)B ? b1 : 0;
    }
    acc = queue_sum_regs<D>(src, b0 * row_vec, n0, ok, Vec<float4>::zero());
    if (P == 2) {
      s_park[warp][lane] = acc;
      acc = queue_sum_regs<D>(src, b1 * row_vec + p.persp_delta, n - n0, ok, Vec<float4>::zero());
      float4 t = s_park[warp][lane];
      Vec<float4>::add(t, acc);
      acc = t;
    }
  } else if (n <= kQueueList) {
    queue_offsets(p, list, s0, 0, n, n0, lane);  // both perspectives in one round trip
    acc = queue_sum<D>(src, list, 0, n0, ok, Vec<float4>::zero());
    if (P == 2) {
      s_park[warp][lane] = acc;
      acc = queue_sum<D>(src, list, n0, n, ok, Vec<float4>::zero());
      float4 t = s_park[warp][lane];
      Vec<float4>::add(t, acc);
      acc = t;
    }
  } else {
    const int B = (int)p.B;
    acc = queue_sum_long(p.sorted_b, B, p.g.n_vec, p.persp_delta, src, s0, 0, n0, n0, ok, lane);
    if (P == 2)
      Vec<float4>::add(acc, queue_sum_long(p.sorted_b, B, p.g.n_vec, p.persp_delta, src, s0, n0, n, n0, ok, lane));
  }
  float4 tot[1] = {acc};
  const bool okv[1] = {ok};
  f = p.row_begin + (int64_t)blockIdx.x * (BLOCK / 32) + warp;  // recomputed, not kept live through the walk
  seg_write<float4, 1>(p, f, col, tot, okv, n > 0);
}

// Light rows, the narrow last column chunk (W <= 8 vectors; 6 for C = 1048),
// packed: G = 32 / W consecutive rows per warp, lane group g (lanes g*W ..
// g*W + W - 1) owning row f0 + g and the chunk's W columns.  A full-width
// warp on this chunk would keep 32 - W lanes idle through a whole row walk.
// The G rows' entries are contiguous in sorted_b, so one warp-wide pass turns
// them into row offsets in a shared-memory list (a value's perspective is
// v >= B); then all groups walk their perspective-0 entries in lockstep
// through a D-slot register queue, then their perspective-1 entries, and
// write dW = acc0 + acc1 -- each column summed in ascending b per
// perspective, the same adds as ft_segsum_lightq_kernel.  A warp whose rows
// hold more than kTailList entries, or one of which is heavy, walks its rows
// straight from sorted_b instead (rare: only the 32 own-king rows are heavy).
constexpr int kTailList = 1280;

template <int W, int D>
__global__ void __launch_bounds__(128, 8) ft_segsum_tail_kernel(const SegParams p) {
  using Ops = Vec<float4>;
  // G rows need G * P + 1 segment bounds, one per lane: at most 15 rows
  constexpr int G = 32 / W < 15 ? 32 / W : 15;
  __shared__ int s_list[4][kTailList];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* list = s_list[warp];
  const int g = lane / W, sub = lane - g * W;
  const bool live_lane = g < G;
  const int P = p.P;
  const int chunk = p.g.n_chunks - 1;
  const int col = p.g.begin(chunk) + sub;
  const int row_vec = p.g.n_vec;
  const int B = (int)p.B;
  const int64_t f0 = p.row_begin + ((int64_t)blockIdx.x * 4 + warp) * G;
  if (f0 >= p.row_end) return;
  const int n_rows = p.row_end - f0 < G ? (int)(p.row_end - f0) : G;
  // segment bounds of the G rows (G * P + 1 values) and their kinds
  const int bnd = lane <= n_rows * P ? p.seg_start[f0 * P + lane] : 0;
  const int kind = lane < n_rows ? p.row_kind[f0 + lane] : 0;
  const bool row_live = live_lane && g < n_rows;
  const int gg = row_live ? g : 0;
  const int s0 = __shfl_sync(kFull, bnd, gg * P);
  const int s1 = __shfl_sync(kFull, bnd, gg * P + 1);  // P == 1: the row's end
  const int e1 = __shfl_sync(kFull, bnd, (gg + 1) * P);
  const int my_kind = __shfl_sync(kFull, kind, gg);
  const int S = __shfl_sync(kFull, bnd, 0);
  const int E = __shfl_sync(kFull, bnd, n_rows * P);
  const bool any_heavy = __any_sync(kFull, lane < n_rows && kind != 0);
  // bounds must nest (S <= s0 <= s1 <= e1 <= E); a corrupt workspace is
  // flagged and its row left empty, so no walk leaves the written list
  const bool sane = S <= s0 && s0 <= s1 && s1 <= e1 && e1 <= E;
  if (row_live && !my_kind && !sane) flag_error(kErrBadSegment);
  const bool walk_row = row_live && !my_kind && sane;
  const int n0 = walk_row ? s1 - s0 : 0;
  const int n1 = walk_row && P == 2 ? e1 - s1 : 0;
  const float4* __restrict__ src = reinterpret_cast<const float4*>(p.dout[0]) + col;
  float4 acc0 = Ops::zero(), acc1 = Ops::zero();
  if (!any_heavy && E - S <= kTailList) {
    for (int e = lane; e < E - S; e += 32) {
      const int v = __ldg(p.sorted_b + S + e);
      const bool q = v >= B;
      int b = v - (q ? B : 0);
      if ((unsigned)b >= (unsigned)B) {  // corrupt workspace: flag, read row 0
        flag_error(kErrBadSegment);
        b = 0;
      }
      list[e] = b * row_vec + (q ? p.persp_delta : 0);
    }
    __syncwarp();
    // each group walks list[at, at + n) with the queue; all groups in lockstep
    auto walk = [&](int at, int n, float4& acc) {
      int n_max = n;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const int t = __shfl_xor_sync(kFull, n_max, o);
        n_max = t > n_max ? t : n_max;
      }
      float4 w[D];
#pragma unroll
      for (int d = 0; d < D; ++d)
        if (d < n) w[d] = Ops::ldg(src + list[at + d]);
      for (int j0 = 0; j0 < n_max; j0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
          const int j = j0 + d;
          if (j < n) {
            Ops::add(acc, w[d]);
            if (j + D < n) w[d] = Ops::ldg(src + list[at + j + D]);
          }
        }
      }
    };
    walk(s0 - S, n0, acc0);
    if (P == 2) walk(s1 - S, n1, acc1);
  } else {
    // entry by entry from sorted_b (a heavy row among the G, or a very long row)
    for (int j = 0; j < n0 + n1; ++j) {
      const int v = __ldg(p.sorted_b + s0 + j);
      const bool q = j >= n0;
      int b = v - (q ? B : 0);
      if ((unsigned)b >= (unsigned)B) {
        flag_error(kErrBadSegment);
        b = 0;
      }
      const float4 x = Ops::ldg(src + (b * row_vec + (q ? p.persp_delta : 0)));
      if (q) Ops::add(acc1, x);
      else Ops::add(acc0, x);
    }
  }
  if (row_live && !my_kind) {
    float4 tot[1] = {acc0};
    if (P == 2) Ops::add(tot[0], acc1);
    const bool okv[1] = {true};
    seg_write<float4, 1>(p, f0 + g, col, tot, okv, n0 + n1 > 0);
  }
}

// Heavy rows: a long sum per column whose only order-preserving parallelism
// is across columns and across the two perspectives.  One warp per (row,
// 32-vector piece of a column chunk, perspective) streams the segment's dOut
// slices through a lane-private kHeavyStages-deep cp.async ring; the row's
// positions are read 32 at a time, one group ahead of the ring, so the issue
// side never waits for them.  With two perspectives each warp stores its sum
// in `heavy_part` and the second of the pair to finish (a per-piece ticket,
// zeroed before the launch; nobody waits) writes dW = acc_white + acc_black.
constexpr int kHeavyWarps = 2;
constexpr int kHeavyStages = 48;
constexpr int kHeavyBatch = 8;
static_assert(kHeavyStages % kHeavyBatch == 0, "a batch never wraps the ring");

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
  const int P = p.P;
  const int wi = blockIdx.x * kHeavyWarps + warp;
  const int q = wi % P;
  const int slot = wi / P / pieces, piece = wi / P - slot * pieces;
  const int nh = *p.n_heavy < p.heavy_cap ? *p.n_heavy : p.heavy_cap;
  if (slot >= nh) return;
  const int64_t f = p.heavy_list[slot];
  if (f < p.row_begin || f >= p.row_end) return;
  const int col = c0 + piece * 32 + lane;
  const bool ok1 = piece * 32 + lane < width;
  const int64_t row_vec = p.g.n_vec;
  const int s = p.seg_start[f * P + q], e = p.seg_start[f * P + q + 1];
  const VT* src = reinterpret_cast<const VT*>(q ? p.dout[1] : p.dout[0]) + (ok1 ? col : 0);
  auto group = [&](int base) {  // decoded positions of entries [base, base + 32)
    return base + lane < e ? decode_position(__ldg(p.sorted_b + base + lane), q, p.B) : -1;
  };
  VT acc = Ops::zero();
  // Entries move in batches of kHeavyBatch, one cp.async group each: the
  // batch's positions come from one group of 32 decoded positions (a batch
  // never straddles two: 32 is a multiple of the batch), its shuffles and
  // copies are issued back to back, and the consume side reads the batch's
  // ring slots together and adds them in order -- the walk costs one chain
  // of dependent steps per batch instead of per entry.
  int t = s;  // issue pointer, kHeavyStages entries ahead of the consume pointer
  int g_base = s, g_cur = group(s), g_next = group(s + 32);
  auto issue_batch = [&](int slot0) {
    if (t - g_base == 32) {  // next group of positions: already loaded; load the one after
      g_base += 32;
      g_cur = g_next;
      g_next = group(g_base + 32);
    }
    const int o = t - g_base;  // 0, 8, 16 or 24
    int b[kHeavyBatch];
#pragma unroll
    for (int k = 0; k < kHeavyBatch; ++k) b[k] = __shfl_sync(kFull, g_cur, o + k);
#pragma unroll
    for (int k = 0; k < kHeavyBatch; ++k)
      if (t + k < e)  // past the segment: the slot is never read
        cp_async_vec<VT>(ring + (slot0 + k) * 32, src + (b[k] >= 0 ? (int64_t)b[k] * row_vec : 0), ok1 && b[k] >= 0);
    cp_async_commit();
    t += kHeavyBatch;
  };
  for (int i = 0; i < kHeavyStages / kHeavyBatch; ++i) issue_batch(i * kHeavyBatch);
  int j = s, stage = 0;
  for (; j + kHeavyBatch <= e; j += kHeavyBatch) {
    cp_async_wait<kHeavyStages / kHeavyBatch - 1>();  // the oldest batch has landed
    VT v[kHeavyBatch];
#pragma unroll
    for (int k = 0; k < kHeavyBatch; ++k) v[k] = ring[(stage + k) * 32];
#pragma unroll
    for (int k = 0; k < kHeavyBatch; ++k) Ops::add(acc, v[k]);
    __syncwarp();
    issue_batch(stage);
    stage = stage + kHeavyBatch == kHeavyStages ? 0 : stage + kHeavyBatch;
  }
  cp_async_wait<0>();  // the last, partial batch (already issued)
  for (; j < e; ++j) {
    Ops::add(acc, ring[stage * 32]);
    ++stage;  // < kHeavyBatch entries from a batch-aligned slot: no wrap
  }
  const bool ok[1] = {ok1};
  if (P == 1) {
    const VT t1[1] = {acc};
    seg_write<VT, 1>(p, f, col, t1, ok, true);
    return;
  }
  // two perspectives: publish this half, the second finisher combines
  VT* part = reinterpret_cast<VT*>(p.heavy_part) + ((int64_t)slot * 2 + q) * row_vec;
  if (ok1) part[col] = acc;
  __threadfence();
  __syncwarp();
  int ticket = 0;
  unsigned* cnt = p.heavy_ticket + (int64_t)slot * p.heavy_ticket_stride + c0 + piece * 32;
  if (lane == 0) ticket = (int)atomicAdd(cnt, 1u);
  ticket = __shfl_sync(kFull, ticket, 0);
  if (ticket != 1) return;
  __threadfence();
  const VT* other = reinterpret_cast<const VT*>(p.heavy_part) + ((int64_t)slot * 2 + (1 - q)) * row_vec;
  VT tot = Ops::zero();
  if (ok1) {
    tot = __ldcg(other + col);  // the other warp's half, from L2
    Ops::add(tot, acc);         // acc_white + acc_black (one fp32 add, order-free)
  }
  const VT t1[1] = {tot};
  seg_write<VT, 1>(p, f, col, t1, ok, true);
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
