// Shared device helpers for the sparse feature-transformer kernels (sm_100a).
//
// Everything here is compiled into ONE translation unit (nnue_ft.cu), so the
// sticky device error word below is a single symbol per device.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nnue {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kBlock = 256;                  // threads per block for all gather kernels
constexpr int kWarpsPerBlock = kBlock / 32;

// Sticky error flags raised by kernels instead of faulting: an index outside
// [-1, num_inputs) is skipped (never dereferenced) and reported here.
__device__ unsigned int g_device_errors = 0;
enum : unsigned {
  kErrBadIndex = 1u,       // feature index < -1 or >= num_inputs
  kErrBadQuantIndex = 2u,  // quantised forward: index outside the table / export map
  kErrBadSegment = 4u,     // backward: a sorted position outside [0, batch) (corrupt workspace)
  kErrBadPsqtIndex = 8u,   // epilogue: PSQT bucket index outside [0, n_psqt)
  kErrBadPosition = 16u,   // encoder: a position the feature functions reject (its rows are all -1)
  kErrExchangeTimeout = 32u,  // exchange: a rank did not arrive at the barrier in time
};

__device__ __forceinline__ void flag_error(unsigned e) { atomicOr(&g_device_errors, e); }

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Vector access policy: float4 rows (128-bit loads) when C % 4 == 0 and the
// pointers are 16-byte aligned, scalar floats otherwise.
template <typename VT>
struct Vec;

template <>
struct Vec<float4> {
  static constexpr int kFloats = 4;
  static __device__ __forceinline__ float4 zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ void add(float4& a, const float4& b) {
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
  }
  static __device__ __forceinline__ float4 ldg(const float4* p) { return __ldg(p); }
  static __device__ __forceinline__ void st_stream(float4* p, const float4& v) { __stcs(p, v); }
};

template <>
struct Vec<float> {
  static constexpr int kFloats = 1;
  static __device__ __forceinline__ float zero() { return 0.f; }
  static __device__ __forceinline__ void add(float& a, const float& b) { a += b; }
  static __device__ __forceinline__ float ldg(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ void st_stream(float* p, const float& v) { __stcs(p, v); }
};

// A feature table split over up to kMaxTables separately allocated row
// blocks (the reference's per-feature parameters, composed.py:49-50): global
// row f lives in block t = the first with f < end[t], at local row
// f - end[t - 1].  n == 1 means one contiguous table (the fast path).
constexpr int kMaxTables = 4;
struct TableSet {
  float* base[kMaxTables];
  int32_t end[kMaxTables];
  int32_t n;
  __host__ __device__ __forceinline__ int find(int64_t f) const {
    int t = 0;
#pragma unroll
    for (int i = 0; i < kMaxTables - 1; ++i)
      if (i < n - 1 && f >= end[i]) t = i + 1;
    return t;
  }
  __host__ __device__ __forceinline__ int64_t start(int t) const { return t ? end[t - 1] : 0; }
};

// Column chunking of one table row of n_vec vectors into n_chunks balanced
// chunks: chunk c covers vectors [begin(c), begin(c + 1)), widths differ by
// at most one.  Chunks are the OUTER grid dimension, so at any moment the
// running blocks touch one column slice of the table / gradient -- a slice
// sized to stay resident in L2 while it is re-read.
struct Geom {
  int32_t n_vec;
  int32_t n_chunks;
  int32_t max_width;  // widest chunk, in vectors
  int32_t exact;      // 1: chunks of exactly max_width vectors + a narrower tail; 0: balanced widths
  __host__ __device__ __forceinline__ int begin(int c) const {
    return exact ? (c < n_chunks ? c * max_width : n_vec) : (int)(((int64_t)c * n_vec) / n_chunks);
  }
  __host__ __device__ __forceinline__ int width(int c) const { return begin(c + 1) - begin(c); }
};

// Warp / block reductions and scans on int32.
__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Inclusive scan over the whole block (blockDim.x a multiple of 32, <= 1024).
// `scratch` must hold 33 ints.  Contains __syncthreads.
__device__ __forceinline__ int block_inclusive_scan(int v, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  int incl = warp_inclusive_scan(v, lane);
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nwarps ? scratch[lane] : 0;
    t = warp_inclusive_scan(t, lane);
    scratch[lane] = t;  // inclusive warp totals
  }
  __syncthreads();
  if (warp > 0) incl += scratch[warp - 1];
  const int total = scratch[nwarps - 1];
  __syncthreads();
  if (threadIdx.x == 0) scratch[32] = total;
  __syncthreads();
  return incl;
}

// ---------------------------------------------------------------------------
// cp.async helpers: every lane copies its own 16 (or 4) bytes into a lane-
// private shared-memory slot and later reads back only what it copied, so
// no barrier is needed; the group count bounds what is still in flight.
// ---------------------------------------------------------------------------
template <typename VT>
__device__ __forceinline__ void cp_async_vec(VT* smem_dst, const VT* gsrc, bool pred);

template <>
__device__ __forceinline__ void cp_async_vec<float4>(float4* smem_dst, const float4* gsrc, bool pred) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
  const int n = pred ? 16 : 0;  // 0 source bytes: zero-fill, source not read
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}

template <>
__device__ __forceinline__ void cp_async_vec<float>(float* smem_dst, const float* gsrc, bool pred) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
  const int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(gsrc), "r"(n) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

}  // namespace nnue
