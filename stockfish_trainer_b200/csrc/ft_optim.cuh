// Ranger22 parameter update, one pass per parameter (sm_100a).
//
// Reference (src/ranger22/optimizer.py): the fused path of Ranger22.step for a
// 1-D / 2-D fp32 CUDA parameter runs _compiled_full_update_{1d,2d} (:48-76,
// :79-107; eager twin :256-301), and every lookahead_mergetime steps
// lookahead_process_step (:569-597) blends p with its slow copy.  Per element,
// in this order and in fp32:
//   v  = v * beta2;        v  = v + (g * g) * (1 - beta2)
//   m  = m * beta1^2;      m  = m + g * (1 - beta1^2)
//   u  = ||p_row||_2       (2-D: per row, dim=1; 1-D: the whole vector),
//                           taken from p BEFORE this step's update
//   corr  = two_nl * (1 - 1 / (u + eps))                       (per row)
//   denom = sqrt(v) * inv_sqrt_bc2 + eps
//   pn    = (m * pnm_a + m_prev * pnm_b) * noise_norm_recip
//   p     = p * (1 - lr * corr);   p = p - (pn / denom) * step_size
//   merge: p = lerp(p, la, w) with torch's two-branch lerp, w = 1 - alpha;
//          la = p
// One thread group per row reads the row of p once for the norm (fp64 sum of
// squares, rounded once), then streams p, g, v, m, m_prev (and la) and
// writes p, v, m (and la): 32 bytes per element, 40 on merge steps.  All
// arithmetic is explicit round-to-nearest (no contraction), the division and
// square root are the IEEE-correct intrinsics.
#pragma once

#include "common.cuh"

namespace nnue {

struct R22Params {
  float* p;
  const float* g;
  float* v;
  float* m;
  const float* mp;
  float* la;     // lookahead copy (read/written only when merge != 0)
  int64_t rows;
  int64_t cols;  // floats per row
  float lr, inv_sqrt_bc2, eps, two_nl, noise_recip, pnm_a, pnm_b, step_size, beta2, omb2, b1sq, omb1sq;
  int32_t merge;
  float w;  // lerp weight toward the lookahead copy (1 - alpha)
};

__device__ __forceinline__ float r22_element(const R22Params& a, float x, float g, float& v, float& m, float mp,
                                             float pscale) {
  v = __fadd_rn(__fmul_rn(v, a.beta2), __fmul_rn(__fmul_rn(g, g), a.omb2));
  m = __fadd_rn(__fmul_rn(m, a.b1sq), __fmul_rn(g, a.omb1sq));
  const float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(v), a.inv_sqrt_bc2), a.eps);
  const float pn = __fmul_rn(__fadd_rn(__fmul_rn(m, a.pnm_a), __fmul_rn(mp, a.pnm_b)), a.noise_recip);
  x = __fmul_rn(x, pscale);
  return __fsub_rn(x, __fmul_rn(__fdiv_rn(pn, denom), a.step_size));
}

// torch.lerp(start, end, weight): weight < 0.5 ? start + weight * (end - start)
//                                              : end - (end - start) * (1 - weight)
__device__ __forceinline__ float r22_lerp(float start, float end, float w) {
  const float d = __fsub_rn(end, start);
  return w < 0.5f ? __fadd_rn(start, __fmul_rn(w, d)) : __fsub_rn(end, __fmul_rn(d, __fsub_rn(1.0f, w)));
}

template <typename VT>
struct R22Vec;

template <>
struct R22Vec<float4> {
  static constexpr int kN = 4;
  static __device__ __forceinline__ float get(const float4& x, int i) {
    return i == 0 ? x.x : i == 1 ? x.y : i == 2 ? x.z : x.w;
  }
  static __device__ __forceinline__ void set(float4& x, int i, float f) {
    if (i == 0) x.x = f;
    else if (i == 1) x.y = f;
    else if (i == 2) x.z = f;
    else x.w = f;
  }
};

template <>
struct R22Vec<float> {
  static constexpr int kN = 1;
  static __device__ __forceinline__ float get(const float& x, int) { return x; }
  static __device__ __forceinline__ void set(float& x, int, float f) { x = f; }
};

// Sum of squares of a row, fp64, reduced over a GROUP of threads (GROUP 32:
// one warp per row; GROUP == blockDim.x: one block per row).
template <int GROUP>
__device__ __forceinline__ double r22_group_sum(double s, double* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if constexpr (GROUP > 32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) scratch[warp] = s;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < GROUP / 32; ++i) t += scratch[i];  // fixed order, same value in every thread
    __syncthreads();
    s = t;
  }
  return s;
}

template <typename VT, int GROUP>
__global__ void __launch_bounds__(GROUP > 256 ? GROUP : 256) ranger22_rows_kernel(const R22Params a) {
  using RV = R22Vec<VT>;
  __shared__ double scratch[32];
  const int gi = threadIdx.x % GROUP;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / GROUP) + threadIdx.x / GROUP;
  const bool live = row < a.rows;  // GROUP > 32: whole block shares one row, always live
  const int64_t nvec = a.cols / RV::kN;
  const int64_t base = (live ? row : 0) * nvec;
  VT* p = reinterpret_cast<VT*>(a.p) + base;
  double ss = 0.0;
  if (live)
    for (int64_t j = gi; j < nvec; j += GROUP) {
      const VT x = p[j];
#pragma unroll
      for (int i = 0; i < RV::kN; ++i) {
        const double d = (double)RV::get(x, i);
        ss += d * d;
      }
    }
  ss = r22_group_sum<GROUP>(ss, scratch);
  if (!live) return;
  const float u = (float)sqrt(ss);
  const float corr = __fmul_rn(a.two_nl, __fsub_rn(1.0f, __fdiv_rn(1.0f, __fadd_rn(u, a.eps))));
  const float pscale = __fsub_rn(1.0f, __fmul_rn(a.lr, corr));
  const VT* g = reinterpret_cast<const VT*>(a.g) + base;
  VT* v = reinterpret_cast<VT*>(a.v) + base;
  VT* m = reinterpret_cast<VT*>(a.m) + base;
  const VT* mp = reinterpret_cast<const VT*>(a.mp) + base;
  VT* la = reinterpret_cast<VT*>(a.la) + base;
  for (int64_t j = gi; j < nvec; j += GROUP) {
    VT x = p[j], gg = g[j], vv = v[j], mm = m[j], mpp = mp[j], ll{};
    if (a.merge) ll = la[j];
#pragma unroll
    for (int i = 0; i < RV::kN; ++i) {
      float vi = RV::get(vv, i), mi = RV::get(mm, i);
      float xi = r22_element(a, RV::get(x, i), RV::get(gg, i), vi, mi, RV::get(mpp, i), pscale);
      if (a.merge) {
        xi = r22_lerp(xi, RV::get(ll, i), a.w);
        RV::set(ll, i, xi);
      }
      RV::set(x, i, xi);
      RV::set(vv, i, vi);
      RV::set(mm, i, mi);
    }
    p[j] = x;
    v[j] = vv;
    m[j] = mm;
    if (a.merge) la[j] = ll;
  }
}

}  // namespace nnue
