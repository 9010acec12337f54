// FT epilogue: the input transform that follows the feature transformer in
// NNUEModel._transform_inputs (reference src/model/model.py:86-115), forward
// and backward, one pass each (sm_100a).
//
// Forward, per position b (fp32; us[b] is 0.0 or 1.0, L1 = l1, h = L1 / 2):
//   wc = clamp(wp[b, :L1], 0, 1),  bc = clamp(bp[b, :L1], 0, 1)   (NaN passes)
//   w_pw[j] = wc[j] * wc[j + h],  b_pw[j] = bc[j] * bc[j + h]      (j < h)
//   l0[b, :h] = (us ? w_pw : b_pw) * (127/128)
//   l0[b, h:] = (us ? b_pw : w_pw) * (127/128)
//   psqt[b]   = (wp[b, L1 + pidx[b]] - bp[b, L1 + pidx[b]]) * (us[b] - 0.5)
// Backward: the gradients torch autograd produces for that graph, term by
// term, so the result is bit-identical to it:
//   g1 = d_l0[b, :h] * (127/128),  g2 = d_l0[b, h:] * (127/128)
//   d_w_pw = where(us, g1, 0) + where(us, 0, g2)       (w_pw feeds both where's)
//   d_b_pw = where(us, 0, g1) + where(us, g2, 0)
//   d_wc[j] = d_w_pw[j] * wc[j + h] + 0,  d_wc[j + h] = 0 + d_w_pw[j] * wc[j]
//                                           (the two select-backward buffers add)
//   d_wp[b, :L1] = where(0 <= wp <= 1, d_wc, 0)          (clamp backward)
//   d_wp[b, L1 + k] = k == pidx[b] ? 0 + d_psqt[b] * (us[b] - 0.5) : 0
//   d_bp[b, L1 + k] = k == pidx[b] ? 0 + -(d_psqt[b] * (us[b] - 0.5)) : 0
// One warp per position; 128-bit accesses when L1 % 8 == 0 and rows are
// 16-byte aligned.  PSQT indices outside [0, n_psqt) are flagged and skipped.
#pragma once

#include "common.cuh"

namespace nnue {

struct EpiParams {
  const float* wp;
  const float* bp;
  const float* us;       // [B] (a [B, 1] float tensor)
  const int64_t* pidx;   // [B]
  float* l0;             // [B, L1]
  float* psqt;           // [B]
  const float* d_l0;     // [B, L1] or null (zero gradient)
  const float* d_psqt;   // [B] or null
  float* d_wp;           // [B, L1 + n_psqt]
  float* d_bp;
  int64_t B;
  int32_t l1;
  int32_t n_psqt;
};

constexpr float kL0Scale = 127.0f / 128.0f;  // exact in fp32

__device__ __forceinline__ float clamp01(float x) { return x < 0.0f ? 0.0f : (x > 1.0f ? 1.0f : x); }
__device__ __forceinline__ bool in01(float x) { return x >= 0.0f && x <= 1.0f; }

template <typename VT>
struct EpiVec;
template <>
struct EpiVec<float4> {
  static constexpr int kN = 4;
  static __device__ __forceinline__ float& at(float4& x, int i) { return i == 0 ? x.x : i == 1 ? x.y : i == 2 ? x.z : x.w; }
};
template <>
struct EpiVec<float> {
  static constexpr int kN = 1;
  static __device__ __forceinline__ float& at(float& x, int) { return x; }
};

template <typename VT>
__global__ void __launch_bounds__(256) ft_epilogue_forward_kernel(const EpiParams a) {
  using EV = EpiVec<VT>;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)a.l1 + a.n_psqt;
  const int hv = a.l1 / 2 / EV::kN;  // half of L1, in vectors
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < a.B;
       b += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const float u = a.us[b];
    const bool us = u != 0.0f;
    const VT* w = reinterpret_cast<const VT*>(a.wp + b * row);
    const VT* bb = reinterpret_cast<const VT*>(a.bp + b * row);
    VT* o = reinterpret_cast<VT*>(a.l0 + b * (int64_t)a.l1);
    for (int q = lane; q < hv; q += 32) {
      VT w0 = w[q], w1 = w[q + hv], b0 = bb[q], b1 = bb[q + hv], first, second;
#pragma unroll
      for (int i = 0; i < EV::kN; ++i) {
        const float wpw = __fmul_rn(clamp01(EV::at(w0, i)), clamp01(EV::at(w1, i)));
        const float bpw = __fmul_rn(clamp01(EV::at(b0, i)), clamp01(EV::at(b1, i)));
        EV::at(first, i) = __fmul_rn(us ? wpw : bpw, kL0Scale);
        EV::at(second, i) = __fmul_rn(us ? bpw : wpw, kL0Scale);
      }
      o[q] = first;
      o[q + hv] = second;
    }
    if (lane == 0) {
      const int64_t k = a.pidx[b];
      if ((uint64_t)k < (uint64_t)a.n_psqt) {
        const float d = __fsub_rn(a.wp[b * row + a.l1 + k], a.bp[b * row + a.l1 + k]);
        a.psqt[b] = __fmul_rn(d, __fsub_rn(u, 0.5f));
      } else {
        flag_error(kErrBadPsqtIndex);
        a.psqt[b] = 0.0f;
      }
    }
  }
}

template <typename VT>
__global__ void __launch_bounds__(256) ft_epilogue_backward_kernel(const EpiParams a) {
  using EV = EpiVec<VT>;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)a.l1 + a.n_psqt;
  const int hv = a.l1 / 2 / EV::kN;
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < a.B;
       b += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const float u = a.us[b];
    const bool us = u != 0.0f;
    const VT* w = reinterpret_cast<const VT*>(a.wp + b * row);
    const VT* bb = reinterpret_cast<const VT*>(a.bp + b * row);
    const VT* g = a.d_l0 ? reinterpret_cast<const VT*>(a.d_l0 + b * (int64_t)a.l1) : nullptr;
    VT* dw = reinterpret_cast<VT*>(a.d_wp + b * row);
    VT* db = reinterpret_cast<VT*>(a.d_bp + b * row);
    for (int q = lane; q < hv; q += 32) {
      VT w0 = w[q], w1 = w[q + hv], b0 = bb[q], b1 = bb[q + hv], ga{}, gb{}, dw0, dw1, db0, db1;
      if (g) {
        ga = g[q];
        gb = g[q + hv];
      }
#pragma unroll
      for (int i = 0; i < EV::kN; ++i) {
        const float g1 = __fmul_rn(EV::at(ga, i), kL0Scale), g2 = __fmul_rn(EV::at(gb, i), kL0Scale);
        const float dwpw = __fadd_rn(us ? g1 : 0.0f, us ? 0.0f : g2);
        const float dbpw = __fadd_rn(us ? 0.0f : g1, us ? g2 : 0.0f);
        const float wx0 = EV::at(w0, i), wx1 = EV::at(w1, i), bx0 = EV::at(b0, i), bx1 = EV::at(b1, i);
        const float dwc0 = __fadd_rn(__fmul_rn(dwpw, clamp01(wx1)), 0.0f);
        const float dwc1 = __fadd_rn(0.0f, __fmul_rn(dwpw, clamp01(wx0)));
        const float dbc0 = __fadd_rn(__fmul_rn(dbpw, clamp01(bx1)), 0.0f);
        const float dbc1 = __fadd_rn(0.0f, __fmul_rn(dbpw, clamp01(bx0)));
        EV::at(dw0, i) = in01(wx0) ? dwc0 : 0.0f;
        EV::at(dw1, i) = in01(wx1) ? dwc1 : 0.0f;
        EV::at(db0, i) = in01(bx0) ? dbc0 : 0.0f;
        EV::at(db1, i) = in01(bx1) ? dbc1 : 0.0f;
      }
      dw[q] = dw0;
      dw[q + hv] = dw1;
      db[q] = db0;
      db[q + hv] = db1;
    }
    const int64_t k = a.pidx[b];
    const bool k_ok = (uint64_t)k < (uint64_t)a.n_psqt;
    if (lane == 0 && !k_ok) flag_error(kErrBadPsqtIndex);
    for (int j = lane; j < a.n_psqt; j += 32) {
      float vw = 0.0f, vb = 0.0f;
      if (k_ok && j == k) {
        const float d = __fmul_rn(a.d_psqt ? a.d_psqt[b] : 0.0f, __fsub_rn(u, 0.5f));
        vw = __fadd_rn(0.0f, d);
        vb = __fadd_rn(0.0f, -d);
      }
      a.d_wp[b * row + a.l1 + j] = vw;
      a.d_bp[b * row + a.l1 + j] = vb;
    }
  }
}

}  // namespace nnue
