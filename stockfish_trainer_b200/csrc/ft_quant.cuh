// Quantised feature transformer (sm_100a): the inference forward the engine
// runs on a serialised net, plus the export + quantisation that produces its
// tables.
//
// Export (reference src/model/modules/features/halfka_v2_hm.py:100-134):
//   coalesced = weight + virtual.repeat(32, 1)            (fp32 add)
//   export row r = bucket * 704 + plane * 64 + sq, planes 0..9 copied from the
//   training row bucket * 768 + plane * 64 + sq; plane 10 takes the opponent
//   king plane (11) except at the bucket's own king square, which takes the own
//   king plane (10).
// Quantisation (reference src/model/quantize.py:83-89, called from
// src/scripts/serialize.py:199-230): x.mul(scale).round() with fp32 multiply and
// round-half-to-even; weights/bias scale 255 -> int16, PSQT scale 600*16 -> int32.
// Accumulation (the engine, not in the reference): int16 two's-complement
// adds for the L1 accumulators starting from the bias, int32 for PSQT from 0.
#pragma once

#include "common.cuh"

namespace nnue {

// Training-space HalfKA row (24576) -> export row (22528).  Exact for the
// indices a position with both kings produces (the own-king feature always
// sits at the bucket's king square).
__device__ __forceinline__ int halfka_export_row(int i) {
  const int bucket = i / 768, rem = i - bucket * 768;
  int plane = rem >> 6;
  plane = plane > 10 ? 10 : plane;
  return bucket * 704 + plane * 64 + (rem & 63);
}

struct QFwdParams {
  const int32_t* idx[2];
  int16_t* acc[2];     // [B, L1]
  int32_t* psqt[2];    // [B, NP]
  const int16_t* Wq;   // [Tq, L1]
  const int32_t* Pq;   // [Tq, NP]
  const int16_t* bias; // [L1]
  int64_t B;
  int32_t K;
  int32_t Tq;
  int32_t n8;          // L1 / 8   (uint4 vectors of 8 int16)
  int32_t np4;         // NP / 4   (int4 vectors of 4 int32)
  int32_t P;
  int32_t map_training;
  int32_t items_per_warp;
};

__device__ __forceinline__ void vadd16x8(uint4& a, const uint4& b) {
  a.x = __vadd2(a.x, b.x);
  a.y = __vadd2(a.y, b.y);
  a.z = __vadd2(a.z, b.z);
  a.w = __vadd2(a.w, b.w);
}

__device__ __forceinline__ void vadd32x4(int4& a, const int4& b) {
  a.x = (int)((unsigned)a.x + (unsigned)b.x);
  a.y = (int)((unsigned)a.y + (unsigned)b.y);
  a.z = (int)((unsigned)a.z + (unsigned)b.z);
  a.w = (int)((unsigned)a.w + (unsigned)b.w);
}

template <int VQ, int U>
__global__ void __launch_bounds__(kBlock) ft_qforward_kernel(const QFwdParams p) {
  const int lane = threadIdx.x & 31;
  bool ok[VQ];
  uint4 bias_r[VQ];
  const uint4* __restrict__ bv = reinterpret_cast<const uint4*>(p.bias) + lane;
#pragma unroll
  for (int v = 0; v < VQ; ++v) {
    ok[v] = lane + 32 * v < p.n8;
    bias_r[v] = ok[v] ? bv[32 * v] : make_uint4(0, 0, 0, 0);
  }
  const bool pok = lane < p.np4;
  const uint4* __restrict__ Wv = reinterpret_cast<const uint4*>(p.Wq) + lane;
  const int4* __restrict__ Pv = reinterpret_cast<const int4*>(p.Pq) + lane;
  const int32_t limit = p.map_training ? 24576 : p.Tq;

  const int64_t n_items = (int64_t)p.P * p.B;
  int64_t item = ((int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5)) * p.items_per_warp;
  const int64_t item_end = item + p.items_per_warp < n_items ? item + p.items_per_warp : n_items;
  for (; item < item_end; ++item) {
    const int persp = item >= p.B ? 1 : 0;
    const int64_t b = item - (int64_t)persp * p.B;
    const int32_t* __restrict__ irow = (persp ? p.idx[1] : p.idx[0]) + b * p.K;
    uint4 acc[VQ];
#pragma unroll
    for (int v = 0; v < VQ; ++v) acc[v] = bias_r[v];
    int4 ps = make_int4(0, 0, 0, 0);

    for (int k0 = 0; k0 < p.K; k0 += 32) {
      const int kk = k0 + lane;
      int f = kk < p.K ? __ldcs(irow + kk) : -1;
      bool valid = (unsigned)f < (unsigned)limit;
      if (valid && p.map_training) f = halfka_export_row(f);
      if (valid && f >= p.Tq) valid = false, f = -2;
      if (!valid && f != -1) flag_error(kErrBadQuantIndex);
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
        uint4 w[U][VQ];
        int4 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
          for (int v = 0; v < VQ; ++v)
            if (has[u] && ok[v]) w[u][v] = __ldg(Wv + (int64_t)rows[u] * p.n8 + 32 * v);
          if (has[u] && pok) q[u] = __ldg(Pv + (int64_t)rows[u] * p.np4);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
          for (int v = 0; v < VQ; ++v)
            if (has[u] && ok[v]) vadd16x8(acc[v], w[u][v]);
          if (has[u] && pok) vadd32x4(ps, q[u]);
        }
      }
    }
    uint4* o = reinterpret_cast<uint4*>(persp ? p.acc[1] : p.acc[0]) + b * p.n8 + lane;
#pragma unroll
    for (int v = 0; v < VQ; ++v)
      if (ok[v]) __stcs(o + 32 * v, acc[v]);
    if (pok) __stcs(reinterpret_cast<int4*>(persp ? p.psqt[1] : p.psqt[0]) + b * p.np4 + lane, ps);
  }
}

struct KingSquares {  // export bucket -> oriented own-king square
  int32_t sq[32];
};

// One block per export row.  W: [24576, C] training rows, V: [768, C] virtual
// rows (nullable), C = L1 + NP.  Writes Wq [22528, L1] int16, Pq [22528, NP]
// int32.  Out-of-range products wrap through int32 -> int16 (callers clip).
__global__ void halfka_export_quantize_kernel(const float* __restrict__ W, const float* __restrict__ V,
                                              int32_t C, int32_t L1, float w_scale, float p_scale,
                                              const KingSquares inv_king_bucket,
                                              int16_t* __restrict__ Wq, int32_t* __restrict__ Pq) {
  const int r = blockIdx.x;  // export row
  const int bucket = r / 704, rem = r - bucket * 704;
  const int plane = rem >> 6, sq = rem & 63;
  int src;
  if (plane < 10) src = bucket * 768 + plane * 64 + sq;
  else if (sq == inv_king_bucket.sq[bucket]) src = bucket * 768 + 640 + sq;
  else src = bucket * 768 + 704 + sq;
  const float* wrow = W + (int64_t)src * C;
  const float* vrow = V ? V + (int64_t)(src % 768) * C : nullptr;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float x = vrow ? __fadd_rn(wrow[c], vrow[c]) : wrow[c];
    if (c < L1) Wq[(int64_t)r * L1 + c] = (int16_t)__float2int_rn(__fmul_rn(x, w_scale));
    else Pq[(int64_t)r * (C - L1) + (c - L1)] = __float2int_rn(__fmul_rn(x, p_scale));
  }
}

__global__ void quantize_i16_kernel(const float* __restrict__ x, int64_t n, float scale, int16_t* __restrict__ q) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) q[i] = (int16_t)__float2int_rn(__fmul_rn(x[i], scale));
}

}  // namespace nnue
