// Feature-index encoder on the device (sm_100a): boards in HBM -> the
// int32 [B, K] index rows (compacted, -1 padded) that the feature
// transformer consumes.  The encoding functions are the host encoder's own
// (feature_encode.h, restating src/rust/feature_extraction.rs), so both
// produce the same rows; only the data movement is device-specific.
//
// A block takes 64 positions: their boards (64 bytes each) are staged in
// shared memory with 16-byte loads, one thread per position builds its 12
// piece bitboards + occupancy there, and one thread per (position,
// perspective) walks the threats / HalfKA features with the lookup tables
// (attack sets, rays, threat offsets; 13 KB) also in shared memory.
#pragma once

#include "common.cuh"
#include "feature_encode.h"

namespace nnue {

struct EncParams {
  const uint8_t* board;                    // [count, 64] piece ids (>= 12: empty)
  int64_t count;
  int32_t feature_set;                     // 0 HalfKAv2_hm, 1 Full_Threats, 2 Full_Threats+HalfKAv2_hm
  int32_t K;                               // row length (32, 128, 160)
  int32_t board_vec16;                     // board pointer is 16-byte aligned
  int32_t* out[2];                         // [count, K] white, black
  int32_t* counts[2];                      // [count] each, nullable
  const nnue_feat::FeatureTables* tables;  // device copy of the host tables
};

constexpr int kEncThreads = 128;
constexpr int kEncPositions = kEncThreads / 2;

// Buffers four indices and writes them as one 16-byte store: a warp's 32
// rows are 32 different rows, so 4-byte stores would cost one L2 request
// per index.  Rows must be 16-byte aligned with K % 4 == 0.
struct Int4Sink {
  int32_t* row;
  int n;
  int4 buf;
  __device__ __forceinline__ void push(int v) {
    const int r = n & 3;
    buf.x = r == 0 ? v : buf.x;
    buf.y = r == 1 ? v : buf.y;
    buf.z = r == 2 ? v : buf.z;
    buf.w = r == 3 ? v : buf.w;
    ++n;
    if (r == 3) reinterpret_cast<int4*>(row)[(n >> 2) - 1] = buf;
  }
  // the -1 tail from n up to K
  __device__ __forceinline__ void finish(int K) {
    int q = n >> 2;
    const int r = n & 3;
    if (r) {
      if (r <= 1) buf.y = -1;
      if (r <= 2) buf.z = -1;
      buf.w = -1;
      reinterpret_cast<int4*>(row)[q++] = buf;
    }
    for (; q < (K >> 2); ++q) reinterpret_cast<int4*>(row)[q] = make_int4(-1, -1, -1, -1);
  }
};

template <bool kVec>
__global__ void __launch_bounds__(kEncThreads) encode_features_kernel(const EncParams p) {
  __shared__ nnue_feat::FeatureTables t;
  __shared__ __align__(16) uint8_t boards[kEncPositions][64];
  __shared__ uint64_t bbs[kEncPositions][13];  // piece bitboards [0, 12) + occupancy [12]
  const int tid = threadIdx.x;
  const int64_t pos0 = (int64_t)blockIdx.x * kEncPositions;
  const int64_t n_here = p.count - pos0 < kEncPositions ? p.count - pos0 : kEncPositions;

  {  // tables: a byte copy of the host struct (its size is a multiple of 16)
    const uint4* src = reinterpret_cast<const uint4*>(p.tables);
    uint4* dst = reinterpret_cast<uint4*>(&t);
    for (int i = tid; i < (int)(sizeof(t) / 16); i += kEncThreads) dst[i] = __ldg(src + i);
  }
  if (p.board_vec16) {
    const uint4* src = reinterpret_cast<const uint4*>(p.board + pos0 * 64);
    uint4* dst = reinterpret_cast<uint4*>(&boards[0][0]);
    for (int i = tid; i < kEncPositions * 4; i += kEncThreads)
      dst[i] = i < n_here * 4 ? __ldcs(src + i) : make_uint4(~0u, ~0u, ~0u, ~0u);
  } else {
    for (int i = tid; i < kEncPositions * 64; i += kEncThreads)
      (&boards[0][0])[i] = i < n_here * 64 ? p.board[pos0 * 64 + i] : (uint8_t)0xFF;
  }
  __syncthreads();
  if (tid < kEncPositions) {
    uint64_t* bb = bbs[tid];
#pragma unroll
    for (int k = 0; k < 12; ++k) bb[k] = 0;
    uint64_t occ = 0;
    const uint8_t* bd = boards[tid];
    for (int sq = 0; sq < 64; ++sq) {
      const int id = bd[sq];
      if (id < 12) {
        bb[id] |= 1ull << sq;
        occ |= 1ull << sq;
      }
    }
    bb[12] = occ;
  }
  __syncthreads();
  const int li = tid >> 1, persp = tid & 1;
  if (li >= n_here) return;
  const int64_t pos = pos0 + li;
  const nnue_feat::PosView v{bbs[li], bbs[li][12], boards[li]};
  int32_t* row = p.out[persp] + pos * p.K;
  int n;
  if constexpr (kVec) {
    Int4Sink sink{row, 0, make_int4(-1, -1, -1, -1)};
    n = nnue_feat::encode_position(t, v, persp, p.feature_set, sink);
    if (n < 0) sink.n = 0;  // rejected: the whole row becomes -1
    sink.finish(p.K);
  } else {
    nnue_feat::RowSink sink{row, 0};
    n = nnue_feat::encode_position(t, v, persp, p.feature_set, sink);
    for (int i = n < 0 ? 0 : n; i < p.K; ++i) row[i] = -1;
  }
  if (n < 0) {  // rejected position: an all -1 row, reported
    flag_error(kErrBadPosition);
    n = 0;
  }
  if (p.counts[persp]) p.counts[persp][pos] = n;
}

}  // namespace nnue
