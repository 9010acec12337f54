// Exchange between the GPUs of one node for the column-sharded FT step:
// block copies into this GPU's and other GPUs' memory (CUDA IPC mappings,
// written with plain stores over NVLink / NVSwitch), followed by a barrier
// among the ranks of the group through flag words in each rank's exchange
// buffer.
//
// Every rank launches the same sequence of exchanges on each channel with the
// same epochs (channels are independent barriers, so exchanges on different
// streams may be in flight at once, one channel each).
// One launch: all blocks copy their rows; each block then makes its stores
// visible system-wide (fence.sc.sys) and counts itself done; the last block
// writes `epoch` into flag[rank] of every rank (st.release.sys) and waits
// until its own flag[0 .. n_ranks) all reach `epoch` (ld.acquire.sys).  Only
// then does the launch complete, so work after it in the stream sees every
// rank's copies into this GPU's memory.  The wait is bounded in time: past
// the limit the kernel raises kErrExchangeTimeout and returns (a rank that
// never arrives cannot hang this GPU).
#pragma once

#include "common.cuh"

namespace nnue {

constexpr int kMaxCopies = 32;
constexpr int kMaxRanks = 16;

struct CopyDesc {
  const float4* src;
  float4* dst;
  int64_t rows;
  int64_t src_ld, dst_ld;  // row strides, in 16-byte vectors
  int32_t width;           // 16-byte vectors per row
  float scale;             // 1: the bytes are copied as they are
};

constexpr int kChannels = 4;  // independent barriers: kMaxRanks flag words each (the last one the block counter)

struct ExchangeParams {
  CopyDesc c[kMaxCopies];
  int64_t row_start[kMaxCopies + 1];  // prefix sums of rows over the copies
  uint32_t* flags[kMaxRanks];         // rank s's flag words of this launch's channel, mapped here
  int32_t n_copies, n_ranks, rank;
  uint32_t epoch;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Warps take R consecutive rows at a time (grid-stride over the rows of all
// copies), lanes over the rows' vectors: all R rows' loads are issued before
// their stores, so R loads per lane are in flight.
template <int R>
__global__ void __launch_bounds__(256) exchange_kernel(const __grid_constant__ ExchangeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t total = p.row_start[p.n_copies];
  int i = 0;  // copy of the first row of the group; rows only grow, so it only grows
  for (int64_t g0 = warp * R; g0 < total; g0 += n_warps * R) {
    while (i + 1 < p.n_copies && g0 >= p.row_start[i + 1]) ++i;
    const float4* src[R];
    float4* dst[R];
    int width[R];
    float scale[R];
    int maxw = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int64_t g = g0 + j;
      int k = i;
      while (k + 1 < p.n_copies && g >= p.row_start[k + 1]) ++k;
      const bool live = g < total;
      const CopyDesc& c = p.c[k];
      const int64_t r = g - p.row_start[k];
      src[j] = c.src + (live ? r * c.src_ld : 0);
      dst[j] = c.dst + (live ? r * c.dst_ld : 0);
      width[j] = live ? c.width : 0;
      scale[j] = c.scale;
      maxw = max(maxw, width[j]);
    }
    for (int v0 = 0; v0 < maxw; v0 += 32) {
      const int v = v0 + lane;
      float4 x[R];
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (v < width[j]) x[j] = __ldg(src[j] + v);
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (v >= width[j]) continue;
        if (scale[j] != 1.f) {
          x[j].x *= scale[j];
          x[j].y *= scale[j];
          x[j].z *= scale[j];
          x[j].w *= scale[j];
        }
        dst[j][v] = x[j];
      }
    }
  }
  // this block's stores, visible to every GPU before it counts itself done
  __threadfence_system();
  __syncthreads();
  __shared__ int s_last;
  uint32_t* own = p.flags[p.rank];
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(own + (kMaxRanks - 1), 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) own[kMaxRanks - 1] = 0;  // every block has counted: ready for the next launch
  __threadfence_system();
  if (threadIdx.x < p.n_ranks) st_release_sys(p.flags[threadIdx.x] + p.rank, p.epoch);
  if (threadIdx.x < p.n_ranks) {
    const uint64_t t0 = global_ns();
    while ((int32_t)(ld_acquire_sys(own + threadIdx.x) - p.epoch) < 0) {
      if (global_ns() - t0 > p.timeout_ns) {
        flag_error(kErrExchangeTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

}  // namespace nnue
