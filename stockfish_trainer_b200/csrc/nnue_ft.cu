// C ABI of the sparse NNUE feature transformer for B200 (sm_100a).
// Declarations and contracts: include/nnue_ft.h.
//
// One translation unit: the kernels live in the *.cuh files included here.

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nnue_ft.h"
#include "common.cuh"
#include "ft_backward.cuh"
#include "ft_forward.cuh"
#include "ft_epilogue.cuh"
#include "ft_optim.cuh"
#include "ft_quant.cuh"
#include "ft_encode.cuh"
#include "ft_exchange.cuh"

namespace nnue {
namespace {

thread_local std::string g_last_error;
std::atomic<unsigned long long> g_launches{0};  // kernel launches issued by this library

inline void count_launch(unsigned n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Optional per-launch timing of the gather kernels (measurement support, off
// by default).  When a kernel class is armed, a CUDA event pair is recorded
// on the launching stream around each launch of that class, so a caller can
// read the kernel's own duration inside a real step, with whatever runs
// concurrently on other streams.  Not for use under stream capture.
enum TimedKernel : int { kTimeForward = 0, kTimeLight = 1, kTimeHeavy = 2, kTimedKinds = 3 };
struct KernelTimer {
  std::mutex mu;
  std::atomic<unsigned> mask{0};
  std::vector<cudaEvent_t> start, stop;  // capacity pairs, created when armed
  std::vector<int> kind;                 // class of each recorded pair
  void release() {
    for (cudaEvent_t e : start) cudaEventDestroy(e);
    for (cudaEvent_t e : stop) cudaEventDestroy(e);
    start.clear();
    stop.clear();
    kind.clear();
    mask = 0;
  }
};
KernelTimer g_timer;

// Records the start event of a timed launch; returns the pair's slot or -1.
int timer_begin(int k, cudaStream_t s) {
  if (!(g_timer.mask.load(std::memory_order_relaxed) & (1u << k))) return -1;  // unarmed: no lock
  std::lock_guard<std::mutex> lock(g_timer.mu);
  const size_t i = g_timer.kind.size();
  if (!(g_timer.mask.load() & (1u << k)) || i >= g_timer.start.size()) return -1;
  if (cudaEventRecord(g_timer.start[i], s) != cudaSuccess) return -1;
  g_timer.kind.push_back(k);
  return (int)i;
}

void timer_end(int slot, cudaStream_t s) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_timer.mu);
  if ((size_t)slot < g_timer.stop.size()) cudaEventRecord(g_timer.stop[slot], s);
}

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NNUE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return NNUE_OK;
}

struct Tuning {
  int64_t fwd_chunk_vec = 32;       // forward column chunk, in 16-byte vectors
  int64_t fwd_items_per_warp = 16;  // (perspective, position) items per warp
  int64_t fwd_unroll = 6;          // table rows in flight per warp (4, 6 or 8; 5 groups: 2, 3, 4 or 6)
  int64_t bwd_unroll = 2;          // dOut rows per batch, light rows (2, 4 or 8)
  int64_t fwd_min_blocks = 4;      // forward: registers sized for 2..6 resident blocks (chunks <= 64 vectors)
  int64_t bwd_min_blocks = 8;      // light rows: registers sized for 4, 5, 6 or 8 resident blocks (else compiler's)
  int64_t fwd_exact_chunks = 1;    // 1: full-width chunks + narrow tail; 0: balanced widths
  int64_t bwd_exact_chunks = 1;
  int64_t bwd_chunk_vec = 32;      // backward column chunk, in 16-byte vectors
  int64_t heavy_threshold = 256;   // rows with more entries are split finer
  int64_t heavy_cap = 512;         // at most this many heavy rows per call
  int64_t sort_blocks_per_sm = 16;  // counting placement: grid of the two passes over the index arrays
  int64_t colsum_parts = 296;      // position ranges of the bias column sum
  int64_t fwd_block = 128;         // forward (1 vector per lane, 4 blocks' registers): threads per block, 256 or 128
  int64_t bwd_block = 128;         // light rows: threads per block (256, 128 or 64; 1 vector per lane, 2-row batches)
  int64_t bwd_queue = 2;           // light rows, one vector per lane: register-queue depth (2, 3, 4 or 6; 0 = batches)
  int64_t bwd_queue_min_blocks = 16;  // queued light rows: register budget for 8, 12 or 16 resident 128-thread blocks
  // queued light rows only when the expected entries per row, B * P * K / (4 T), reach this: on B200 the queue
  // is 7-8% faster at ~60 entries per row (B = 65536, Full_Threats+HalfKAv2_hm^), even at ~15 and 5% slower at ~8
  int64_t bwd_queue_min_entries = 32;
  // forward, one vector per lane: index groups of 32 slots read per item, 1, 5 or 8; 0 = the fewest covering K
  // (1 for K <= 32, 5 for K <= 160): on B200 5 groups instead of 8 made the K = 160 forward 4% faster
  int64_t fwd_groups = 0;
  int64_t fwd_queue_blocks = 8;    // forward with 1 or 5 groups: register budget for 8, 12 or 16 resident 128-thread blocks
  // the narrow last column chunk packed several items (forward) / rows (light rows) per warp: 0 off, 1 on the
  // caller's stream, 2 on the library's side stream beside the main kernel (where the call forks one), 3 (forward
  // only) as 2 from 2^17 items (both perspectives) up, else off.  On B200 the packed light-row tail on the side
  // stream made the step 2-4% faster at every size; the forward's only at the largest batches (1.5% at 2 x 65536
  // items, 1.5% slower at 2 x 8192).
  int64_t fwd_tail = 3;
  int64_t bwd_tail = 2;
  // where the heavy rows run: 0 = on the side stream after the packed tail chunk, beside the light rows;
  // 1 = the same, before the tail chunk (their long sequential walks start at once: the longest side-stream
  // task when the light rows are short, as on a narrow column slice); 2 = alone on the caller's stream before
  // the light rows (beside 64 light warps per SM each heavy warp gets a small share of the issue slots)
  int64_t bwd_heavy_first = 0;
  // exchange kernel: rows each warp copies at once (1, 2 or 4) and resident blocks per SM (grid size); on 4
  // B200s 2 rows and 8 blocks moved the column-sharded step's 103 MB per rank in 0.26 ms (1 and 4: 0.30 ms)
  int64_t xchg_rows = 2;
  int64_t xchg_blocks_per_sm = 8;
};
Tuning g_tune;

struct ParamRef {
  const char* name;
  int64_t* field;
  int64_t lo, hi;
};

ParamRef* params() {
  static ParamRef p[] = {
      {"fwd_chunk_vec", &g_tune.fwd_chunk_vec, 0, 1 << 20},
      {"fwd_items_per_warp", &g_tune.fwd_items_per_warp, 1, 1024},
      {"fwd_unroll", &g_tune.fwd_unroll, 2, 8},
      {"bwd_unroll", &g_tune.bwd_unroll, 2, 8},
      {"fwd_exact_chunks", &g_tune.fwd_exact_chunks, 0, 1},
      {"bwd_exact_chunks", &g_tune.bwd_exact_chunks, 0, 1},
      {"fwd_min_blocks", &g_tune.fwd_min_blocks, 0, 6},
      {"bwd_min_blocks", &g_tune.bwd_min_blocks, 0, 8},
      {"bwd_chunk_vec", &g_tune.bwd_chunk_vec, 0, 1 << 20},
      {"heavy_threshold", &g_tune.heavy_threshold, 1, int64_t(1) << 40},
      {"heavy_cap", &g_tune.heavy_cap, 0, 1 << 24},
      {"sort_blocks_per_sm", &g_tune.sort_blocks_per_sm, 1, 1 << 16},
      {"colsum_parts", &g_tune.colsum_parts, 1, 1 << 16},
      {"bwd_block", &g_tune.bwd_block, 64, 256},
      {"fwd_block", &g_tune.fwd_block, 128, 256},
      {"bwd_queue", &g_tune.bwd_queue, 0, 6},
      {"bwd_queue_min_blocks", &g_tune.bwd_queue_min_blocks, 8, 16},
      {"bwd_queue_min_entries", &g_tune.bwd_queue_min_entries, 0, int64_t(1) << 40},
      {"fwd_groups", &g_tune.fwd_groups, 0, 8},
      {"fwd_queue_blocks", &g_tune.fwd_queue_blocks, 8, 16},
      {"fwd_tail", &g_tune.fwd_tail, 0, 3},
      {"bwd_tail", &g_tune.bwd_tail, 0, 2},
      {"bwd_heavy_first", &g_tune.bwd_heavy_first, 0, 2},
      {"xchg_rows", &g_tune.xchg_rows, 1, 4},
      {"xchg_blocks_per_sm", &g_tune.xchg_blocks_per_sm, 1, 16},
      {nullptr, nullptr, 0, 0},
  };
  return p;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Column geometry: ceil(n_vec / chunk) balanced chunks, chunk clamped to
// [8, 256] vectors, so a lane never needs more than 8 vectors (the widest
// kernel instance).  `chunk` <= 0 asks for one chunk per row when the row
// has <= 256 vectors.
constexpr int kMaxLaneVectors = 8;

Geom make_geom(int32_t n_vec, int64_t chunk, bool exact) {
  Geom g;
  g.n_vec = n_vec;
  if (chunk <= 0) chunk = 32 * kMaxLaneVectors;
  chunk = std::min<int64_t>(std::max<int64_t>(chunk, 8), 32 * kMaxLaneVectors);
  g.n_chunks = (int32_t)std::max<int64_t>(1, ceil_div(n_vec, chunk));
  g.exact = exact ? 1 : 0;
  g.max_width = exact ? (int32_t)std::min<int64_t>(chunk, n_vec) : (int32_t)ceil_div(n_vec, g.n_chunks);
  return g;
}

int lanes_per_row(const Geom& g) { return (g.max_width + 31) / 32; }

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// Forward, one vector per lane, IG index groups per item (K <= 32 * IG in
// one pass): 128-thread blocks, register budget for BLOCKS resident blocks.
template <typename VT, int IG, int D, int BLOCKS>
void launch_forward_g(const FwdParams& p, dim3 g4, cudaStream_t s) {
  if (p.tabs.n > 1) ft_forward_kernel<VT, 1, D, BLOCKS, true, 128, IG><<<g4, 128, 0, s>>>(p);
  else ft_forward_kernel<VT, 1, D, BLOCKS, false, 128, IG><<<g4, 128, 0, s>>>(p);
}

template <typename VT, int IG>
void launch_forward_g_any(const FwdParams& p, dim3 g4, cudaStream_t s) {
  const int64_t b = g_tune.fwd_queue_blocks, d = g_tune.fwd_unroll;
  if (b >= 16) {
    if (d <= 2) launch_forward_g<VT, IG, 2, 16>(p, g4, s);
    else launch_forward_g<VT, IG, 3, 16>(p, g4, s);
  } else if (b >= 12) {
    if (d <= 3) launch_forward_g<VT, IG, 3, 12>(p, g4, s);
    else launch_forward_g<VT, IG, 4, 12>(p, g4, s);
  } else {
    if (d <= 4) launch_forward_g<VT, IG, 4, 8>(p, g4, s);
    else launch_forward_g<VT, IG, 6, 8>(p, g4, s);
  }
}

template <typename VT, int V, int D, int MINB>
void launch_forward_vd(FwdParams p, int chunk0, int n_chunks, cudaStream_t s) {
  const int64_t n_items = (int64_t)p.P * p.B;
  const int64_t warps = ceil_div(n_items, p.items_per_warp);
  p.chunk0 = chunk0;
  dim3 grid((unsigned)ceil_div(warps, kWarpsPerBlock), (unsigned)n_chunks);
  count_launch();
  if constexpr (V == 1) {
    const int64_t groups = g_tune.fwd_groups ? g_tune.fwd_groups : (p.K <= 32 ? 1 : p.K <= 160 ? 5 : 8);
    if (groups < 8 && g_tune.fwd_block == 128) {
      const dim3 g4((unsigned)ceil_div(warps, 4), (unsigned)n_chunks);
      if (groups <= 1) launch_forward_g_any<VT, 1>(p, g4, s);
      else launch_forward_g_any<VT, 5>(p, g4, s);
      return;
    }
  }
  if constexpr (MINB == 4 && V == 1) {
    if (g_tune.fwd_block == 128) {  // blocks of 4 warps, registers as for 4 blocks of 8
      dim3 g4((unsigned)ceil_div(warps, 4), (unsigned)n_chunks);
      if (p.tabs.n > 1) ft_forward_kernel<VT, V, D, 8, true, 128><<<g4, 128, 0, s>>>(p);
      else ft_forward_kernel<VT, V, D, 8, false, 128><<<g4, 128, 0, s>>>(p);
      return;
    }
  }
  if (p.tabs.n > 1) ft_forward_kernel<VT, V, D, MINB, true><<<grid, kBlock, 0, s>>>(p);
  else ft_forward_kernel<VT, V, D, MINB, false><<<grid, kBlock, 0, s>>>(p);
}

template <typename VT, int V, int D>
void launch_forward_vd(const FwdParams& p, int chunk0, int n_chunks, cudaStream_t s) {
  // two vectors per lane need twice the registers: cap their budget at 3 blocks
  switch (V == 1 ? g_tune.fwd_min_blocks : std::min<int64_t>(g_tune.fwd_min_blocks, 3)) {
    case 3: launch_forward_vd<VT, V, D, 3>(p, chunk0, n_chunks, s); return;
    case 4: launch_forward_vd<VT, V, D, 4>(p, chunk0, n_chunks, s); return;
    case 5: launch_forward_vd<VT, V, D, 5>(p, chunk0, n_chunks, s); return;
    case 6: launch_forward_vd<VT, V, D, 6>(p, chunk0, n_chunks, s); return;
    default: launch_forward_vd<VT, V, D, 2>(p, chunk0, n_chunks, s); return;
  }
}

template <typename VT, int V>
void launch_forward_v(const FwdParams& p, int chunk0, int n_chunks, cudaStream_t s) {
  if constexpr (V <= 2) {
    if (g_tune.fwd_unroll >= 8) launch_forward_vd<VT, V, 8>(p, chunk0, n_chunks, s);
    else if (g_tune.fwd_unroll >= 6) launch_forward_vd<VT, V, 6>(p, chunk0, n_chunks, s);
    else launch_forward_vd<VT, V, 4>(p, chunk0, n_chunks, s);
  } else {
    launch_forward_vd<VT, V, 4, 1>(p, chunk0, n_chunks, s);  // wide chunks: compiler's register budget
  }
}

template <typename VT>
void launch_forward_range(const FwdParams& p, int chunk0, int n_chunks, int width, cudaStream_t s) {
  switch ((width + 31) / 32) {
    case 1: launch_forward_v<VT, 1>(p, chunk0, n_chunks, s); break;
    case 2: launch_forward_v<VT, 2>(p, chunk0, n_chunks, s); break;
    case 3: launch_forward_v<VT, 3>(p, chunk0, n_chunks, s); break;
    case 4: launch_forward_v<VT, 4>(p, chunk0, n_chunks, s); break;
    default: launch_forward_v<VT, 8>(p, chunk0, n_chunks, s); break;
  }
}

// The packed narrow last chunk (ft_forward_tail_kernel): W = the tail's width.
template <int W, int IG>
void launch_forward_tail_w(FwdParams p, cudaStream_t s) {
  constexpr int G = 32 / W;
  p.items_per_warp = 1;  // one packed group of G items per warp: enough warps at small batches
  const int64_t n_items = (int64_t)p.P * p.B;
  const int64_t warps = ceil_div(n_items, (int64_t)p.items_per_warp * G);
  count_launch();
  ft_forward_tail_kernel<W, 6, IG, 8, 128><<<(unsigned)ceil_div(warps, 4), 128, 0, s>>>(p);
}

template <int IG>
bool launch_forward_tail_ig(const FwdParams& p, int width, cudaStream_t s) {
  switch (width) {
    case 2: launch_forward_tail_w<2, IG>(p, s); return true;
    case 3: launch_forward_tail_w<3, IG>(p, s); return true;
    case 4: launch_forward_tail_w<4, IG>(p, s); return true;
    case 6: launch_forward_tail_w<6, IG>(p, s); return true;
    case 8: launch_forward_tail_w<8, IG>(p, s); return true;
    default: return false;
  }
}

// Launches the packed tail kernel for the last column chunk when it applies
// (16-byte vectors, one table, full-width chunks + a narrow tail, K covered by
// one index pass); returns whether it did.
template <typename VT>
bool launch_forward_tail(const FwdParams& p, cudaStream_t s) {
  if (!std::is_same<VT, float4>::value || !p.g.exact || p.g.n_chunks < 2 || p.tabs.n > 1) return false;
  const int width = p.g.width(p.g.n_chunks - 1);
  if (width >= p.g.max_width || width > 8 || p.g.max_width > 32) return false;
  if (p.K <= 32) return launch_forward_tail_ig<1>(p, width, s);
  if (p.K <= 160) return launch_forward_tail_ig<5>(p, width, s);
  return false;
}

// fwd_tail: 0 the last chunk like the others; 1 packed, on the caller's
// stream before the main gather; 2 packed, on the forked side stream when
// there is one (beside the main gather), else as 1; 3 as 2 for large batches.
template <typename VT>
void launch_forward(const FwdParams& p, cudaStream_t s, cudaStream_t side) {
  const int slot = timer_begin(kTimeForward, s);
  int64_t mode = g_tune.fwd_tail;
  if (mode == 3) mode = (int64_t)p.P * p.B >= (int64_t(1) << 17) ? 2 : 0;
  bool packed = false;
  if (mode) packed = launch_forward_tail<VT>(p, mode == 2 && side ? side : s);
  launch_forward_range<VT>(p, 0, p.g.n_chunks - (packed ? 1 : 0), p.g.max_width, s);
  timer_end(slot, s);
}

// Builds a table set from per-block pointers and row counts (n_tables >= 1).
int make_tables(const char* what, float* const* bases, const int64_t* rows, int32_t n_tables, TableSet& t,
                int64_t& total) {
  if (n_tables < 1 || n_tables > kMaxTables)
    return fail(NNUE_ERR_UNSUPPORTED, "%s: 1..%d tables supported, got %d", what, kMaxTables, (int)n_tables);
  if (!bases || !rows) return fail(NNUE_ERR_INVALID_ARGUMENT, "%s: null table list", what);
  t = TableSet{};
  t.n = n_tables;
  total = 0;
  for (int i = 0; i < n_tables; ++i) {
    if (rows[i] < 0) return fail(NNUE_ERR_INVALID_ARGUMENT, "%s: negative row count", what);
    if (rows[i] > 0 && !bases[i]) return fail(NNUE_ERR_INVALID_ARGUMENT, "%s: null table %d", what, i);
    total += rows[i];
    if (total > INT32_MAX) return fail(NNUE_ERR_UNSUPPORTED, "%s: tables exceed int32 index range", what);
    t.base[i] = bases[i];
    t.end[i] = (int32_t)total;
  }
  return NNUE_OK;
}

bool tables_aligned16(const TableSet& t) {
  for (int i = 0; i < t.n; ++i)
    if (!aligned16(t.base[i])) return false;
  return true;
}

// `side`: a stream already forked from `s` (joined back by the caller), or
// null; the packed tail chunk may run there, beside the main gather.
int forward_impl(const int32_t* idx0, const int32_t* idx1, int P, int64_t B, int32_t K, const float* W,
                 int64_t T, int32_t C, const float* bias, float* out0, float* out1, cudaStream_t s,
                 const TableSet* tabs = nullptr, cudaStream_t side = nullptr) {
  if (B < 0 || K < 0 || T < 0 || C <= 0) return fail(NNUE_ERR_INVALID_ARGUMENT, "forward: bad sizes");
  if (T > INT32_MAX) return fail(NNUE_ERR_UNSUPPORTED, "forward: num_inputs exceeds int32 index range");
  if (B == 0) return NNUE_OK;
  if (!idx0 || !out0 || !bias || (T > 0 && !W && !tabs) || (P == 2 && (!idx1 || !out1)))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "forward: null pointer");
  const bool v4 = (C % 4 == 0) && (tabs ? tables_aligned16(*tabs) : aligned16(W)) && aligned16(bias) &&
                  aligned16(out0) && (P == 1 || aligned16(out1));
  FwdParams p{};
  p.idx[0] = idx0;
  p.idx[1] = P == 2 ? idx1 : idx0;
  p.out[0] = out0;
  p.out[1] = P == 2 ? out1 : out0;
  p.W = W;
  p.bias = bias;
  p.B = B;
  p.K = K;
  p.T = (int32_t)T;
  p.P = P;
  p.items_per_warp = (int32_t)g_tune.fwd_items_per_warp;
  if (tabs && tabs->n > 1) p.tabs = *tabs;
  else p.tabs.n = 1;
  if (tabs && tabs->n == 1) p.W = tabs->base[0];
  p.g = v4 ? make_geom(C / 4, g_tune.fwd_chunk_vec, g_tune.fwd_exact_chunks)
             : make_geom(C, g_tune.fwd_chunk_vec * 4, g_tune.fwd_exact_chunks);
  if (lanes_per_row(p.g) > kMaxLaneVectors) return fail(NNUE_ERR_UNSUPPORTED, "forward: column chunk too wide");
  if (T * (int64_t)p.g.n_vec > INT32_MAX)
    return fail(NNUE_ERR_UNSUPPORTED, "forward: table exceeds 2^31 %s", v4 ? "16-byte vectors" : "floats");
  if (v4) launch_forward<float4>(p, s, side);
  else launch_forward<float>(p, s, side);
  return check_launch("forward");
}

// ---------------------------------------------------------------------------
// backward plan: workspace layout shared by prepare / apply / size query
// ---------------------------------------------------------------------------
struct BwdPlan {
  int64_t B = 0, T = 0, NK = 0, nnz_max = 0;
  int32_t K = 0, C = 0, P = 0;
  int64_t scan_blocks = 0;
  int64_t heavy_cap = 0, heavy_threshold = 0, parts = 0;
  size_t off_seg = 0, off_bsum = 0, off_ka = 0, off_va = 0;
  size_t off_nheavy = 0, off_heavy = 0, off_kind = 0, off_partial = 0, off_cursor = 0, off_big = 0;
  size_t off_hpart = 0, off_hticket = 0;
  size_t total = 0;
};

int make_plan(int64_t B, int32_t K, int64_t T, int32_t C, int32_t P, BwdPlan& pl) {
  if (P != 1 && P != 2) return fail(NNUE_ERR_INVALID_ARGUMENT, "backward: n_persp must be 1 or 2");
  if (B < 0 || K < 0 || T <= 0 || C <= 0) return fail(NNUE_ERR_INVALID_ARGUMENT, "backward: bad sizes");
  // the segment sort counts repeats of one position in 16-bit counters
  if (K >= 65536) return fail(NNUE_ERR_UNSUPPORTED, "backward: max_active must be < 65536");
  pl.B = B;
  pl.K = K;
  pl.T = T;
  pl.C = C;
  pl.P = P;
  pl.NK = T * P;
  if (pl.NK >= (int64_t(1) << 30))
    return fail(NNUE_ERR_UNSUPPORTED, "backward: num_inputs * n_persp must be < 2^30");
  pl.nnz_max = (int64_t)P * B * K;
  if (pl.nnz_max >= INT32_MAX) return fail(NNUE_ERR_UNSUPPORTED, "backward: n_persp * batch * max_active >= 2^31");
  pl.scan_blocks = ceil_div(pl.NK + 1, kScanTile);
  pl.heavy_cap = std::min<int64_t>(g_tune.heavy_cap, T);
  pl.heavy_threshold = g_tune.heavy_threshold;
  pl.parts = std::max<int64_t>(1, std::min<int64_t>(g_tune.colsum_parts, B));
  const int64_t n_vec_floats = C;  // float64 partial column sums
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + std::max<size_t>(bytes, 1));
    return at;
  };
  pl.off_seg = take(sizeof(int32_t) * (pl.NK + 1));
  pl.off_bsum = take(sizeof(int32_t) * (pl.scan_blocks + 1));
  pl.off_ka = take(sizeof(int32_t) * pl.nnz_max);  // spare values (long-segment sort)
  pl.off_va = take(sizeof(int32_t) * pl.nnz_max);  // the sorted values
  pl.off_nheavy = take(sizeof(int32_t));
  pl.off_heavy = take(sizeof(int32_t) * pl.heavy_cap);
  pl.off_kind = take(sizeof(uint8_t) * T);
  pl.off_partial = take(sizeof(double) * P * pl.parts * n_vec_floats);
  pl.off_cursor = take(sizeof(int32_t) * pl.NK);
  pl.off_big = take(sizeof(int32_t) * (pl.NK + 1));
  pl.off_hpart = take(P == 2 ? sizeof(float) * pl.heavy_cap * 2 * C : 0);
  pl.off_hticket = take(P == 2 ? sizeof(uint32_t) * pl.heavy_cap * C : 0);
  pl.total = o;
  return NNUE_OK;
}

struct Ws {
  int32_t *seg, *bsum, *ka, *va, *nheavy, *heavy;
  uint8_t* kind;
  double* partial;
  int32_t *cursor, *big;
  float* hpart;
  uint32_t* hticket;
};

Ws carve(const BwdPlan& pl, void* base) {
  char* b = static_cast<char*>(base);
  Ws w;
  w.seg = reinterpret_cast<int32_t*>(b + pl.off_seg);
  w.bsum = reinterpret_cast<int32_t*>(b + pl.off_bsum);
  w.ka = reinterpret_cast<int32_t*>(b + pl.off_ka);
  w.va = reinterpret_cast<int32_t*>(b + pl.off_va);
  w.nheavy = reinterpret_cast<int32_t*>(b + pl.off_nheavy);
  w.heavy = reinterpret_cast<int32_t*>(b + pl.off_heavy);
  w.kind = reinterpret_cast<uint8_t*>(b + pl.off_kind);
  w.partial = reinterpret_cast<double*>(b + pl.off_partial);
  w.cursor = reinterpret_cast<int32_t*>(b + pl.off_cursor);
  w.big = reinterpret_cast<int32_t*>(b + pl.off_big);
  w.hpart = reinterpret_cast<float*>(b + pl.off_hpart);
  w.hticket = reinterpret_cast<uint32_t*>(b + pl.off_hticket);
  return w;
}

// the sorted position lists (grouped by key, ascending within a key)
const int32_t* sorted_values(const BwdPlan&, const Ws& w) { return w.va; }

void run_scan(int32_t* data, ScanLen L, int64_t max_len, int32_t* bsum, cudaStream_t s) {
  const int64_t nb = ceil_div(max_len, kScanTile);
  if (nb == 0) return;
  count_launch();
  scan_reduce_kernel<<<(unsigned)nb, kBlock, 0, s>>>(data, L, bsum);
  count_launch();
  scan_top_kernel<<<1, 1024, 0, s>>>(bsum, nb);
  count_launch();
  scan_down_kernel<<<(unsigned)nb, kBlock, 0, s>>>(data, data, L, bsum);
}

int prepare_impl(const int32_t* idx0, const int32_t* idx1, const BwdPlan& pl, const Ws& w, cudaStream_t s) {
  if (cudaMemsetAsync(w.seg, 0, sizeof(int32_t) * (pl.NK + 1), s) != cudaSuccess ||
      cudaMemsetAsync(w.nheavy, 0, sizeof(int32_t), s) != cudaSuccess)
    return check_launch("backward_prepare: memset");
  RawSrc raw{};
  raw.idx[0] = idx0;
  raw.idx[1] = pl.P == 2 ? idx1 : idx0;
  raw.n_raw = pl.B * pl.K;
  raw.K = pl.K;
  raw.T = (int32_t)pl.T;
  raw.P = pl.P;
  if (cudaMemsetAsync(w.big, 0, sizeof(int32_t), s) != cudaSuccess) return check_launch("backward_prepare: memset");
  const unsigned grid = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>(ceil_div(raw.n_raw, 4 * kBlock), 148 * g_tune.sort_blocks_per_sm));
  count_launch();
  count_keys_kernel<<<grid, kBlock, 0, s>>>(raw, w.seg);
  run_scan(w.seg, ScanLen{pl.NK + 1}, pl.NK + 1, w.bsum, s);
  if (cudaMemcpyAsync(w.cursor, w.seg, sizeof(int32_t) * pl.NK, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return check_launch("backward_prepare: cursor copy");
  count_launch();
  place_keys_kernel<<<grid, kBlock, 0, s>>>(raw, w.cursor, w.va, pl.nnz_max);
  count_launch();
  order_segments_kernel<<<(unsigned)ceil_div(pl.NK, kWarpsPerBlock), kBlock, 0, s>>>(w.seg, pl.NK, w.va, w.big);
  count_launch();
  order_big_segments_kernel<<<(unsigned)std::min<int64_t>(pl.NK, 2 * 148), kBigThreads, 0, s>>>(
      w.seg, pl.P, pl.B, w.va, w.ka, w.big);
  count_launch();
  classify_rows_kernel<<<(unsigned)ceil_div(pl.T, kBlock), kBlock, 0, s>>>(
      w.seg, (int32_t)pl.T, pl.P, (int32_t)std::min<int64_t>(pl.heavy_threshold, INT32_MAX),
      (int32_t)pl.heavy_cap, w.nheavy, w.heavy, w.kind);
  return check_launch("backward_prepare");
}

template <typename VT, int V, int U>
void launch_segsum_vu(SegParams p, int chunk0, int n_chunks, cudaStream_t s) {
  p.chunk0 = chunk0;
  dim3 grid((unsigned)ceil_div(p.row_end - p.row_begin, kWarpsPerBlock), (unsigned)n_chunks);
  count_launch();
  if constexpr (V == 1 && U == 2) {
    // smaller blocks: a block's warp slots are released only when its
    // longest row is done, and light rows differ widely in length
    const int64_t rows = p.row_end - p.row_begin;
    if (g_tune.bwd_block == 64 && g_tune.bwd_min_blocks == 8) {
      ft_segsum_light_kernel<VT, 1, 2, 32, 64><<<dim3((unsigned)ceil_div(rows, 2), (unsigned)n_chunks), 64, 0, s>>>(p);
      return;
    }
    if (g_tune.bwd_block == 128 && g_tune.bwd_min_blocks == 8) {
      ft_segsum_light_kernel<VT, 1, 2, 16, 128><<<dim3((unsigned)ceil_div(rows, 4), (unsigned)n_chunks), 128, 0, s>>>(
          p);
      return;
    }
  }
  if constexpr (V <= 2) {
    // two vectors per lane need twice the registers: cap their budget at 4 blocks
    switch (V == 1 ? g_tune.bwd_min_blocks : std::min<int64_t>(g_tune.bwd_min_blocks, 4)) {
      case 4: ft_segsum_light_kernel<VT, V, U, 4><<<grid, kBlock, 0, s>>>(p); return;
      case 5: ft_segsum_light_kernel<VT, V, U, 5><<<grid, kBlock, 0, s>>>(p); return;
      case 6: ft_segsum_light_kernel<VT, V, U, 6><<<grid, kBlock, 0, s>>>(p); return;
      case 8: ft_segsum_light_kernel<VT, V, U, 8><<<grid, kBlock, 0, s>>>(p); return;
      default: break;
    }
  }
  ft_segsum_light_kernel<VT, V, U><<<grid, kBlock, 0, s>>>(p);
}

template <typename VT, int V>
void launch_segsum_v(const SegParams& p, int chunk0, int n_chunks, cudaStream_t s) {
  if constexpr (V <= 2) {
    if (g_tune.bwd_unroll >= 8) launch_segsum_vu<VT, V, 8>(p, chunk0, n_chunks, s);
    else if (g_tune.bwd_unroll <= 2) launch_segsum_vu<VT, V, 2>(p, chunk0, n_chunks, s);
    else launch_segsum_vu<VT, V, 4>(p, chunk0, n_chunks, s);
  } else if constexpr (V <= 4) {
    launch_segsum_vu<VT, V, 4>(p, chunk0, n_chunks, s);
  } else {
    launch_segsum_vu<VT, V, 2>(p, chunk0, n_chunks, s);
  }
}

template <typename VT>
void launch_segsum_range(const SegParams& p, int chunk0, int n_chunks, int width, cudaStream_t s) {
  switch ((width + 31) / 32) {
    case 1: launch_segsum_v<VT, 1>(p, chunk0, n_chunks, s); break;
    case 2: launch_segsum_v<VT, 2>(p, chunk0, n_chunks, s); break;
    case 3: launch_segsum_v<VT, 3>(p, chunk0, n_chunks, s); break;
    case 4: launch_segsum_v<VT, 4>(p, chunk0, n_chunks, s); break;
    default: launch_segsum_v<VT, 8>(p, chunk0, n_chunks, s); break;
  }
}

template <int D, int MINB, int THREADS = 128>
void launch_segsum_queue_d(SegParams p, int n_chunks, cudaStream_t s) {
  const int64_t rows = p.row_end - p.row_begin;
  p.chunk0 = 0;
  count_launch();
  ft_segsum_lightq_kernel<D, MINB, THREADS>
      <<<dim3((unsigned)ceil_div(rows, THREADS / 32), (unsigned)n_chunks), THREADS, 0, s>>>(p);
}

// Queued light rows (one vector per lane) over column chunks [0, n_chunks):
// depth x register budget (x block size: 128 threads, or 64 with 32 resident
// blocks).
bool launch_segsum_queue(const SegParams& p, int n_chunks, cudaStream_t s) {
  const int64_t mb = g_tune.bwd_queue_min_blocks;
  if (g_tune.bwd_block == 64 && mb >= 16 && (g_tune.bwd_queue == 2 || g_tune.bwd_queue == 3)) {
    if (g_tune.bwd_queue == 2) launch_segsum_queue_d<2, 32, 64>(p, n_chunks, s);
    else launch_segsum_queue_d<3, 32, 64>(p, n_chunks, s);
    return true;
  }
  switch (g_tune.bwd_queue) {
    case 2: launch_segsum_queue_d<2, 16>(p, n_chunks, s); return true;
    case 3:
      if (mb >= 16) launch_segsum_queue_d<3, 16>(p, n_chunks, s);
      else launch_segsum_queue_d<3, 12>(p, n_chunks, s);
      return true;
    case 4:
      if (mb >= 16) launch_segsum_queue_d<4, 16>(p, n_chunks, s);
      else if (mb >= 12) launch_segsum_queue_d<4, 12>(p, n_chunks, s);
      else launch_segsum_queue_d<4, 8>(p, n_chunks, s);
      return true;
    case 6:
      if (mb >= 12) launch_segsum_queue_d<6, 12>(p, n_chunks, s);
      else launch_segsum_queue_d<6, 8>(p, n_chunks, s);
      return true;
    default: return false;
  }
}

// The packed narrow last chunk of the light rows (ft_segsum_tail_kernel).
template <int W>
void launch_segsum_tail_w(const SegParams& p, cudaStream_t s) {
  constexpr int G = 32 / W < 15 ? 32 / W : 15;  // rows per warp, as in ft_segsum_tail_kernel
  const int64_t rows = p.row_end - p.row_begin;
  count_launch();
  ft_segsum_tail_kernel<W, 4><<<(unsigned)ceil_div(rows, 4 * G), 128, 0, s>>>(p);
}

// Launches the packed tail kernel for the last column chunk when it applies
// (16-byte vectors addressed from dout[0], full-width chunks + a narrow tail);
// returns whether it did.
bool launch_segsum_tail(const SegParams& p, bool delta_ok, cudaStream_t s) {
  if (!delta_ok || !p.g.exact || p.g.n_chunks < 2 || p.g.max_width > 32) return false;
  switch (p.g.width(p.g.n_chunks - 1)) {
    case 2: launch_segsum_tail_w<2>(p, s); return true;
    case 3: launch_segsum_tail_w<3>(p, s); return true;
    case 4: launch_segsum_tail_w<4>(p, s); return true;
    case 6: launch_segsum_tail_w<6>(p, s); return true;
    case 8: launch_segsum_tail_w<8>(p, s); return true;
    default: return false;
  }
}

// tail_done: the packed last chunk was already launched on the side stream.
template <typename VT>
void launch_segsum_light(const SegParams& p, bool queue_ok, bool delta_ok, bool tail_done, cudaStream_t s) {
  const int slot = timer_begin(kTimeLight, s);
  int n_chunks = p.g.n_chunks;
  if (tail_done) --n_chunks;
  else if (std::is_same<VT, float4>::value && g_tune.bwd_tail == 1 && launch_segsum_tail(p, delta_ok, s)) --n_chunks;
  if (!(std::is_same<VT, float4>::value && queue_ok && lanes_per_row(p.g) == 1 && launch_segsum_queue(p, n_chunks, s)))
    launch_segsum_range<VT>(p, 0, n_chunks, p.g.max_width, s);
  timer_end(slot, s);
}

template <typename VT>
constexpr size_t heavy_smem_bytes() {
  return sizeof(VT) * 32 * kHeavyStages * kHeavyWarps;
}

template <typename VT>
int launch_segsum_heavy(SegParams p, cudaStream_t s) {
  if (p.heavy_cap == 0) return NNUE_OK;
  constexpr size_t smem = heavy_smem_bytes<VT>();
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(ft_segsum_heavy_kernel<VT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return check_launch("backward_apply: heavy kernel shared memory");
  const int pieces_max = lanes_per_row(p.g);
  p.chunk0 = 0;
  dim3 grid((unsigned)ceil_div((int64_t)p.heavy_cap * pieces_max * p.P, kHeavyWarps), (unsigned)p.g.n_chunks);
  count_launch();
  const int slot = timer_begin(kTimeHeavy, s);
  ft_segsum_heavy_kernel<VT><<<grid, 32 * kHeavyWarps, smem, s>>>(p);
  timer_end(slot, s);
  return NNUE_OK;
}

// The encoder's lookup tables live in a static device array (no device
// allocation); each device gets its copy on its first encoder call, a
// synchronous upload.
__device__ nnue_feat::FeatureTables g_enc_tables_dev;
std::mutex g_enc_mu;
const nnue_feat::FeatureTables* g_enc_tables[64] = {};

int encoder_tables(const nnue_feat::FeatureTables** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("encode_features: device");
  if (dev < 0 || dev >= 64) return fail(NNUE_ERR_UNSUPPORTED, "encode_features: device %d", dev);
  std::lock_guard<std::mutex> lock(g_enc_mu);
  if (!g_enc_tables[dev]) {
    void* d = nullptr;
    if (cudaMemcpyToSymbol(g_enc_tables_dev, &nnue_feat::feature_tables(), sizeof(nnue_feat::FeatureTables)) !=
            cudaSuccess ||
        cudaGetSymbolAddress(&d, g_enc_tables_dev) != cudaSuccess)
      return check_launch("encode_features: table upload");
    g_enc_tables[dev] = static_cast<const nnue_feat::FeatureTables*>(d);
  }
  *out = g_enc_tables[dev];
  return NNUE_OK;
}

// Per-device side stream + fork/join events.  Heavy rows and the bias column
// sum run there, concurrently with the light-row kernel on the caller's
// stream.  Created once per device and kept for the life of the process.
struct DeviceAux {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_aux_mu;
DeviceAux g_aux[64];

int device_aux(DeviceAux** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(NNUE_ERR_UNSUPPORTED, "device ordinal %d >= 64", dev);
  DeviceAux& a = g_aux[dev];
  if (!a.side) {
    int lo = 0, hi = 0;
    if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
        cudaStreamCreateWithPriority(&a.side, cudaStreamNonBlocking, hi) != cudaSuccess ||
        cudaEventCreateWithFlags(&a.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&a.join, cudaEventDisableTiming) != cudaSuccess)
      return check_launch("creating the side stream");
  }
  *out = &a;
  return NNUE_OK;
}

void launch_colsum(const float* g0, const float* g1, const BwdPlan& pl, bool vec4, double* partial, float* dB,
                   int32_t accumulate, cudaStream_t s) {
  ColParams c{};
  c.dout[0] = g0;
  c.dout[1] = pl.P == 2 ? g1 : g0;
  c.B = pl.B;
  c.P = pl.P;
  c.C = pl.C;
  c.parts = (int32_t)pl.parts;
  c.vec4 = vec4 ? 1 : 0;
  c.partial = partial;
  count_launch();
  colsum_partial_kernel<<<dim3((unsigned)pl.parts, (unsigned)pl.P), kBlock, 0, s>>>(c);
  count_launch();
  colsum_final_kernel<<<(unsigned)ceil_div(pl.C, kWarpsPerBlock), kBlock, 0, s>>>(partial, pl.P, (int32_t)pl.parts,
                                                                                 pl.C, dB, accumulate);
}

int apply_impl(const float* g0, const float* g1, const BwdPlan& pl, const Ws& w, float* dW, float* dB,
               int32_t accumulate, int64_t row_begin, int64_t row_end, bool with_bias, cudaStream_t s,
               const TableSet* dws = nullptr) {
  if (row_begin < 0 || row_end > pl.T || row_begin > row_end)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "backward_apply: row range [%lld, %lld) outside [0, %lld)",
                (long long)row_begin, (long long)row_end, (long long)pl.T);
  if (row_begin == row_end && !with_bias) return NNUE_OK;
  const bool v4 = (pl.C % 4 == 0) && aligned16(g0) && (pl.P == 1 || aligned16(g1)) &&
                  (dws ? tables_aligned16(*dws) : aligned16(dW)) && (!with_bias || aligned16(dB)) &&
                  aligned16(w.partial);
  SegParams p{};
  p.dout[0] = g0;
  p.dout[1] = pl.P == 2 ? g1 : g0;
  p.sorted_b = sorted_values(pl, w);
  p.seg_start = w.seg;
  p.heavy_list = w.heavy;
  p.n_heavy = w.nheavy;
  p.row_kind = w.kind;
  p.dW = dW;
  p.B = pl.B;
  p.T = (int32_t)pl.T;
  p.P = pl.P;
  p.accumulate = accumulate ? 1 : 0;
  p.heavy_cap = (int32_t)pl.heavy_cap;
  p.row_begin = (int32_t)row_begin;
  p.row_end = (int32_t)row_end;
  if (dws && dws->n > 1) p.dws = *dws;
  else p.dws.n = 1;
  p.heavy_part = w.hpart;
  p.heavy_ticket = w.hticket;
  if (dws && dws->n == 1) p.dW = dws->base[0];
  p.g = v4 ? make_geom(pl.C / 4, g_tune.bwd_chunk_vec, g_tune.bwd_exact_chunks)
             : make_geom(pl.C, g_tune.bwd_chunk_vec * 4, g_tune.bwd_exact_chunks);
  if (lanes_per_row(p.g) > kMaxLaneVectors) return fail(NNUE_ERR_UNSUPPORTED, "backward: column chunk too wide");
  p.heavy_ticket_stride = p.g.n_vec;
  if (pl.B * (int64_t)p.g.n_vec > INT32_MAX)
    return fail(NNUE_ERR_UNSUPPORTED, "backward: grad_output exceeds 2^31 %s per perspective",
                v4 ? "16-byte vectors" : "floats");
  // Queued light rows address both perspectives' gradient rows by 32-bit
  // offsets from dout[0]: usable when dout[1] - dout[0] (in vectors) plus any
  // row offset stays inside int32.
  bool queue_ok = false, delta_ok = false;
  if (v4) {
    const int64_t delta =
        ((int64_t)reinterpret_cast<uintptr_t>(p.dout[1]) - (int64_t)reinterpret_cast<uintptr_t>(p.dout[0])) / 16;
    const int64_t span = pl.B * (int64_t)p.g.n_vec;
    // K / 4: the mean share of the K index slots that are active, measured on the
    // synthetic positions for both feature sets (41 of 160, 17 of 32)
    const int64_t expected_per_row = pl.B * pl.P * (int64_t)pl.K / (4 * std::max<int64_t>(pl.T, 1));
    if (delta >= INT32_MIN && delta + span <= (int64_t)INT32_MAX + 1) {
      p.persp_delta = (int32_t)delta;
      delta_ok = true;
      queue_ok = expected_per_row >= g_tune.bwd_queue_min_entries;
    }
  }

  const bool rows = row_end > row_begin;
  bool tail_done = false;
  DeviceAux* aux = nullptr;
  int rc = device_aux(&aux);
  if (rc != NNUE_OK) return rc;
  auto launch_heavy = [&](cudaStream_t hs) -> int {
    if (pl.P == 2 && pl.heavy_cap > 0 &&
        cudaMemsetAsync(w.hticket, 0, sizeof(uint32_t) * pl.heavy_cap * p.g.n_vec, hs) != cudaSuccess)
      return check_launch("backward_apply: heavy tickets");
    return v4 ? launch_segsum_heavy<float4>(p, hs) : launch_segsum_heavy<float>(p, hs);
  };
  // bwd_heavy_first 2: the heavy rows alone on the caller's stream first -- their warps then get the
  // issue slots the light rows' 64 warps per SM would otherwise share with them
  const bool heavy_alone = rows && g_tune.bwd_heavy_first == 2;
  if (heavy_alone && (rc = launch_heavy(s)) != NNUE_OK) return rc;
  {
    // fork: heavy rows and the bias column sum on the side stream
    std::lock_guard<std::mutex> lock(g_aux_mu);
    if (cudaEventRecord(aux->fork, s) != cudaSuccess || cudaStreamWaitEvent(aux->side, aux->fork, 0) != cudaSuccess)
      return check_launch("backward_apply: fork");
    // bwd_tail 2: the light rows' packed last chunk here, beside the main light-row kernel
    const bool tail_here = rows && v4 && g_tune.bwd_tail == 2;
    if (tail_here && g_tune.bwd_heavy_first != 1) tail_done = launch_segsum_tail(p, delta_ok, aux->side);
    if (rows && !heavy_alone && (rc = launch_heavy(aux->side)) != NNUE_OK) return rc;
    if (tail_here && g_tune.bwd_heavy_first == 1) tail_done = launch_segsum_tail(p, delta_ok, aux->side);
    if (with_bias) launch_colsum(g0, g1, pl, v4, w.partial, dB, p.accumulate, aux->side);
    if (cudaEventRecord(aux->join, aux->side) != cudaSuccess) return check_launch("backward_apply: join record");
  }
  if (rows && v4) {
    launch_segsum_light<float4>(p, queue_ok, delta_ok, tail_done, s);
  } else if (rows) {
    launch_segsum_light<float>(p, false, false, false, s);
  }
  // A later record of `join` by another call is further down the same
  // in-order side stream, so waiting on it also covers this call's work.
  if (cudaStreamWaitEvent(s, aux->join, 0) != cudaSuccess) return check_launch("backward_apply: join");
  return check_launch("backward_apply");
}

int check_bwd_args(const int32_t* idx0, const int32_t* idx1, int P, void* ws, size_t ws_bytes,
                   const BwdPlan& pl) {
  if (!idx0 || (P == 2 && !idx1)) return fail(NNUE_ERR_INVALID_ARGUMENT, "backward: null index pointer");
  if (!ws) return fail(NNUE_ERR_WORKSPACE, "backward: null workspace");
  if (ws_bytes < pl.total)
    return fail(NNUE_ERR_WORKSPACE, "backward: workspace %zu bytes < required %zu", ws_bytes, pl.total);
  if (reinterpret_cast<uintptr_t>(ws) & 255u) return fail(NNUE_ERR_WORKSPACE, "backward: workspace not 256-byte aligned");
  return NNUE_OK;
}

// ---------------------------------------------------------------------------
// Gather probe (measurement only): every warp sums `per_warp` random 512-byte
// rows of a table, 8 row loads in flight per warp -- the FT's access pattern
// with none of its bookkeeping.  Its bandwidth versus table size is the
// ceiling a gather kernel can reach from L2 / HBM on this GPU.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kBlock) gather_probe_kernel(const float4* __restrict__ table, int64_t rows,
                                                              const int32_t* __restrict__ idx, int32_t per_warp,
                                                              float4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int32_t* my = idx + wid * per_warp;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = 0; j0 + 32 <= per_warp; j0 += 32) {
    int r = __ldg(my + j0 + lane);
    r = (unsigned)r < (unsigned)rows ? r : 0;
    for (int u0 = 0; u0 < 32; u0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(table + (int64_t)__shfl_sync(kFull, r, u0 + u) * 32 + lane);
#pragma unroll
      for (int u = 0; u < 8; ++u) Vec<float4>::add(acc, v[u]);
    }
  }
  out[wid * 32 + lane] = acc;
}

// ---------------------------------------------------------------------------
// quantised forward
// ---------------------------------------------------------------------------
template <int VQ>
void launch_qforward_v(const QFwdParams& p, cudaStream_t s) {
  constexpr int U = VQ <= 4 ? 4 : 2;
  const int64_t n_items = (int64_t)p.P * p.B;
  const int64_t warps = ceil_div(n_items, p.items_per_warp);
  count_launch();
  ft_qforward_kernel<VQ, U><<<(unsigned)ceil_div(warps, kWarpsPerBlock), kBlock, 0, s>>>(p);
}

}  // namespace
}  // namespace nnue

// ---------------------------------------------------------------------------
// Scratch for nnue_ft_backward_noalloc: a fixed device array that exists on
// every GPU that loads this library, for as long as the process lives.  Host
// code must not pass the symbol itself to a kernel (on the host it is only a
// stand-in); its device address comes from cudaGetSymbolAddress with the
// device current, looked up on every call (a cheap lookup, and never stale:
// the first call on a device also loads the module there, which is why that
// first call belongs before any stream capture).
// ---------------------------------------------------------------------------
static constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace nnue {
namespace {
int noalloc_scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return fail(NNUE_ERR_CUDA, "backward_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  *out = p;
  return NNUE_OK;
}
}  // namespace
}  // namespace nnue

using namespace nnue;

extern "C" {

int nnue_ft_version(void) { return 100; }

uint64_t nnue_ft_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int nnue_ft_encode_features(const uint8_t* board, int64_t count, int32_t feature_set, int32_t* white,
                            int32_t* black, int32_t* white_count, int32_t* black_count, void* stream) {
  if (feature_set < 0 || feature_set > 2 || count < 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "encode_features: feature_set %d, count %lld", (int)feature_set,
                (long long)count);
  if (count == 0) return NNUE_OK;
  if (!board || !white || !black) return fail(NNUE_ERR_INVALID_ARGUMENT, "encode_features: null pointer");
  if (count > (int64_t)INT32_MAX * kEncPositions)
    return fail(NNUE_ERR_UNSUPPORTED, "encode_features: %lld positions", (long long)count);
  const nnue_feat::FeatureTables* tables = nullptr;
  int rc = encoder_tables(&tables);
  if (rc != NNUE_OK) return rc;
  EncParams p{};
  p.board = board;
  p.count = count;
  p.feature_set = feature_set;
  p.K = feature_set == 0 ? nnue_feat::kHalfkaMax
        : feature_set == 1 ? nnue_feat::kThreatMax
                           : nnue_feat::kThreatMax + nnue_feat::kHalfkaMax;
  p.board_vec16 = aligned16(board) ? 1 : 0;
  p.out[0] = white;
  p.out[1] = black;
  p.counts[0] = white_count;
  p.counts[1] = black_count;
  p.tables = tables;
  count_launch();
  const unsigned grid = (unsigned)ceil_div(count, kEncPositions);
  if (aligned16(white) && aligned16(black))  // rows are 16-byte multiples (K % 4 == 0)
    encode_features_kernel<true><<<grid, kEncThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  else
    encode_features_kernel<false><<<grid, kEncThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("encode_features");
}

int nnue_ft_kernel_timer_arm(uint32_t kernels, int32_t capacity) {
  if (kernels >= (1u << kTimedKinds) || capacity < 0 || (kernels && capacity == 0))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "kernel_timer_arm: bad kernel mask %u or capacity %d", kernels,
                (int)capacity);
  std::lock_guard<std::mutex> lock(g_timer.mu);
  g_timer.release();
  if (!kernels) return NNUE_OK;
  for (int32_t i = 0; i < capacity; ++i) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
      if (a) cudaEventDestroy(a);
      g_timer.release();
      return check_launch("kernel_timer_arm: event create");
    }
    g_timer.start.push_back(a);
    g_timer.stop.push_back(b);
  }
  g_timer.kind.reserve(capacity);
  g_timer.mask.store(kernels);
  return NNUE_OK;
}

int nnue_ft_kernel_timer_read(int32_t kernel, float* ms, int32_t max, int32_t* count) {
  if (kernel < 0 || kernel >= kTimedKinds || !count || max < 0 || (max > 0 && !ms))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "kernel_timer_read: bad arguments");
  std::lock_guard<std::mutex> lock(g_timer.mu);
  int32_t n = 0;
  for (size_t i = 0; i < g_timer.kind.size(); ++i) {
    if (g_timer.kind[i] != kernel) continue;
    if (n < max) {
      if (cudaEventSynchronize(g_timer.stop[i]) != cudaSuccess ||
          cudaEventElapsedTime(&ms[n], g_timer.start[i], g_timer.stop[i]) != cudaSuccess)
        return check_launch("kernel_timer_read");
    }
    ++n;
  }
  *count = n;
  return NNUE_OK;
}

const char* nnue_ft_last_error(void) { return g_last_error.c_str(); }

int nnue_ft_device_errors(uint32_t* flags, int clear) {
  if (!flags) return fail(NNUE_ERR_INVALID_ARGUMENT, "device_errors: null flags");
  if (cudaDeviceSynchronize() != cudaSuccess) return check_launch("device_errors: synchronize");
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_errors, sizeof(v)) != cudaSuccess) return check_launch("device_errors: read");
  if (clear) {
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_device_errors, &zero, sizeof(zero)) != cudaSuccess)
      return check_launch("device_errors: clear");
  }
  *flags = v;
  return NNUE_OK;
}

int nnue_ft_set_param(const char* name, int64_t value) {
  if (!name) return fail(NNUE_ERR_INVALID_ARGUMENT, "set_param: null name");
  for (ParamRef* p = params(); p->name; ++p) {
    if (std::strcmp(p->name, name) == 0) {
      if (value < p->lo || value > p->hi)
        return fail(NNUE_ERR_INVALID_ARGUMENT, "set_param: %s=%lld outside [%lld, %lld]", name, (long long)value,
                    (long long)p->lo, (long long)p->hi);
      *p->field = value;
      return NNUE_OK;
    }
  }
  return fail(NNUE_ERR_INVALID_ARGUMENT, "set_param: unknown parameter '%s'", name);
}

int64_t nnue_ft_get_param(const char* name) {
  if (!name) return -1;
  for (ParamRef* p = params(); p->name; ++p)
    if (std::strcmp(p->name, name) == 0) return *p->field;
  return -1;
}

int nnue_ft_forward(const int32_t* idx, int64_t batch, int32_t max_active, const float* weight, int64_t num_inputs,
                    int32_t output_size, const float* bias, float* output, void* stream) {
  return forward_impl(idx, nullptr, 1, batch, max_active, weight, num_inputs, output_size, bias, output, nullptr,
                      static_cast<cudaStream_t>(stream));
}

int nnue_ft_forward_pair(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                         const float* weight, int64_t num_inputs, int32_t output_size, const float* bias, float* out0,
                         float* out1, void* stream) {
  return forward_impl(idx0, idx1, 2, batch, max_active, weight, num_inputs, output_size, bias, out0, out1,
                      static_cast<cudaStream_t>(stream));
}

int nnue_ft_forward_pair_prepare(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                                 const float* weight, int64_t num_inputs, int32_t output_size, const float* bias,
                                 float* out0, float* out1, void* workspace, size_t workspace_bytes, void* stream) {
  BwdPlan pl;
  int rc = make_plan(batch, max_active, num_inputs, output_size, 2, pl);
  if (rc != NNUE_OK) return rc;
  rc = check_bwd_args(idx0, idx1, 2, workspace, workspace_bytes, pl);
  if (rc != NNUE_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceAux* aux = nullptr;
  rc = device_aux(&aux);
  if (rc != NNUE_OK) return rc;
  {
    // the backward's index-only phase (and the forward's packed tail chunk)
    // run on the side stream, concurrently with the forward gather on the
    // caller's stream
    std::lock_guard<std::mutex> lock(g_aux_mu);
    if (cudaEventRecord(aux->fork, s) != cudaSuccess || cudaStreamWaitEvent(aux->side, aux->fork, 0) != cudaSuccess)
      return check_launch("forward_pair_prepare: fork");
    rc = forward_impl(idx0, idx1, 2, batch, max_active, weight, num_inputs, output_size, bias, out0, out1, s, nullptr,
                      aux->side);
    if (rc != NNUE_OK) return rc;
    rc = prepare_impl(idx0, idx1, pl, carve(pl, workspace), aux->side);
    if (rc != NNUE_OK) return rc;
    if (cudaEventRecord(aux->join, aux->side) != cudaSuccess) return check_launch("forward_pair_prepare: join record");
  }
  if (cudaStreamWaitEvent(s, aux->join, 0) != cudaSuccess) return check_launch("forward_pair_prepare: join");
  return NNUE_OK;
}

int nnue_ft_forward_pair_tables(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                                const float* const* tables, const int64_t* table_rows, int32_t n_tables,
                                int32_t output_size, const float* bias, float* out0, float* out1, void* stream) {
  TableSet t;
  int64_t T = 0;
  int rc = make_tables("forward_pair_tables", const_cast<float* const*>(tables), table_rows, n_tables, t, T);
  if (rc != NNUE_OK) return rc;
  return forward_impl(idx0, idx1, 2, batch, max_active, nullptr, T, output_size, bias, out0, out1,
                      static_cast<cudaStream_t>(stream), &t);
}

int nnue_ft_forward_pair_tables_prepare(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                                        const float* const* tables, const int64_t* table_rows, int32_t n_tables,
                                        int32_t output_size, const float* bias, float* out0, float* out1,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  TableSet t;
  int64_t T = 0;
  int rc = make_tables("forward_pair_tables_prepare", const_cast<float* const*>(tables), table_rows, n_tables, t, T);
  if (rc != NNUE_OK) return rc;
  BwdPlan pl;
  rc = make_plan(batch, max_active, T, output_size, 2, pl);
  if (rc != NNUE_OK) return rc;
  rc = check_bwd_args(idx0, idx1, 2, workspace, workspace_bytes, pl);
  if (rc != NNUE_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  DeviceAux* aux = nullptr;
  rc = device_aux(&aux);
  if (rc != NNUE_OK) return rc;
  {
    std::lock_guard<std::mutex> lock(g_aux_mu);
    if (cudaEventRecord(aux->fork, s) != cudaSuccess || cudaStreamWaitEvent(aux->side, aux->fork, 0) != cudaSuccess)
      return check_launch("forward_pair_tables_prepare: fork");
    rc = prepare_impl(idx0, idx1, pl, carve(pl, workspace), aux->side);
    if (rc != NNUE_OK) return rc;
    if (cudaEventRecord(aux->join, aux->side) != cudaSuccess)
      return check_launch("forward_pair_tables_prepare: join record");
  }
  rc = forward_impl(idx0, idx1, 2, batch, max_active, nullptr, T, output_size, bias, out0, out1, s, &t);
  if (rc != NNUE_OK) return rc;
  if (cudaStreamWaitEvent(s, aux->join, 0) != cudaSuccess) return check_launch("forward_pair_tables_prepare: join");
  return NNUE_OK;
}

int nnue_ft_backward_apply_tables(const float* grad0, const float* grad1, int64_t batch, int32_t max_active,
                                  float* const* weight_grads, const int64_t* table_rows, int32_t n_tables,
                                  int32_t output_size, float* bias_grad, int32_t accumulate, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  TableSet t;
  int64_t T = 0;
  int rc = make_tables("backward_apply_tables", weight_grads, table_rows, n_tables, t, T);
  if (rc != NNUE_OK) return rc;
  BwdPlan pl;
  rc = make_plan(batch, max_active, T, output_size, 2, pl);
  if (rc != NNUE_OK) return rc;
  if (!bias_grad || (batch > 0 && (!grad0 || !grad1)))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "backward_apply_tables: null pointer");
  if (!workspace || workspace_bytes < pl.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(NNUE_ERR_WORKSPACE, "backward_apply_tables: workspace missing, misaligned or smaller than %zu bytes",
                pl.total);
  return apply_impl(grad0, grad1, pl, carve(pl, workspace), t.base[0], bias_grad, accumulate, 0, pl.T, true,
                    static_cast<cudaStream_t>(stream), &t);
}

int nnue_ft_merge_virtual(const float* weight, int64_t rows, const float* virtual_weight, int64_t period,
                          int32_t cols, float* out, void* stream) {
  if (rows < 0 || cols < 0 || period <= 0 || rows % period != 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "merge_virtual: need rows a multiple of period > 0");
  if (rows == 0 || cols == 0) return NNUE_OK;
  if (!weight || !virtual_weight || !out) return fail(NNUE_ERR_INVALID_ARGUMENT, "merge_virtual: null pointer");
  const bool v4 = cols % 4 == 0 && aligned16(weight) && aligned16(virtual_weight) && aligned16(out);
  const int64_t row_vec = v4 ? cols / 4 : cols;
  const int64_t n = rows * row_vec;
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  count_launch();
  if (v4)
    merge_virtual_kernel<float4><<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(weight),
                                                      reinterpret_cast<const float4*>(virtual_weight), n, row_vec,
                                                      period, reinterpret_cast<float4*>(out));
  else
    merge_virtual_kernel<float><<<grid, 256, 0, s>>>(weight, virtual_weight, n, row_vec, period, out);
  return check_launch("merge_virtual");
}

size_t nnue_ft_backward_workspace_size(int64_t batch, int32_t max_active, int64_t num_inputs, int32_t output_size,
                                       int32_t n_persp) {
  BwdPlan pl;
  if (make_plan(batch, max_active, num_inputs, output_size, n_persp, pl) != NNUE_OK) return 0;
  return pl.total;
}

int nnue_ft_backward_prepare(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                             int32_t n_persp, int64_t num_inputs, int32_t output_size, void* workspace,
                             size_t workspace_bytes, void* stream) {
  BwdPlan pl;
  int rc = make_plan(batch, max_active, num_inputs, output_size, n_persp, pl);
  if (rc != NNUE_OK) return rc;
  rc = check_bwd_args(idx0, idx1, n_persp, workspace, workspace_bytes, pl);
  if (rc != NNUE_OK) return rc;
  return prepare_impl(idx0, idx1, pl, carve(pl, workspace), static_cast<cudaStream_t>(stream));
}

int nnue_ft_backward_apply(const float* grad0, const float* grad1, int64_t batch, int32_t max_active, int32_t n_persp,
                           int64_t num_inputs, int32_t output_size, float* weight_grad, float* bias_grad,
                           int32_t accumulate, void* workspace, size_t workspace_bytes, void* stream) {
  BwdPlan pl;
  int rc = make_plan(batch, max_active, num_inputs, output_size, n_persp, pl);
  if (rc != NNUE_OK) return rc;
  if (!weight_grad || !bias_grad || (batch > 0 && (!grad0 || (n_persp == 2 && !grad1))))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "backward_apply: null pointer");
  if (!workspace || workspace_bytes < pl.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(NNUE_ERR_WORKSPACE, "backward_apply: workspace missing, misaligned or smaller than %zu bytes",
                pl.total);
  return apply_impl(grad0, grad1, pl, carve(pl, workspace), weight_grad, bias_grad, accumulate, 0, pl.T, true,
                    static_cast<cudaStream_t>(stream));
}

int nnue_ft_backward_apply_rows(const float* grad0, const float* grad1, int64_t batch, int32_t max_active,
                                int32_t n_persp, int64_t num_inputs, int32_t output_size, float* weight_grad,
                                float* bias_grad, int32_t accumulate, int64_t row_begin, int64_t row_end,
                                int32_t with_bias, void* workspace, size_t workspace_bytes, void* stream) {
  BwdPlan pl;
  int rc = make_plan(batch, max_active, num_inputs, output_size, n_persp, pl);
  if (rc != NNUE_OK) return rc;
  if (!weight_grad || (with_bias && !bias_grad) || (batch > 0 && (!grad0 || (n_persp == 2 && !grad1))))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "backward_apply_rows: null pointer");
  if (!workspace || workspace_bytes < pl.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(NNUE_ERR_WORKSPACE, "backward_apply_rows: workspace missing, misaligned or smaller than %zu bytes",
                pl.total);
  return apply_impl(grad0, grad1, pl, carve(pl, workspace), weight_grad, bias_grad, accumulate, row_begin, row_end,
                    with_bias != 0, static_cast<cudaStream_t>(stream));
}

int nnue_ft_backward(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active, const float* grad0,
                     const float* grad1, int32_t n_persp, int64_t num_inputs, int32_t output_size, float* weight_grad,
                     float* bias_grad, int32_t accumulate, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = nnue_ft_backward_prepare(idx0, idx1, batch, max_active, n_persp, num_inputs, output_size, workspace,
                                    workspace_bytes, stream);
  if (rc != NNUE_OK) return rc;
  return nnue_ft_backward_apply(grad0, grad1, batch, max_active, n_persp, num_inputs, output_size, weight_grad,
                                bias_grad, accumulate, workspace, workspace_bytes, stream);
}

int nnue_ft_quantized_forward_pair(const int32_t* idx0, const int32_t* idx1, int32_t n_persp, int64_t batch,
                                   int32_t max_active, const int16_t* weight_q, const int32_t* psqt_q,
                                   int64_t table_rows, int32_t l1, int32_t n_psqt, const int16_t* bias_q,
                                   int32_t map_training, int16_t* acc0, int16_t* acc1, int32_t* psqt0, int32_t* psqt1,
                                   void* stream) {
  if (n_persp != 1 && n_persp != 2) return fail(NNUE_ERR_INVALID_ARGUMENT, "quantized_forward: n_persp must be 1 or 2");
  if (batch < 0 || max_active < 0 || table_rows <= 0 || table_rows > INT32_MAX || l1 <= 0 || n_psqt < 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "quantized_forward: bad sizes");
  if (l1 % 8 != 0 || n_psqt % 4 != 0 || n_psqt > 128 || l1 > 8 * 32 * 8)
    return fail(NNUE_ERR_UNSUPPORTED, "quantized_forward: need l1 %% 8 == 0 (<= 2048) and n_psqt %% 4 == 0 (<= 128)");
  if (batch == 0) return NNUE_OK;
  if (!idx0 || !weight_q || !psqt_q || !bias_q || !acc0 || !psqt0 ||
      (n_persp == 2 && (!idx1 || !acc1 || !psqt1)))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "quantized_forward: null pointer");
  const void* ptrs[] = {weight_q, psqt_q, bias_q, acc0, psqt0, n_persp == 2 ? acc1 : acc0,
                        n_persp == 2 ? psqt1 : psqt0};
  for (const void* q : ptrs)
    if (!aligned16(q)) return fail(NNUE_ERR_INVALID_ARGUMENT, "quantized_forward: pointers must be 16-byte aligned");
  QFwdParams p{};
  p.idx[0] = idx0;
  p.idx[1] = n_persp == 2 ? idx1 : idx0;
  p.acc[0] = acc0;
  p.acc[1] = n_persp == 2 ? acc1 : acc0;
  p.psqt[0] = psqt0;
  p.psqt[1] = n_persp == 2 ? psqt1 : psqt0;
  p.Wq = weight_q;
  p.Pq = psqt_q;
  p.bias = bias_q;
  p.B = batch;
  p.K = max_active;
  p.Tq = (int32_t)table_rows;
  p.n8 = l1 / 8;
  p.np4 = n_psqt / 4;
  p.P = n_persp;
  p.map_training = map_training ? 1 : 0;
  p.items_per_warp = (int32_t)g_tune.fwd_items_per_warp;
  if (p.np4 > 32) return fail(NNUE_ERR_UNSUPPORTED, "quantized_forward: n_psqt > 128");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch ((p.n8 + 31) / 32) {
    case 1: launch_qforward_v<1>(p, s); break;
    case 2: launch_qforward_v<2>(p, s); break;
    case 3: launch_qforward_v<3>(p, s); break;
    case 4: launch_qforward_v<4>(p, s); break;
    case 5: launch_qforward_v<5>(p, s); break;
    case 6: launch_qforward_v<6>(p, s); break;
    default: launch_qforward_v<8>(p, s); break;
  }
  return check_launch("quantized_forward");
}

int nnue_ft_halfka_export_quantize(const float* weight, const float* virtual_weight, int32_t l1, int32_t n_psqt,
                                   float w_scale, float psqt_scale, int16_t* weight_q, int32_t* psqt_q, void* stream) {
  if (!weight || !weight_q || (n_psqt > 0 && !psqt_q) || l1 <= 0 || n_psqt < 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "halfka_export_quantize: bad arguments");
  // inverse king buckets (halfka_v2_hm.py:9-25): bucket -> oriented king square
  static const int kKingBuckets[64] = {
      -1, -1, -1, -1, 31, 30, 29, 28, -1, -1, -1, -1, 27, 26, 25, 24, -1, -1, -1, -1, 23, 22,
      21, 20, -1, -1, -1, -1, 19, 18, 17, 16, -1, -1, -1, -1, 15, 14, 13, 12, -1, -1, -1, -1,
      11, 10, 9,  8,  -1, -1, -1, -1, 7,  6,  5,  4,  -1, -1, -1, -1, 3,  2,  1,  0};
  KingSquares inv{};
  for (int sq = 0; sq < 64; ++sq)
    if (kKingBuckets[sq] >= 0) inv.sq[kKingBuckets[sq]] = sq;
  count_launch();
  halfka_export_quantize_kernel<<<22528, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      weight, virtual_weight, l1 + n_psqt, l1, w_scale, psqt_scale, inv, weight_q, psqt_q);
  return check_launch("halfka_export_quantize");
}

int nnue_ft_quantize_i16(const float* x, int64_t n, float scale, int16_t* q, void* stream) {
  if (n < 0 || (n > 0 && (!x || !q))) return fail(NNUE_ERR_INVALID_ARGUMENT, "quantize_i16: bad arguments");
  if (n == 0) return NNUE_OK;
  count_launch();
  quantize_i16_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, scale, q);
  return check_launch("quantize_i16");
}

namespace {
int epilogue_launch(bool backward, const float* wp, const float* bp, int64_t batch, int32_t l1, int32_t n_psqt,
                    const float* us, const int64_t* pidx, float* l0, float* psqt, const float* g_l0,
                    const float* g_psqt, float* g_wp, float* g_bp, void* stream) {
  const char* what = backward ? "epilogue_backward" : "epilogue_forward";
  if (batch < 0 || l1 <= 0 || l1 % 2 != 0 || n_psqt < 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "%s: need batch >= 0, even l1 > 0, n_psqt >= 0", what);
  if (batch == 0) return NNUE_OK;
  if (!wp || !bp || !us || !pidx || (!backward && (!l0 || !psqt)) || (backward && (!g_wp || !g_bp)))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  EpiParams a{};
  a.wp = wp;
  a.bp = bp;
  a.us = us;
  a.pidx = pidx;
  a.l0 = l0;
  a.psqt = psqt;
  a.d_l0 = g_l0;
  a.d_psqt = g_psqt;
  a.d_wp = g_wp;
  a.d_bp = g_bp;
  a.B = batch;
  a.l1 = l1;
  a.n_psqt = n_psqt;
  const bool v4 = l1 % 8 == 0 && (l1 + n_psqt) % 4 == 0 && aligned16(wp) && aligned16(bp) &&
                  (backward ? (aligned16(g_wp) && aligned16(g_bp) && (!g_l0 || aligned16(g_l0))) : aligned16(l0));
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(batch, 8), 148 * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  count_launch();
  if (backward) {
    if (v4) ft_epilogue_backward_kernel<float4><<<grid, 256, 0, s>>>(a);
    else ft_epilogue_backward_kernel<float><<<grid, 256, 0, s>>>(a);
  } else {
    if (v4) ft_epilogue_forward_kernel<float4><<<grid, 256, 0, s>>>(a);
    else ft_epilogue_forward_kernel<float><<<grid, 256, 0, s>>>(a);
  }
  return check_launch(what);
}
}  // namespace

int nnue_ft_epilogue_forward(const float* wp, const float* bp, int64_t batch, int32_t l1, int32_t n_psqt,
                             const float* us, const int64_t* psqt_indices, float* l0, float* psqt, void* stream) {
  return epilogue_launch(false, wp, bp, batch, l1, n_psqt, us, psqt_indices, l0, psqt, nullptr, nullptr, nullptr,
                         nullptr, stream);
}

int nnue_ft_epilogue_backward(const float* wp, const float* bp, int64_t batch, int32_t l1, int32_t n_psqt,
                              const float* us, const int64_t* psqt_indices, const float* grad_l0,
                              const float* grad_psqt, float* grad_wp, float* grad_bp, void* stream) {
  return epilogue_launch(true, wp, bp, batch, l1, n_psqt, us, psqt_indices, nullptr, nullptr, grad_l0, grad_psqt,
                         grad_wp, grad_bp, stream);
}

int nnue_ft_ranger22_step(float* param, const float* grad, float* variance_ma, float* gma_cur, const float* gma_prev,
                          float* lookahead, int64_t rows, int64_t cols, const float* scalars, int32_t lookahead_merge,
                          float lookahead_alpha, void* stream) {
  if (rows < 0 || cols < 0) return fail(NNUE_ERR_INVALID_ARGUMENT, "ranger22_step: negative sizes");
  if (rows == 0 || cols == 0) return NNUE_OK;
  if (!param || !grad || !variance_ma || !gma_cur || !gma_prev || !scalars || (lookahead_merge && !lookahead))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "ranger22_step: null pointer");
  R22Params a{};
  a.p = param;
  a.g = grad;
  a.v = variance_ma;
  a.m = gma_cur;
  a.mp = gma_prev;
  a.la = lookahead_merge ? lookahead : param;
  a.rows = rows;
  a.cols = cols;
  a.lr = scalars[0];
  a.inv_sqrt_bc2 = scalars[1];
  a.eps = scalars[2];
  a.two_nl = scalars[3];
  a.noise_recip = scalars[4];
  a.pnm_a = scalars[5];
  a.pnm_b = scalars[6];
  a.step_size = scalars[7];
  a.beta2 = scalars[8];
  a.omb2 = scalars[9];
  a.b1sq = scalars[10];
  a.omb1sq = scalars[11];
  a.merge = lookahead_merge ? 1 : 0;
  a.w = 1.0f - lookahead_alpha;
  const bool v4 = cols % 4 == 0 && aligned16(param) && aligned16(grad) && aligned16(variance_ma) &&
                  aligned16(gma_cur) && aligned16(gma_prev) && (!lookahead_merge || aligned16(lookahead));
  const int64_t nvec = v4 ? cols / 4 : cols;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  count_launch();
  if (nvec <= 32 * 64) {  // one warp per row, 8 rows per block
    const unsigned grid = (unsigned)ceil_div(rows, 8);
    if (v4) ranger22_rows_kernel<float4, 32><<<grid, 256, 0, s>>>(a);
    else ranger22_rows_kernel<float, 32><<<grid, 256, 0, s>>>(a);
  } else {  // one block per row
    if (rows > INT32_MAX) return fail(NNUE_ERR_UNSUPPORTED, "ranger22_step: too many long rows");
    if (v4) ranger22_rows_kernel<float4, 512><<<(unsigned)rows, 512, 0, s>>>(a);
    else ranger22_rows_kernel<float, 512><<<(unsigned)rows, 512, 0, s>>>(a);
  }
  return check_launch("ranger22_step");
}

size_t nnue_ft_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int nnue_ft_backward_noalloc(const int32_t* idx0, const int32_t* idx1, int64_t batch, int32_t max_active,
                             const float* grad0, const float* grad1, int32_t n_persp, int64_t num_inputs,
                             int32_t output_size, float* weight_grad, float* bias_grad, int32_t accumulate,
                             void* stream) {
  BwdPlan pl;
  int rc = make_plan(batch, max_active, num_inputs, output_size, n_persp, pl);
  if (rc != NNUE_OK) return rc;
  if (pl.total > kNoAllocScratchBytes)
    return fail(NNUE_ERR_UNSUPPORTED,
                "backward_noalloc: these sizes need %zu bytes of scratch but the library's fixed scratch holds %zu; "
                "use nnue_ft_backward with a caller workspace",
                pl.total, kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = noalloc_scratch_address(&scratch);
  if (rc != NNUE_OK) return rc;
  return nnue_ft_backward(idx0, idx1, batch, max_active, grad0, grad1, n_persp, num_inputs, output_size, weight_grad,
                          bias_grad, accumulate, scratch, kNoAllocScratchBytes, stream);
}

// ---- exchange between the GPUs of one node --------------------------------
int nnue_ft_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return check_launch("exchange_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return check_launch("exchange_alloc: zeroing / IPC handle");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == NNUE_FT_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return NNUE_OK;
}

int nnue_ft_exchange_free(void* ptr) {
  if (!ptr) return NNUE_OK;
  if (cudaFree(ptr) != cudaSuccess) return check_launch("exchange_free");
  return NNUE_OK;
}

int nnue_ft_exchange_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return check_launch("exchange_open: cudaIpcOpenMemHandle");
  return NNUE_OK;
}

int nnue_ft_exchange_close(void* ptr) {
  if (!ptr) return NNUE_OK;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) return check_launch("exchange_close");
  return NNUE_OK;
}

int nnue_ft_exchange(const nnue_ft_copy_desc* copies, int32_t n_copies, uint32_t* const* flags, int32_t n_ranks,
                     int32_t rank, int32_t channel, uint32_t epoch, int32_t timeout_ms, void* stream) {
  if (n_copies < 0 || n_copies > kMaxCopies || (n_copies && !copies))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: 0..%d copies", kMaxCopies);
  if (!flags || n_ranks < 1 || n_ranks > kMaxRanks - 1 || rank < 0 || rank >= n_ranks || timeout_ms <= 0)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: bad group (1..%d ranks)", kMaxRanks - 1);
  if (channel < 0 || channel >= kChannels)
    return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: channel %d outside [0, %d)", (int)channel, kChannels);
  static_assert(kChannels * kMaxRanks * sizeof(uint32_t) <= NNUE_FT_EXCHANGE_FLAG_BYTES, "flag words");
  ExchangeParams p{};
  p.n_copies = n_copies;
  p.n_ranks = n_ranks;
  p.rank = rank;
  p.epoch = epoch;
  p.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  for (int r = 0; r < n_ranks; ++r) {
    if (!flags[r] || reinterpret_cast<uintptr_t>(flags[r]) % 4 != 0)
      return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: flag words of rank %d null or misaligned", r);
    p.flags[r] = flags[r] + channel * kMaxRanks;
  }
  int64_t rows = 0;
  for (int i = 0; i < n_copies; ++i) {
    const nnue_ft_copy_desc& c = copies[i];
    if (c.rows < 0 || c.width < 0 || c.src_ld < c.width || c.dst_ld < c.width)
      return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: copy %d has bad sizes", i);
    if (c.rows > 0 && c.width > 0 && (!aligned16(c.src) || !aligned16(c.dst)))
      return fail(NNUE_ERR_INVALID_ARGUMENT, "exchange: copy %d: null or not 16-byte aligned", i);
    p.c[i].src = static_cast<const float4*>(c.src);
    p.c[i].dst = static_cast<float4*>(c.dst);
    p.c[i].rows = c.width > 0 ? c.rows : 0;
    p.c[i].src_ld = c.src_ld;
    p.c[i].dst_ld = c.dst_ld;
    p.c[i].width = c.width;
    p.c[i].scale = c.scale;
    p.row_start[i] = rows;
    rows += p.c[i].rows;
  }
  p.row_start[n_copies] = rows;
  if (n_copies == 0) {  // a barrier only: one copy-less launch
    p.c[0] = CopyDesc{};
  }
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int R = g_tune.xchg_rows >= 4 ? 4 : g_tune.xchg_rows >= 2 ? 2 : 1;
  const int64_t warps_wanted = std::max<int64_t>(1, ceil_div(rows, R));
  const unsigned grid = (unsigned)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)sms * g_tune.xchg_blocks_per_sm, ceil_div(warps_wanted, 8)));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  count_launch();
  if (R == 4) exchange_kernel<4><<<grid, 256, 0, st>>>(p);
  else if (R == 2) exchange_kernel<2><<<grid, 256, 0, st>>>(p);
  else exchange_kernel<1><<<grid, 256, 0, st>>>(p);
  return check_launch("exchange");
}

int nnue_ft_gather_probe(const float* table, int64_t rows, const int32_t* idx, int32_t per_warp, int32_t n_warps,
                         float* out, void* stream) {
  if (!table || !idx || !out || rows <= 0 || per_warp < 32 || per_warp % 32 != 0 || n_warps <= 0 ||
      n_warps % kWarpsPerBlock != 0 || !aligned16(table) || !aligned16(out))
    return fail(NNUE_ERR_INVALID_ARGUMENT, "gather_probe: bad arguments");
  count_launch();
  gather_probe_kernel<<<(unsigned)(n_warps / kWarpsPerBlock), kBlock, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(table), rows, idx, per_warp, reinterpret_cast<float4*>(out));
  return check_launch("gather_probe");
}

}  // extern "C"
