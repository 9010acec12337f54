// Host-side synthetic positions and feature-index encoding.
//
// The encoder restates the reference's feature functions
// (src/rust/feature_extraction.rs): HalfKAv2_hm (:391-404, :677-685, :745-752),
// Full_Threats (:581-675, :687-739, :754-832) and their composition with
// component offsets and a -1 tail (:213-241, :457-460).  Standard chess attack
// sets (the reference takes them from the sfbinpack crate) are built here from
// the rules of chess.  Board: 64 piece ids (type * 2 + colour, 12 = empty).
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/nnue_ft.h"
#include "feature_encode.h"

namespace nnue_feat {

namespace {

uint64_t step_attacks(int sq, const int (*steps)[2], int n) {
  uint64_t bb = 0;
  const int f0 = sq & 7, r0 = sq >> 3;
  for (int i = 0; i < n; ++i) {
    const int f = f0 + steps[i][0], r = r0 + steps[i][1];
    if (f >= 0 && f < 8 && r >= 0 && r < 8) bb |= 1ull << (r * 8 + f);
  }
  return bb;
}

// Squares beyond sq in direction (df, dr), up to the edge.
uint64_t ray(int sq, int df, int dr) {
  uint64_t bb = 0;
  int f = (sq & 7) + df, r = (sq >> 3) + dr;
  while (f >= 0 && f < 8 && r >= 0 && r < 8) {
    bb |= 1ull << (r * 8 + f);
    f += df;
    r += dr;
  }
  return bb;
}

void build(FeatureTables& t) {
  const int kn[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};
  const int kg[8][2] = {{1, 0}, {1, 1}, {0, 1}, {-1, 1}, {-1, 0}, {-1, -1}, {0, -1}, {1, -1}};
  const int pw[2][2] = {{-1, 1}, {1, 1}};
  const int pb[2][2] = {{-1, -1}, {1, -1}};
  // (file step, rank step) of the ray directions kRayE .. kRaySE
  const int dirs[8][2] = {{1, 0}, {0, 1}, {1, 1}, {-1, 1}, {-1, 0}, {0, -1}, {-1, -1}, {1, -1}};
  for (int sq = 0; sq < 64; ++sq) {
    t.knight[sq] = step_attacks(sq, kn, 8);
    t.king[sq] = step_attacks(sq, kg, 8);
    t.pawn[kWhite][sq] = step_attacks(sq, pw, 2);
    t.pawn[kBlack][sq] = step_attacks(sq, pb, 2);
    for (int d = 0; d < 8; ++d) t.ray[d][sq] = ray(sq, dirs[d][0], dirs[d][1]);
  }
  for (int sq = 0; sq < 64; ++sq) {
    t.empty_attacks[kPawn][sq] = 0;
    for (int pt = kKnight; pt <= kKing; ++pt) t.empty_attacks[pt][sq] = piece_attacks(t, pt, sq, 0);
  }
  const int buckets[64] = {-1, -1, -1, -1, 31, 30, 29, 28, -1, -1, -1, -1, 27, 26, 25, 24,
                           -1, -1, -1, -1, 23, 22, 21, 20, -1, -1, -1, -1, 19, 18, 17, 16,
                           -1, -1, -1, -1, 15, 14, 13, 12, -1, -1, -1, -1, 11, 10, 9,  8,
                           -1, -1, -1, -1, 7,  6,  5,  4,  -1, -1, -1, -1, 3,  2,  1,  0};
  const int valid_targets[12] = {6, 6, 10, 10, 8, 8, 8, 8, 10, 10, 0, 0};
  const int threat_map[6][6] = {{0, 1, -1, 2, -1, -1}, {0, 1, 2, 3, 4, -1}, {0, 1, 2, 3, -1, -1},
                                {0, 1, 2, 3, -1, -1},  {0, 1, 2, 3, 4, -1}, {-1, -1, -1, -1, -1, -1}};
  for (int i = 0; i < 64; ++i) t.king_bucket[i] = buckets[i];
  for (int i = 0; i < 12; ++i) t.num_valid_targets[i] = valid_targets[i];
  for (int a = 0; a < 6; ++a)
    for (int b = 0; b < 6; ++b) t.threat_map[a][b] = threat_map[a][b];
  // threat_feature_calc (feature_extraction.rs:788-832): colour-major piece order
  int piece_offset = 0;
  for (int color = 0; color < 2; ++color) {
    for (int pt = 0; pt < 6; ++pt) {
      const int pi = 2 * pt + color;
      t.threat[pi][65] = piece_offset;
      int square_offset = 0;
      for (int from = 0; from < 64; ++from) {
        t.threat[pi][from] = square_offset;
        if (pt != kPawn) {
          square_offset += popcount64(t.empty_attacks[pt][from]);
        } else if (from >= 8 && from <= 55) {
          const int push = color == kWhite ? from + 8 : from - 8;
          square_offset += popcount64(t.pawn[color][from] | (1ull << push));
        }
      }
      t.threat[pi][64] = square_offset;
      piece_offset += valid_targets[pi] * square_offset;
    }
  }
  t.threat_total = piece_offset;
  t.pad[0] = t.pad[1] = t.pad[2] = 0;
}

}  // namespace

const FeatureTables& feature_tables() {
  static FeatureTables t;
  static std::once_flag once;
  std::call_once(once, [] { build(t); });
  return t;
}

}  // namespace nnue_feat

namespace {

using namespace nnue_feat;

struct Pos {
  uint64_t by_piece[12];
  uint64_t occ;
  const uint8_t* board;
  PosView view() const { return PosView{by_piece, occ, board}; }
};

void load(const uint8_t* board, Pos& p) {
  std::fill(p.by_piece, p.by_piece + 12, 0ull);
  p.occ = 0;
  p.board = board;
  for (int sq = 0; sq < 64; ++sq) {
    const int id = board[sq];
    if (id < 12) {
      p.by_piece[id] |= 1ull << sq;
      p.occ |= 1ull << sq;
    }
  }
}

// splitmix64 (Steele, Lea & Flood 2014) and a multiply-shift range reduction.
inline uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline uint32_t uniform(uint64_t& s, uint32_t n) { return (uint32_t)(((splitmix64(s) >> 32) * n) >> 32); }

void draw_position(uint64_t& s, uint8_t* board, uint8_t* stm) {
  std::fill(board, board + 64, (uint8_t)kEmpty);
  const int wk = (int)uniform(s, 64);
  int bk = (int)uniform(s, 63);
  if (bk >= wk) ++bk;
  board[wk] = kKing * 2 + kWhite;
  board[bk] = kKing * 2 + kBlack;
  const int n = (int)uniform(s, 31);
  for (int i = 0; i < n; ++i) {
    const int pt = (int)uniform(s, 5);
    const int color = (int)uniform(s, 2);
    int sq;
    do {
      sq = pt == kPawn ? 8 + (int)uniform(s, 48) : (int)uniform(s, 64);
    } while (board[sq] != kEmpty);
    board[sq] = (uint8_t)(pt * 2 + color);
  }
  *stm = (uint8_t)uniform(s, 2);
}

template <typename F>
void parallel_for(int64_t n, int nthreads, F&& fn) {
  if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
  nthreads = (int)std::min<int64_t>(nthreads, std::max<int64_t>(1, n / 256));
  if (nthreads <= 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < nthreads; ++t) {
    const int64_t a = n * t / nthreads, b = n * (t + 1) / nthreads;
    th.emplace_back([&fn, a, b] { fn(a, b); });
  }
  for (auto& x : th) x.join();
}

}  // namespace

extern "C" {

int nnue_generate_positions(uint64_t seed, int64_t first, int64_t count, uint8_t* board, uint8_t* stm) {
  if (count < 0 || (count > 0 && (!board || !stm))) return NNUE_ERR_INVALID_ARGUMENT;
  feature_tables();
  parallel_for(count, 0, [&](int64_t a, int64_t b) {
    int32_t scratch[kThreatMax];
    for (int64_t i = a; i < b; ++i) {
      uint64_t s = seed * 0xD1B54A32D192ED03ull + (uint64_t)(first + i) * 0x9E3779B97F4A7C15ull;
      uint8_t* bd = board + i * 64;
      for (;;) {
        draw_position(s, bd, stm + i);
        Pos p;
        load(bd, p);
        const FeatureTables& t = feature_tables();
        RowSink sw{scratch, 0}, sb{scratch, 0};
        if (encode_threats(t, p.view(), kWhite, sw, kThreatMax) >= 0 &&
            encode_threats(t, p.view(), kBlack, sb, kThreatMax) >= 0)
          break;
      }
    }
  });
  return NNUE_OK;
}

int nnue_encode_features(const uint8_t* board, int64_t count, int32_t feature_set, int32_t* white, int32_t* black,
                         int32_t* white_count, int32_t* black_count, int32_t nthreads) {
  if (feature_set < 0 || feature_set > 2 || count < 0 || (count > 0 && (!board || !white || !black)))
    return NNUE_ERR_INVALID_ARGUMENT;
  const int K = feature_set == 0 ? kHalfkaMax : feature_set == 1 ? kThreatMax : kThreatMax + kHalfkaMax;
  feature_tables();
  std::vector<int> status(std::max<int64_t>(count, 1), 0);
  parallel_for(count, nthreads, [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) {
      Pos p;
      load(board + i * 64, p);
      int32_t* rows[2] = {white + i * K, black + i * K};
      int32_t* counts[2] = {white_count, black_count};
      for (int c = 0; c < 2; ++c) {
        RowSink sink{rows[c], 0};
        const int n = encode_position(feature_tables(), p.view(), c, feature_set, sink);
        if (n < 0) {
          status[i] = n;
          std::fill(rows[c], rows[c] + K, -1);
          if (counts[c]) counts[c][i] = 0;
          continue;
        }
        std::fill(rows[c] + n, rows[c] + K, -1);
        if (counts[c]) counts[c][i] = n;
      }
    }
  });
  for (int64_t i = 0; i < count; ++i)
    if (status[i] != 0) return NNUE_ERR_INVALID_ARGUMENT;
  return NNUE_OK;
}

int nnue_threat_table_total(void) { return feature_tables().threat_total; }

}  // extern "C"
