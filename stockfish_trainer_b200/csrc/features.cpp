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

namespace {

constexpr int kEmpty = 12;
constexpr int kPawn = 0, kKnight = 1, kBishop = 2, kRook = 3, kQueen = 4, kKing = 5;
constexpr int kWhite = 0, kBlack = 1;
constexpr uint64_t kAFile = 0x0101010101010101ull, kHFile = 0x8080808080808080ull;
constexpr int kHalfkaInputs = 24576, kHalfkaMax = 32;
constexpr int kThreatInputs = 60720, kThreatMax = 128;

const int kKingBuckets[64] = {-1, -1, -1, -1, 31, 30, 29, 28, -1, -1, -1, -1, 27, 26, 25, 24,
                              -1, -1, -1, -1, 23, 22, 21, 20, -1, -1, -1, -1, 19, 18, 17, 16,
                              -1, -1, -1, -1, 15, 14, 13, 12, -1, -1, -1, -1, 11, 10, 9,  8,
                              -1, -1, -1, -1, 7,  6,  5,  4,  -1, -1, -1, -1, 3,  2,  1,  0};
const int kNumValidTargets[12] = {6, 6, 10, 10, 8, 8, 8, 8, 10, 10, 0, 0};
const int kThreatMap[6][6] = {{0, 1, -1, 2, -1, -1}, {0, 1, 2, 3, 4, -1}, {0, 1, 2, 3, -1, -1},
                              {0, 1, 2, 3, -1, -1},  {0, 1, 2, 3, 4, -1}, {-1, -1, -1, -1, -1, -1}};

struct Tables {
  uint64_t knight[64], king[64], pawn[2][64];
  int threat[12][66];
  int threat_total;
};

inline int popcount(uint64_t x) { return __builtin_popcountll(x); }
inline int lsb(uint64_t x) { return __builtin_ctzll(x); }

uint64_t step_attacks(int sq, const int (*steps)[2], int n) {
  uint64_t bb = 0;
  const int f0 = sq & 7, r0 = sq >> 3;
  for (int i = 0; i < n; ++i) {
    const int f = f0 + steps[i][0], r = r0 + steps[i][1];
    if (f >= 0 && f < 8 && r >= 0 && r < 8) bb |= 1ull << (r * 8 + f);
  }
  return bb;
}

uint64_t slide(int sq, uint64_t occ, const int (*dirs)[2], int n) {
  uint64_t bb = 0;
  const int f0 = sq & 7, r0 = sq >> 3;
  for (int i = 0; i < n; ++i) {
    int f = f0 + dirs[i][0], r = r0 + dirs[i][1];
    while (f >= 0 && f < 8 && r >= 0 && r < 8) {
      const int s = r * 8 + f;
      bb |= 1ull << s;
      if (occ >> s & 1) break;
      f += dirs[i][0];
      r += dirs[i][1];
    }
  }
  return bb;
}

const int kDiag[4][2] = {{1, 1}, {1, -1}, {-1, 1}, {-1, -1}};
const int kOrth[4][2] = {{1, 0}, {-1, 0}, {0, 1}, {0, -1}};

const Tables& tables();

uint64_t piece_attacks(int pt, int sq, uint64_t occ) {
  const Tables& t = tables();
  switch (pt) {
    case kKnight: return t.knight[sq];
    case kKing: return t.king[sq];
    case kBishop: return slide(sq, occ, kDiag, 4);
    case kRook: return slide(sq, occ, kOrth, 4);
    case kQueen: return slide(sq, occ, kDiag, 4) | slide(sq, occ, kOrth, 4);
    default: return 0;
  }
}

const Tables& tables() {
  static Tables t;
  static std::once_flag once;
  std::call_once(once, [] {
    const int kn[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};
    const int kg[8][2] = {{1, 0}, {1, 1}, {0, 1}, {-1, 1}, {-1, 0}, {-1, -1}, {0, -1}, {1, -1}};
    const int pw[2][2] = {{-1, 1}, {1, 1}};
    const int pb[2][2] = {{-1, -1}, {1, -1}};
    for (int sq = 0; sq < 64; ++sq) {
      t.knight[sq] = step_attacks(sq, kn, 8);
      t.king[sq] = step_attacks(sq, kg, 8);
      t.pawn[kWhite][sq] = step_attacks(sq, pw, 2);
      t.pawn[kBlack][sq] = step_attacks(sq, pb, 2);
    }
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
            uint64_t a = pt == kKnight ? t.knight[from]
                         : pt == kKing ? t.king[from]
                         : pt == kBishop ? slide(from, 0, kDiag, 4)
                         : pt == kRook   ? slide(from, 0, kOrth, 4)
                                         : slide(from, 0, kDiag, 4) | slide(from, 0, kOrth, 4);
            square_offset += popcount(a);
          } else if (from >= 8 && from <= 55) {
            const int push = color == kWhite ? from + 8 : from - 8;
            square_offset += popcount(t.pawn[color][from] | (1ull << push));
          }
        }
        t.threat[pi][64] = square_offset;
        piece_offset += kNumValidTargets[pi] * square_offset;
      }
    }
    t.threat_total = piece_offset;
  });
  return t;
}

inline int halfka_orient(int color, int ksq) { return ((ksq & 7) < 4 ? 7 : 0) ^ (color == kBlack ? 56 : 0); }
inline int threat_orient(int color, int ksq) { return ((ksq & 7) >= 4 ? 7 : 0) ^ (color == kBlack ? 56 : 0); }

struct Pos {
  uint64_t by_piece[12];
  uint64_t occ;
  const uint8_t* board;
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

int king_sq(const Pos& p, int color) {
  const uint64_t k = p.by_piece[kKing * 2 + color];
  return k ? lsb(k) : -1;
}

// fill_halfka_feature_indices_sparse: occupied squares ascending.
int halfka(const Pos& p, int color, int32_t* out) {
  const int ksq = king_sq(p, color);
  if (ksq < 0) return -1;
  const int m = halfka_orient(color, ksq);
  const int bucket = kKingBuckets[ksq ^ m];
  int n = 0;
  for (uint64_t occ = p.occ; occ; occ &= occ - 1) {
    const int sq = lsb(occ);
    const int id = p.board[sq];
    const int piece_index = (id >> 1) * 2 + ((id & 1) != color);
    out[n++] = (sq ^ m) + piece_index * 64 + bucket * 768;
  }
  return n;
}

// full_threat_index (feature_extraction.rs:687-739)
int threat_index(int persp, int attacker, int from, int to, int attacked, int ksq) {
  const Tables& t = tables();
  const bool enemy = (attacker & 1) != (attacked & 1);
  const int m = threat_orient(persp, ksq);
  from ^= m;
  to ^= m;
  if (persp == kBlack) {
    attacker ^= 1;
    attacked ^= 1;
  }
  const int at = attacker >> 1, dt = attacked >> 1;
  const int mapped = kThreatMap[at][dt];
  if (mapped < 0 || (at == dt && (enemy || at != kPawn) && from < to)) return -1;
  uint64_t mask;
  if (at == kPawn) {
    const int ac = attacker & 1;
    const int push = ac == kWhite ? from + 8 : from - 8;
    mask = t.pawn[ac][from] | (1ull << push);
  } else {
    mask = piece_attacks(at, from, 0);
  }
  const int* row = t.threat[attacker];
  return row[65] + ((attacked & 1) * (kNumValidTargets[attacker] / 2) + mapped) * row[64] + row[from] +
         popcount(((1ull << to) - 1) & mask);
}

// fill_full_threat_feature_indices_sparse (feature_extraction.rs:581-675).
// Returns the count, or -1 (no king) / -2 (more than `cap` features).
int threats(const Pos& p, int persp, int32_t* out, int cap) {
  const int ksq = king_sq(p, persp);
  if (ksq < 0) return -1;
  const uint64_t pawns = p.by_piece[kPawn * 2 + kWhite] | p.by_piece[kPawn * 2 + kBlack];
  int n = 0;
  auto push = [&](int attacker, int from, int to) -> bool {
    const int idx = threat_index(persp, attacker, from, to, p.board[to], ksq);
    if (idx >= 0) {
      if (n >= cap) return false;
      out[n++] = idx;
    }
    return true;
  };
  const int order[2] = {persp, 1 - persp};
  for (int ci = 0; ci < 2; ++ci) {
    const int color = order[ci];
    for (int pt = 0; pt < 6; ++pt) {
      const int attacker = pt * 2 + color;
      const uint64_t bb = p.by_piece[attacker];
      if (pt == kPawn) {
        uint64_t left, right, fwd;
        int dl, dr, df;
        if (color == kWhite) {
          left = (bb & ~kHFile) << 9;
          right = (bb & ~kAFile) << 7;
          fwd = bb << 8;
          dl = -9, dr = -7, df = -8;
        } else {
          left = (bb & ~kAFile) >> 9;
          right = (bb & ~kHFile) >> 7;
          fwd = bb >> 8;
          dl = 9, dr = 7, df = 8;
        }
        for (uint64_t x = left & p.occ; x; x &= x - 1)
          if (!push(attacker, lsb(x) + dl, lsb(x))) return -2;
        for (uint64_t x = right & p.occ; x; x &= x - 1)
          if (!push(attacker, lsb(x) + dr, lsb(x))) return -2;
        for (uint64_t x = fwd & pawns; x; x &= x - 1)
          if (!push(attacker, lsb(x) + df, lsb(x))) return -2;
      } else {
        for (uint64_t f = bb; f; f &= f - 1) {
          const int from = lsb(f);
          for (uint64_t x = piece_attacks(pt, from, p.occ) & p.occ; x; x &= x - 1)
            if (!push(attacker, from, lsb(x))) return -2;
        }
      }
    }
  }
  return n;
}

// FeatureSet::fill_feature_indices_sparse: components in order, offsets added,
// compacted; caller fills the -1 tail.
int encode_one(const Pos& p, int color, int fs, int32_t* out) {
  int n = 0;
  if (fs == 1 || fs == 2) {
    const int c = threats(p, color, out, kThreatMax);
    if (c < 0) return c;
    n = c;
  }
  if (fs == 0 || fs == 2) {
    const int offset = fs == 2 ? kThreatInputs : 0;
    const int c = halfka(p, color, out + n);
    if (c < 0) return c;
    if (c > kHalfkaMax) return -2;
    for (int i = 0; i < c; ++i) out[n + i] += offset;
    n += c;
  }
  return n;
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
  tables();
  parallel_for(count, 0, [&](int64_t a, int64_t b) {
    int32_t scratch[kThreatMax];
    for (int64_t i = a; i < b; ++i) {
      uint64_t s = seed * 0xD1B54A32D192ED03ull + (uint64_t)(first + i) * 0x9E3779B97F4A7C15ull;
      uint8_t* bd = board + i * 64;
      for (;;) {
        draw_position(s, bd, stm + i);
        Pos p;
        load(bd, p);
        if (threats(p, kWhite, scratch, kThreatMax) >= 0 && threats(p, kBlack, scratch, kThreatMax) >= 0) break;
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
  tables();
  std::vector<int> status(std::max<int64_t>(count, 1), 0);
  parallel_for(count, nthreads, [&](int64_t a, int64_t b) {
    for (int64_t i = a; i < b; ++i) {
      Pos p;
      load(board + i * 64, p);
      int32_t* rows[2] = {white + i * K, black + i * K};
      int32_t* counts[2] = {white_count, black_count};
      for (int c = 0; c < 2; ++c) {
        const int n = encode_one(p, c, feature_set, rows[c]);
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

int nnue_threat_table_total(void) { return tables().threat_total; }

}  // extern "C"
