// Feature-index encoder, written once for the host (features.cpp, compiled
// by the host compiler) and the device (ft_encode.cuh, compiled by nvcc), so
// both produce the same indices by construction.
//
// It restates the reference's feature functions (src/rust/feature_extraction.rs):
// HalfKAv2_hm (:391-404, :677-685, :745-752), Full_Threats (:581-675,
// :687-739, :754-832) and their composition with component offsets
// (:213-241).  Standard chess attack sets (the reference takes them from the
// sfbinpack crate) come from FeatureTables, built from the rules of chess.
#pragma once

#include <stdint.h>

#include "feature_tables.h"

#if defined(__CUDACC__)
#define NNUE_HD __host__ __device__ __forceinline__
#else
#define NNUE_HD inline
#endif

namespace nnue_feat {

NNUE_HD int popcount64(uint64_t x) {
#if defined(__CUDA_ARCH__)
  return __popcll(x);
#else
  return __builtin_popcountll(x);
#endif
}

NNUE_HD int lsb64(uint64_t x) {  // x != 0
#if defined(__CUDA_ARCH__)
  return __ffsll((long long)x) - 1;
#else
  return __builtin_ctzll(x);
#endif
}

NNUE_HD int msb64(uint64_t x) {  // x != 0
#if defined(__CUDA_ARCH__)
  return 63 - __clzll((long long)x);
#else
  return 63 - __builtin_clzll(x);
#endif
}

// Attacks along one ray, up to and including the nearest occupied square.
NNUE_HD uint64_t ray_attacks(const FeatureTables& t, int d, int sq, uint64_t occ) {
  uint64_t a = t.ray[d][sq];
  const uint64_t blockers = a & occ;
  if (blockers) a ^= t.ray[d][d < 4 ? lsb64(blockers) : msb64(blockers)];
  return a;
}

NNUE_HD uint64_t diagonal_attacks(const FeatureTables& t, int sq, uint64_t occ) {
  return ray_attacks(t, kRayNE, sq, occ) | ray_attacks(t, kRayNW, sq, occ) | ray_attacks(t, kRaySW, sq, occ) |
         ray_attacks(t, kRaySE, sq, occ);
}

NNUE_HD uint64_t orthogonal_attacks(const FeatureTables& t, int sq, uint64_t occ) {
  return ray_attacks(t, kRayE, sq, occ) | ray_attacks(t, kRayN, sq, occ) | ray_attacks(t, kRayW, sq, occ) |
         ray_attacks(t, kRayS, sq, occ);
}

// sfbinpack attacks::piece_attacks for N, B, R, Q, K (pawns are handled by
// their callers).
NNUE_HD uint64_t piece_attacks(const FeatureTables& t, int pt, int sq, uint64_t occ) {
  switch (pt) {
    case kKnight: return t.knight[sq];
    case kKing: return t.king[sq];
    case kBishop: return diagonal_attacks(t, sq, occ);
    case kRook: return orthogonal_attacks(t, sq, occ);
    case kQueen: return diagonal_attacks(t, sq, occ) | orthogonal_attacks(t, sq, occ);
    default: return 0;
  }
}

NNUE_HD int halfka_orient(int color, int ksq) { return ((ksq & 7) < 4 ? 7 : 0) ^ (color == kBlack ? 56 : 0); }
NNUE_HD int threat_orient(int color, int ksq) { return ((ksq & 7) >= 4 ? 7 : 0) ^ (color == kBlack ? 56 : 0); }

// One position: bitboards per piece id, occupancy and the board bytes.
struct PosView {
  const uint64_t* by_piece;  // [12]
  uint64_t occ;
  const uint8_t* board;      // [64]
};

NNUE_HD int king_sq(const PosView& p, int color) {
  const uint64_t k = p.by_piece[kKing * 2 + color];
  return k ? lsb64(k) : -1;
}

// A pawn on the first or last rank has no slot in the threat table
// (pawn slots exist for from in 8..55 only, feature_extraction.rs:800-806).
NNUE_HD bool pawns_on_valid_ranks(const PosView& p) {
  const uint64_t back_ranks = 0xFF000000000000FFull;
  return ((p.by_piece[kPawn * 2 + kWhite] | p.by_piece[kPawn * 2 + kBlack]) & back_ranks) == 0;
}

// Output sinks take the indices in order.  RowSink writes them straight into
// a row; the device encoder uses a buffering sink (ft_encode.cuh).
struct RowSink {
  int32_t* row;
  int n;
  NNUE_HD void push(int v) { row[n++] = v; }
};

// fill_halfka_feature_indices_sparse: occupied squares ascending, each index
// plus `offset`.  Returns the count, or -1 (no king of that colour) or -2
// (more than kHalfkaMax pieces).
template <class Sink>
NNUE_HD int encode_halfka(const FeatureTables& t, const PosView& p, int color, int offset, Sink& out) {
  const int ksq = king_sq(p, color);
  if (ksq < 0) return -1;
  if (popcount64(p.occ) > kHalfkaMax) return -2;
  const int m = halfka_orient(color, ksq);
  const int base = t.king_bucket[ksq ^ m] * 768 + offset;
  int n = 0;
  for (uint64_t occ = p.occ; occ; occ &= occ - 1) {
    const int sq = lsb64(occ);
    const int id = p.board[sq];
    const int piece_index = (id >> 1) * 2 + ((id & 1) != color);
    out.push((sq ^ m) + piece_index * 64 + base);
    ++n;
  }
  return n;
}

// full_threat_index (feature_extraction.rs:687-739); -1 = no feature.
NNUE_HD int threat_index(const FeatureTables& t, int persp, int attacker, int from, int to, int attacked, int ksq) {
  const bool enemy = (attacker & 1) != (attacked & 1);
  const int m = threat_orient(persp, ksq);
  from ^= m;
  to ^= m;
  if (persp == kBlack) {
    attacker ^= 1;
    attacked ^= 1;
  }
  const int at = attacker >> 1, dt = attacked >> 1;
  const int mapped = t.threat_map[at][dt];
  if (mapped < 0 || (at == dt && (enemy || at != kPawn) && from < to)) return -1;
  uint64_t mask;
  if (at == kPawn) {
    const int ac = attacker & 1;
    const int push = ac == kWhite ? from + 8 : from - 8;  // from in 8..55 (pawns_on_valid_ranks)
    mask = t.pawn[ac][from] | (1ull << push);
  } else {
    mask = t.empty_attacks[at][from];
  }
  const int32_t* row = t.threat[attacker];
  return row[65] + ((attacked & 1) * (t.num_valid_targets[attacker] / 2) + mapped) * row[64] + row[from] +
         popcount64(((1ull << to) - 1) & mask);
}

// fill_full_threat_feature_indices_sparse (feature_extraction.rs:581-675):
// attacker colours in the order (perspective, other), piece types P..K,
// pawns as left captures, right captures, pushes onto pawns; other pieces
// by origin square, targets ascending.  Returns the count, or -1 (no king /
// a pawn on a back rank) or -2 (more than `cap` features).
template <class Sink>
NNUE_HD int encode_threats(const FeatureTables& t, const PosView& p, int persp, Sink& out, int cap) {
  const int ksq = king_sq(p, persp);
  if (ksq < 0 || !pawns_on_valid_ranks(p)) return -1;
  const uint64_t kAFile = 0x0101010101010101ull, kHFile = 0x8080808080808080ull;
  const uint64_t pawns = p.by_piece[kPawn * 2 + kWhite] | p.by_piece[kPawn * 2 + kBlack];
  int n = 0;
  int attacker = 0;
  // one feature per pawn target in `set`; false when the row overflows
  auto pawn_set = [&](uint64_t set, int delta) -> bool {
    for (uint64_t x = set; x; x &= x - 1) {
      const int to = lsb64(x);
      const int idx = threat_index(t, persp, attacker, to + delta, to, p.board[to], ksq);
      if (idx >= 0) {
        if (n >= cap) return false;
        out.push(idx);
        ++n;
      }
    }
    return true;
  };
  for (int ci = 0; ci < 2; ++ci) {
    const int color = ci == 0 ? persp : 1 - persp;
    for (int pt = 0; pt < 6; ++pt) {
      attacker = pt * 2 + color;
      const uint64_t bb = p.by_piece[attacker];
      if (pt == kPawn) {
        // left captures, right captures, pushes onto pawns; `delta` maps a
        // target square back to the pawn's square
        const bool white = color == kWhite;
        const uint64_t left = (white ? (bb & ~kHFile) << 9 : (bb & ~kAFile) >> 9) & p.occ;
        const uint64_t right = (white ? (bb & ~kAFile) << 7 : (bb & ~kHFile) >> 7) & p.occ;
        const uint64_t push = (white ? bb << 8 : bb >> 8) & pawns;
        if (!pawn_set(left, white ? -9 : 9) || !pawn_set(right, white ? -7 : 7) || !pawn_set(push, white ? -8 : 8))
          return -2;
      } else {
        for (uint64_t f = bb; f; f &= f - 1) {
          const int from = lsb64(f);
          for (uint64_t x = piece_attacks(t, pt, from, p.occ) & p.occ; x; x &= x - 1) {
            const int to = lsb64(x);
            const int idx = threat_index(t, persp, attacker, from, to, p.board[to], ksq);
            if (idx >= 0) {
              if (n >= cap) return -2;
              out.push(idx);
              ++n;
            }
          }
        }
      }
    }
  }
  return n;
}

// FeatureSet::fill_feature_indices_sparse: components in order (threats,
// then HalfKA offset by the threat inputs), compacted; the caller fills the
// -1 tail.  feature_set 0 = HalfKAv2_hm, 1 = Full_Threats, 2 = both.
// Returns the count or a negative status (the position is rejected; the
// sink may hold a partial row).
template <class Sink>
NNUE_HD int encode_position(const FeatureTables& t, const PosView& p, int color, int feature_set, Sink& out) {
  int n = 0;
  if (feature_set == 1 || feature_set == 2) {
    const int c = encode_threats(t, p, color, out, kThreatMax);
    if (c < 0) return c;
    n = c;
  }
  if (feature_set == 0 || feature_set == 2) {
    const int c = encode_halfka(t, p, color, feature_set == 2 ? kThreatInputs : 0, out);
    if (c < 0) return c;
    n += c;
  }
  return n;
}

}  // namespace nnue_feat
