// Lookup tables of the feature encoder, shared by the host encoder
// (features.cpp) and the device encoder (ft_encode.cuh).  Plain data: the
// device copy is a byte copy of the host struct.
//
// Board encoding: 64 piece ids, square a1 = 0 ... h8 = 63, id = type * 2 +
// colour (type P=0, N=1, B=2, R=3, Q=4, K=5; colour white = 0, black = 1),
// anything >= 12 is an empty square.
#pragma once

#include <stdint.h>

namespace nnue_feat {

constexpr int kEmpty = 12;
constexpr int kPawn = 0, kKnight = 1, kBishop = 2, kRook = 3, kQueen = 4, kKing = 5;
constexpr int kWhite = 0, kBlack = 1;
constexpr int kHalfkaInputs = 24576, kHalfkaMax = 32;
constexpr int kThreatInputs = 60720, kThreatMax = 128;

// Ray directions: 0-3 step to higher square numbers (E +1, N +8, NE +9,
// NW +7), 4-7 to lower ones (W -1, S -8, SW -9, SE -7).  The nearest
// blocker on a ray is its lowest set square for 0-3, its highest for 4-7.
constexpr int kRayE = 0, kRayN = 1, kRayNE = 2, kRayNW = 3, kRayW = 4, kRayS = 5, kRaySW = 6, kRaySE = 7;

struct alignas(16) FeatureTables {
  uint64_t knight[64], king[64], pawn[2][64];  // attack sets (pawn: captures of that colour)
  uint64_t ray[8][64];                         // squares beyond sq in direction d, up to the edge
  uint64_t empty_attacks[6][64];               // attack set on an empty board (pawn rows unused)
  // threat_feature_calc (feature_extraction.rs:788-832), per piece id:
  // [from] = square offset of `from`, [64] = squares total, [65] = piece offset
  int32_t threat[12][66];
  int32_t king_bucket[64];                     // HalfKAv2_hm king buckets (feature_extraction.rs:391-404)
  int32_t num_valid_targets[12];               // NUM_VALID_TARGETS (:27)
  int32_t threat_map[6][6];                    // THREAT_MAP (:28-35)
  int32_t threat_total;
  int32_t pad[3];
};

// Built once, thread-safe.
const FeatureTables& feature_tables();

}  // namespace nnue_feat
