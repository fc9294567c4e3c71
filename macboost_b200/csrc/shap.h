// TreeSHAP contributions: host-side path tables for the GPU kernel.
//
// Replaces MacBooster.predictContributions (Sources/MacBoost/SHAP.swift:39-52)
// and its bias column (shapBias, SHAP.swift:56-72).  The forest is
// decomposed once into root-to-leaf paths (a path-dependent TreeSHAP value
// is a sum over leaves, each leaf's share depending only on its own path).
// On a path, all splits on one feature merge into one "unique feature":
// the product z of their cover fractions (in root-to-leaf order) and one
// test that is true exactly when the row satisfies every one of those
// splits -- an interval (lo, hi] and a NaN verdict for numeric splits, a
// 256-bit set of admitted codes for categorical ones.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "model.h"

namespace mb {

constexpr int kShapMaxUnique = 32;  // distinct features on one path

// Device layouts (16 and 32 bytes).
struct ShapPathRec {
  uint32_t first;  // index of the path's first unique-feature record
  uint32_t U;      // unique features on the path (1..kShapMaxUnique)
  double leaf;     // leaf value
};

constexpr uint32_t kShapNanOk = 1u;   // a NaN value satisfies the numeric splits
constexpr uint32_t kShapHasCat = 2u;  // categorical splits: test `mask`

struct ShapUniqueRec {
  double z;        // product of cover(child) / cover(parent) over the feature's splits
  float lo;        // value must satisfy !(v <= lo) (NaN lo: no lower bound)
  float hi;        // and v <= hi (+inf: no upper bound)
  uint32_t slot;   // staged input slot of the feature
  uint32_t flags;  // kShapNanOk | kShapHasCat
  uint32_t mask;   // index of the admitted-code set (8 words) when kShapHasCat
  uint32_t pad;
};

// Path blocks staged into shared memory by the kernel: at most kShapBlockPaths
// paths and kShapBlockUniq unique-feature records each.
constexpr int kShapBlockPaths = 64;
constexpr int kShapBlockUniq = 256;

struct ShapForest {
  std::vector<ShapPathRec> paths;     // class-major, trees in file order, leaves left to right
  std::vector<uint32_t> class_begin;  // K + 1 offsets into `paths`
  std::vector<uint32_t> block_path;   // nblocks + 1 path boundaries of the staged blocks
  std::vector<uint32_t> block_uniq;   // nblocks + 1 unique-record boundaries
  std::vector<uint32_t> class_block;  // K + 1 offsets into the blocks
  std::vector<ShapUniqueRec> uniq;
  std::vector<uint32_t> masks;        // 8 words per admitted-code set
  std::vector<int32_t> slot_feature;  // staged slot -> feature (empty: no path reads a feature)
  std::vector<int32_t> feature_slot;  // feature -> slot, or -1 when no path uses it
  std::vector<float> bias;            // K expected values, rounded to float32
  std::vector<double> coef;           // (kShapMaxUnique + 1) x (2 kShapMaxUnique + 1)
  int max_unique = 0;
};

// Builds the tables.  Fails for a cover array whose length is neither 0 nor
// the tree's node count, or a path with more than kShapMaxUnique features.
bool build_shap(const Model& m, ShapForest& s, std::string& err);

// coef[U * kShapCoefRow + kShapMaxUnique + s] = s! (U - 1 - s)! / U! for
// 0 <= s < U, and 0 for every other s in [-kShapMaxUnique, kShapMaxUnique].
constexpr int kShapCoefRow = 2 * kShapMaxUnique + 1;

}  // namespace mb
