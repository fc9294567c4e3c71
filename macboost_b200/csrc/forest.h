// Device forest layout and launch plan.
//
// A MacBoost forest (implicit heaps, Booster.swift:119-146) is flattened once
// per model into a byte blob of *tree blocks*; each block is staged into
// shared memory with one bulk copy.  Only the features that some reachable
// split uses are staged per row tile; they are renumbered into `slots`.
//
// COMPLETE layout (forests no deeper than kMaxCompleteDepth).  Every tree is
// padded to the forest depth D: a leaf reached at depth d < D becomes a
// complete subtree whose 2^(D-d) leaves all carry that leaf's value (its heap
// index is kept in a side table for leaf-index output), so each tree is a
// fixed D steps of child = 2n + 1 + go_right.  A block of Tb trees holds
//   records [Tb][2^D - 1]  uint2    internal nodes
//   leaves  [Tb][2^D]      float    leaf values (at byte offset leaf_off)
//
// EXPLICIT layout (deeper, sparse trees such as leaf-wise models).  The
// reachable nodes of each tree are stored breadth-first with both children of
// a node adjacent, so child = first_child + go_right.  A block holds
//   tree_start [Tb]        uint32   first record of each tree (16-B padded)
//   records    [...]       uint2
// and blocks are variable-sized (block_off[] gives their byte offsets).
//
// Node record (uint2):
//   x bits 0..2  flags  bit0: numeric node -> NaN goes left;
//                             categorical node -> codes >= 32 go left
//                       bit1: categorical split
//                       bit2: categorical split with a full 256-bit mask
//   x bit 3      explicit layout: leaf record (y = leaf value bits)
//   x bits 4..   slot of the split feature (complete: bits 4..31;
//                explicit: bits 4..15, first child in bits 16..31)
//   y            float bits of the threshold (numeric),
//                mask bits 0..31 (categorical, bits 32..dataBins uniform),
//                or the index of the node's 8-word mask (full mask).
//
// Both layouts pad the forest to a multiple of the kernel's tree group size
// with trees whose every leaf is -0.0f: x + (-0.0f) == x bit for bit for any
// float x, so padding never changes a margin.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "model.h"

namespace mb {

struct uint2_like {
  uint32_t x, y;
};

constexpr uint32_t kRecDefaultLeft = 1u;
constexpr uint32_t kRecCategorical = 2u;
constexpr uint32_t kRecFullMask = 4u;
constexpr uint32_t kRecLeaf = 8u;

// Shared-memory budget per CTA on B200 (sm_100: 227 KB opt-in).
constexpr size_t kSmemBudget = 232448;
constexpr size_t kSmemHeader = 128;  // mbarriers + flags

// Deepest forest flattened to the complete layout.
constexpr int kMaxCompleteDepth = 8;
// Explicit layout limits: 12-bit slot, 16-bit child index.
constexpr int64_t kMaxExplicitSlots = 4096;
constexpr int64_t kMaxExplicitNodes = 65535;

enum class Layout : int { kComplete = 0, kExplicit = 1 };

// Trees walked concurrently by one thread (independent dependency chains).
// A multiple of K so that tree j of a group always scores class j % K.
inline int group_size(int K) {
  if (K <= 0 || K > 16) return 8;
  if (K >= 8) return K;
  return K * (8 / K);
}

struct LaunchPlan {
  int R = 0;              // rows per tile == threads per CTA
  int tile_bufs = 0;      // 1 or 2 (double-buffered row tiles)
  int Tb = 0;             // trees per block
  int nblocks = 0;        // blocks in the forest
  uint32_t buf_bytes = 0; // bytes of one forest buffer in shared memory
  size_t smem = 0;        // dynamic shared memory bytes per CTA
  std::string note;
};

struct FlatForest {
  Layout layout = Layout::kComplete;
  int T = 0;              // real trees
  int Tpad = 0;           // incl. padding
  int G = 8;              // tree group size
  int K = 1;
  int S = 0;              // staged feature slots
  std::vector<int32_t> slot_feature;   // [S] model feature of each slot
  LaunchPlan plan;
  std::vector<uint8_t> blob;           // all blocks
  std::vector<uint64_t> block_off;     // [nblocks + 1] byte offsets in blob
  std::vector<uint32_t> full_masks;    // [n][8]
  std::vector<int32_t> leaf_heap;      // complete: [Tpad][2^D]; explicit: [records]
  // complete layout
  int D = 0;
  uint32_t leaf_off = 0;
  // explicit layout: leaf_heap is indexed by (block record base + record)
  std::vector<uint32_t> block_rec_base; // [nblocks] first record index of each block
  int max_depth = 0;
  int64_t nodes = 0;                     // records in the blob (excl. padding)
};

// Flatten a validated model into the device layout and choose a launch plan.
bool flatten_forest(const Model& m, FlatForest& out, std::string& err);

// Human-readable JSON description of a flattened forest.
std::string describe_forest(const FlatForest& f);

}  // namespace mb
