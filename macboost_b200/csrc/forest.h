// Device forest layout and launch plan.
//
// A MacBoost forest (implicit heaps, Booster.swift:119-146) is flattened once
// per model into a byte blob of *tree blocks*; each block is staged into
// shared memory with bulk copies.  Rows are scored one per thread from a row
// tile in shared memory that holds one 4*R-byte row per *slot*.
//
// Slots.  Every feature some reachable split reads gets one staging slot,
// filled from HBM with a bulk copy of R consecutive values of that feature.
// With NaN planes (the default), a feature read by a numeric split whose
// missing values go LEFT also gets a second slot holding the same values with
// NaN replaced by -Inf (each thread rewrites its own row of it after the tile
// lands).  A numeric node then reads the slot of its default direction and
// routes with a single unordered compare, right = !(v <= t):
//   raw slot : NaN fails v <= t and goes right        (default right)
//   -Inf slot: -Inf <= t for every finite threshold    (default left)
// -Inf itself behaves identically in both slots.  Thresholds are finite
// because the model file cannot hold anything else (JSON numbers that fit a
// float32).  Without planes the default direction is a record flag instead.
//
// COMPLETE layout (forests no deeper than kMaxCompleteDepth).  Every tree is
// padded to the forest depth D: a leaf reached at depth d < D becomes a
// complete subtree whose 2^(D-d) leaves all carry that leaf's value and heap
// index, so each tree is a fixed D steps of child = 2n + 1 + go_right.  A
// block of Tb trees holds
//   records [Tb][2^D]  uint2   slot 0 unused, heap node n in slot n + 1, so
//                               that every heap level starts on a 128-byte
//                               line (conflict-free record loads)
//   leaves  [Tb][2^D]  float   at byte offset leaf_off (128-aligned)
//
// EXPLICIT layout (deeper, sparse trees such as leaf-wise models).  The
// reachable nodes of each tree are stored breadth-first with both children of
// a node adjacent, so child = first_child + go_right.  Leaf records loop on
// themselves, so all trees of a group walk the same number of steps.  A block
// holds
//   header [4 + Tb + Tb/G]  uint32  [0] trees, [1] first tree index, [4 + i]
//                            first record of tree i, [4 + Tb + g] steps of
//                            group g (padded to 16 bytes)
//   records [...]    uint2
// and blocks are variable-sized (block_off[] gives their byte offsets).
//
// Node record (uint2):
//   x bits 0..2  flags  bit0: no-planes numeric node -> NaN goes left;
//                             categorical node -> codes >= 32 go left
//                       bit1: categorical split
//                       bit2: categorical split with a full 256-bit mask
//   x bits 7..17 byte offset of the slot row in the tile (a multiple of 4*R)
//   x bits 18..31 explicit layout: index distance to the first child
//   explicit-layout leaf: x = the -Inf slot | bit0, child distance 0,
//                         y = leaf value bits
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
constexpr uint32_t kRecSlotMask = 0x3FF80u;   // bits 7..17
constexpr int kRecChildShift = 18;
// Complete layout without planes or categorical splits (FlatForest::payload):
// a numeric record's slot word, as a float, is the operand of the walk's
// fmax(v, c) -- a NaN for default-right nodes (fmax keeps v, and the unordered
// compare sends NaN right), a finite value at or below -2^127 for default-left
// ones (fmax turns NaN into it) -- with the slot offset in bits 7..17.
constexpr uint32_t kRecPayloadLeft = 0xFF000000u;
constexpr uint32_t kRecPayloadRight = 0xFFC00000u;  // a quiet NaN
constexpr uint32_t kMaxChildDelta = 16383u;
constexpr uint32_t kMaxCompactDelta = 2047u;  // 8 x distance still fits bits 18-31

// Shared-memory budget per CTA on B200 (sm_100: 227 KB opt-in).
constexpr size_t kSmemBudget = 232448;
constexpr size_t kSmemHeader = 640;  // mbarriers: 4 per CTA at 0, then 2 per warp at 128

// Deepest forest flattened to the complete layout.
constexpr int kMaxCompleteDepth = 8;
constexpr int64_t kMaxExplicitNodes = 16384;

enum class Layout : int { kComplete = 0, kExplicit = 1 };

// Trees walked concurrently by one thread (independent dependency chains).
// Always a multiple of K, so that tree j of a group scores class j % K.  The
// planner picks one of group_options(K); groups of 12 or more trees need the
// register budget of at most max_threads_for_group(K, G) threads per CTA.
std::vector<int> group_options(int K);
int max_threads_for_group(int K, int G);

struct LaunchPlan {
  int R = 0;              // rows per tile == threads per CTA
  int tile_bufs = 0;      // 1 or 2 (double-buffered row tiles)
  bool planes = true;     // NaN planes (see above) or default-left flags
  int Tb = 0;             // trees per block (complete layout)
  int nblocks = 0;        // blocks in the forest
  uint32_t buf_bytes = 0; // bytes of one forest buffer in shared memory
  uint32_t tile_bytes = 0;// bytes of one row-tile buffer
  size_t smem = 0;        // dynamic shared memory bytes per CTA
  double est_clk_per_row = 0;  // planner's estimate (SM clocks per row)
  std::string note;
  // Restrictions from MACBOOST_PLAN (0: none).  grid: at most this many CTAs
  // per launch, so that every persistent CTA (and warp) loops over several
  // row tiles even on small inputs; chunk: rows per host chunk of a
  // host-memory predict (default: 256 MB of staged input or output).
  int grid_cap = 0;
  int64_t chunk_rows = 0;
  // Row chunks (tiles) after each warp's (CTA's) first are claimed from
  // per-stream counters; "claim=0" fixes the order instead.
  bool claim = true;
};

struct FlatForest {
  Layout layout = Layout::kComplete;
  int T = 0;              // real trees
  int Tpad = 0;           // incl. padding
  int G = 8;              // tree group size
  int K = 1;
  int S_stage = 0;        // staged slots (one per used feature)
  int S_total = 0;        // staged + -Inf slots + category-code slots beside values
  std::vector<int32_t> stage_feature;  // [S_stage] model feature of each staged slot
  std::vector<int32_t> conv_src;       // -Inf slot fills: source slot ...
  std::vector<int32_t> conv_dst;       // ... and destination slot (may be equal)
  // category codes: the kernel writes each staged value of slot code_src[i]
  // as its category code (integer bits) into slot code_dst[i] (the same slot
  // when only categorical splits read the feature), and categorical records
  // address the code slots
  std::vector<int32_t> code_src, code_dst;
  LaunchPlan plan;
  std::vector<uint8_t> blob;           // all blocks
  std::vector<uint64_t> block_off;     // [nblocks + 1] byte offsets in blob
  std::vector<uint32_t> full_masks;    // [n][8]
  std::vector<int32_t> leaf_heap;      // complete: [Tpad][2^D]; explicit: [records]
  std::vector<uint32_t> block_rec_base;// explicit: first record index of each block
  int D = 0;                           // complete layout depth
  uint32_t leaf_off = 0;               // complete layout: leaves offset in a block
  int max_depth = 0;
  int64_t nodes = 0;
  // complete layout: records of heap nodes 0, 1, 2 of each padded tree (3 per
  // tree, x | y << 32), passed to the kernel as a parameter; empty when the
  // forest is deeper than it allows (more than kTopTrees trees, or D < 2)
  std::vector<uint64_t> top_recs;
  uint32_t neg_inf_slot_bytes = 0xFFFFFFFFu;  // explicit: tile offset of the -Inf slot
  // explicit: record bits 18-31 hold 8 x the child distance (every distance
  // at most kMaxCompactDelta), else the distance itself
  bool compact_children = false;

  // Binned-code layout (see forest_codes.cpp): each staged value becomes its
  // rank among the forest's distinct thresholds of that feature, stored as
  // code_bytes-wide codes; node records are 4 bytes.
  bool codes = false;
  // Complete layout: numeric records hold kRecPayloadLeft/Right (launched as
  // layout 3).
  bool payload = false;
  int code_bytes = 1;                  // 1 (u8) or 2 (u16)
  int S_code = 0;                      // code slots in the tile
  uint32_t code_tile_bytes = 0;        // bytes of the code tile (after the raw tile)
  int search_depth = 0;                // d: search tables hold 2^d floats (index 0 unused)
  std::vector<float> search;           // [tables][2^d] Eytzinger-ordered thresholds
  std::vector<int32_t> bin_plan;       // [S_stage][4]: table, NaN-right slot, NaN-left slot,
                                       //               categorical slot (-1: none)
  std::vector<uint32_t> cat_masks;     // [n][8] masks of categorical nodes
};

// Flatten a validated model into the device layout and choose a launch plan.
// `force_planes`: -1 choose, 0 never, 1 always (when it fits).  The binned-code
// layout is used when it applies and the planner estimates it faster
// (MACBOOST_PLAN="codes=0" / "codes=1" restricts the choice).
bool flatten_forest(const Model& m, FlatForest& out, std::string& err, int force_planes = -1);

// Binned-code flattening of a complete-layout forest; false (with `why`) when
// the forest does not qualify (too deep, too many distinct thresholds).
bool flatten_codes(const Model& m, FlatForest& out, std::string& why, int force_G = 0,
                   int force_R = 0);

// The "grid" restriction of MACBOOST_PLAN (0 when unset), for launchers that
// have no forest plan (the binned-data kernels).
int plan_grid_cap_from_env();
// The "shapglobal" restriction (0 when unset): TreeSHAP accumulators in global
// memory, at most that many 128-row CTAs per SM.
int plan_shap_global_from_env();
// The "shapdense" restriction: 0 keeps TreeSHAP off its 128-register build
// (-1 when unset).
int plan_shap_dense_from_env();

// Human-readable JSON description of a flattened forest.
std::string describe_forest(const FlatForest& f);

}  // namespace mb
