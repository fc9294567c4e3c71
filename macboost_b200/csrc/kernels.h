// Kernel-side argument block and launch entry points (implemented in the
// kernels_*.cu files, called by the host engine).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mb {

// Output kinds of the predict path.
enum Kind : int {
  kKindPredict = 0,  // MacBooster.predict: raw margins, exp for log-link objectives
  kKindRaw = 1,      // raw margins
  kKindProba = 2,    // predict_proba: sigmoid [1-p, p] (K == 1) or softmax (K > 1), float64 math
  kKindLeaf = 3,     // leaf heap index per (row, tree), int32
  kKindCli = 4,      // what `macboost predict` writes: fp32 softmax (K > 1) / sigmoid (binary)
};

// Kernel error bits (written to KArgs::err).
constexpr unsigned kErrWaitTimeout = 1u;

struct KArgs {
  // Rows: feature-major x[f * ld + i] for i < rows.
  const float* x;
  long long rows;
  long long ld;
  int bulk;                        // 1: x and ld allow 16-byte bulk copies of row runs
  const int* stage_feature;        // [S_stage] feature of each staged slot, or null = identity
  const int* conv_src;             // [n_conv] -Inf slot fills (src slot -> dst slot)
  const int* conv_dst;
  int S_stage, n_conv;
  const int* code_src;             // [n_codes] category-code fills (value slot -> code slot)
  const int* code_dst;
  int n_codes;
  // Forest (device copy of FlatForest).
  const unsigned char* blob;
  const unsigned long long* block_off;  // [nblocks + 1]
  const unsigned* block_rec_base;       // explicit layout: first record index per block
  const unsigned* masks;                // full categorical masks, 8 words each
  const int* leaf_heap;
  const float* base;                    // [K] starting margins
  int K, G, T, D, Tb, nblocks;      // G: trees walked at once per thread
  // Binned-code layout: per staged slot {search table, NaN-right code byte
  // offset, NaN-left code byte offset, categorical code byte offset} (-1: none),
  // the Eytzinger search tables [tables][2^search_depth], the code tile size.
  const int* bin_plan;
  const float* search;
  int search_depth;
  unsigned code_tile_bytes;
  unsigned neg_inf_slot;           // explicit layout: tile offset of the constant -Inf slot
  int compact_children;            // explicit layout: record bits 18-31 hold 8 x child distance
  unsigned buf_bytes, leaf_off, tile_bytes;
  int data_bins;
  // Output.
  int kind;
  int log_link;
  int binary;                      // objective is binary logistic (kKindCli sigmoid)
  float* out;                      // float output (kinds 0-2) or null
  int* out_leaf;                   // leaf output (kind 3) or null
  // Launch plan.
  int R, tile_bufs;
  long long ntiles;
  unsigned* err;
  // Bound of every mbarrier wait, in ns of %globaltimer (kDefaultWaitNs
  // unless MACBOOST_WAIT_LIMIT_US says otherwise).
  unsigned long long wait_ns;
  // Test hook (MACBOOST_TEST_STALL_TILES=1, off by default): row-tile
  // barriers expect their bytes but no copy is issued, so the tile waits run
  // out with nothing in flight and the abort path is exercised.
  int stall_tiles;
  // Per-warp pipeline: {next, done} counters from which warps claim row
  // chunks after their first (zero at launch, zero again when the last warp
  // leaves), or null for the fixed order c + k * gridDim.x * warps.
  unsigned long long* sched;
};

constexpr int kSchedSlots = 256;  // counter pairs per device replica (streams)

constexpr unsigned long long kDefaultWaitNs = 2000000000ull;  // 2 s

// Complete layout: the records of heap nodes 0, 1 and 2 of every tree, passed
// by value as a kernel parameter, so the first two levels of the walk read the
// constant bank (uniform per warp) instead of shared memory.  Record of node k
// of tree t at rec[3 t + k], as the 8-byte shared-memory record (x | y << 32).
constexpr int kTopTrees = 1200;
struct TopRecords {
  unsigned long long rec[3 * kTopTrees];
};

// Launch the forest kernel on `stream`.  layout: 0 complete, 1 explicit,
// 2 complete with binned codes (code_bytes 1 or 2), 3 complete with the
// default direction in the record word (FlatForest::payload); planes: NaN planes in the
// tile; cat: the model has categorical splits; top (complete layout only):
// the first two levels' records, or null to read every level from shared memory.
cudaError_t launch_forest(int layout, bool planes, bool cat, const KArgs& a, size_t smem,
                          int grid, cudaStream_t stream, int code_bytes = 1,
                          const TopRecords* top = nullptr);

// Largest number of co-resident CTAs per SM for that kernel.
cudaError_t forest_occupancy(int layout, bool planes, bool cat, int K, int G, int R,
                             size_t smem, int* ctas, int code_bytes = 1, bool top = false);

// TreeSHAP contributions (kernels_shap.cu).  Rows: feature-major
// x[slot_map[s] * ld + i] (x[s * ld + i] when slot_map is null) for the S
// staged slots; output rows x K x (F + 1) float32.
struct ShapArgs {
  const float* x;
  long long rows, ld;
  const int* slot_map;
  int S;
  const void* paths;            // ShapPathRec[...]
  const void* uniq;             // ShapUniqueRec[...]
  const unsigned* masks;        // admitted-code sets, 8 words each
  const unsigned* block_path;   // [nblocks + 1] path boundaries of the staged blocks
  const unsigned* block_uniq;   // [nblocks + 1] unique-record boundaries
  const unsigned* class_block;  // [K + 1] block boundaries per class
  const double* coef;           // Shapley weights, (kShapMaxUnique + 1) x kShapCoefRow
  const int* feature_slot;      // [F]
  const float* bias;            // [K]
  int K, F, data_bins;
  float* out;
  double* scratch;              // global accumulators (gridDim x S x R) when not in shared memory
  int R;                        // rows per CTA (= threads per CTA, <= 256)
  long long ntiles;
  unsigned* err;                // kErrWaitTimeout when a staged block never arrived
};
// Dynamic shared memory of the contributions kernel (maxu: longest path in
// distinct features; smem_variant: row tile and accumulators in shared memory).
size_t shap_smem_bytes(int maxu, bool smem_variant, int S, int R);
// dense: the build with launch bounds (128, 4), global accumulators and paths
// of at most 12 distinct features only
cudaError_t shap_occupancy(int maxu, bool smem_variant, int R, size_t smem, int* ctas,
                           bool dense = false);
cudaError_t launch_shap(const ShapArgs& a, int maxu, bool smem_variant, size_t smem, int grid,
                        cudaStream_t stream, bool dense = false);
// Binned data (kernels_binned.cu).  Tiled bins as MacBoost's trainer keeps
// them: bins[(f / 8) * n * 8 + i * 8 + f % 8] for n rows.
cudaError_t launch_bin_data(const float* x, long long rows, long long cols, long long ld,
                            int layout, const float* edges, int num_bins,
                            const unsigned char* categorical, unsigned char* bins,
                            cudaStream_t stream);
// Trees in split form (NodeSplit: feature, bin, flags; 8 mask words per node).
struct BinnedArgs {
  const unsigned char* bins;
  long long n;                  // rows
  long long cols;               // features in the bin matrix
  int num_bins;
  int T;
  const long long* tree_off;    // [T + 1] node offsets
  const int* feature;
  const unsigned* sbin;
  const unsigned* flags;
  const unsigned* catmask;
  const float* leaf;
  int max_depth;
  int K;
  // per-tree mode (predict_tree_binned / assign_leaves): class-major preds
  // (K x n, updated in place) and tree-major leaf indices (T x n); either may be null
  float* preds;
  int* leaf_idx;
  // forest mode (predict on a dataset): margins from `base` in tree order, then
  // the predict epilogue of output kind `ka.kind` into ka.out (row-major);
  // kKindLeaf writes row-major leaf indices into ka.out_leaf
  int forest_mode;
  const float* base;
  KArgs ka;
  unsigned* err;                // kErrBadTree when a split names a missing feature or child
  long long node_hint;          // nodes of all T trees when the caller knows them, else 0
  unsigned rec_cap;             // set by launch_binned: shared bytes for staged node records
};
constexpr unsigned kErrBadTree = 2u;
cudaError_t launch_binned(const BinnedArgs& a, cudaStream_t stream);

// Row-major [rows][F] -> feature-major [F][ld] (ld >= rows).
cudaError_t launch_transpose(const float* in, long long rows, int F, float* out, long long ld,
                             cudaStream_t stream);

}  // namespace mb
