// Kernel-side argument block and launch entry points (implemented in
// kernels.cu, called by the host engine).
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
};

// Kernel error bits (written to KArgs::err).
constexpr unsigned kErrWaitTimeout = 1u;

struct KArgs {
  // Rows: feature-major x[f * ld + i] for i < rows.
  const float* x;
  long long rows;
  long long ld;
  int bulk;                        // 1: x, ld allow 16-byte bulk copies of row segments
  const int* slot_feature;         // [S] feature of each staged slot, or null = identity
  // Forest (device copy of FlatForest).
  const unsigned char* blob;
  const unsigned long long* block_off;  // [nblocks + 1]
  const unsigned* block_rec_base;       // explicit layout: first record index per block
  const unsigned* masks;                // full categorical masks, 8 words each
  const int* leaf_heap;
  const float* base;                    // [K] starting margins
  int S, K, T, G, D, Tb, nblocks;
  unsigned buf_bytes, leaf_off;
  int data_bins;
  // Output.
  int kind;
  int log_link;
  float* out;                      // float output (kinds 0-2) or null
  int* out_leaf;                   // leaf output (kind 3) or null
  // Launch plan.
  int R, tile_bufs;
  long long ntiles;
  unsigned* err;
};

// Launch the forest kernel for `layout` (0 complete, 1 explicit) on `stream`.
// Returns the CUDA error of the launch.
cudaError_t launch_forest(int layout, int cat, const KArgs& a, size_t smem, int grid,
                          cudaStream_t stream);

// Row-major [rows][F] -> feature-major [F][ld] (ld >= rows).
cudaError_t launch_transpose(const float* in, long long rows, int F, float* out, long long ld,
                             cudaStream_t stream);

// Largest number of co-resident CTAs per SM for the given kernel and smem.
cudaError_t forest_occupancy(int layout, int cat, int K, int R, size_t smem, int* ctas);

}  // namespace mb
