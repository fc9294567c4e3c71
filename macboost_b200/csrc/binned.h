// Binned data: MacBoost's .mbds dataset files, binning raw values into the
// trainer's tiled layout, and tree walks over binned rows on the GPU.
//
// Replaces, on the GPU: bin_data (Sources/MacBoost/Shaders.swift:41-76),
// predict_tree_binned and assign_leaves (Shaders.swift:1741-1781); on the
// host: BinnedDataset.load (Sources/MacBoost/Dataset.swift:41-83).  A model
// read from a file walks a dataset's bins after each numeric threshold is
// mapped back to the bin it was trained at (the trainer writes threshold =
// edges[f * (numBins - 2) + bin], Booster.swift:938), which routes every row
// exactly as the float predictor does on the values the bins came from.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace mb {

struct Engine;

// BinnedDataset (Dataset.swift:11-19).
struct Dataset {
  int64_t rows = 0;
  int64_t cols = 0;
  int32_t num_bins = 0;
  std::vector<int64_t> categorical;   // sorted feature indices
  bool has_names = false;
  std::vector<std::string> names;
  std::vector<float> edges;           // cols x (num_bins - 2)
  std::vector<float> labels;          // rows
  std::vector<uint8_t> bins;          // ceil(cols / 8) * 8 * rows, tiled
};

// BinnedDataset.load: little-endian "MBDS" header, version 1, tile width 8.
bool load_mbds(const char* path, Dataset& d, std::string& err);

// Trees in the trainer's split form (NodeSplit, Shaders.swift:466).
struct SplitTrees {
  std::vector<long long> tree_off;
  std::vector<int> feature;
  std::vector<unsigned> sbin, flags, catmask;
  std::vector<float> leaf;
  int max_depth = 0;
};

// A model's trees against a dataset's edges: each numeric threshold becomes
// the first edge index equal to it; fails when a threshold is no edge.
bool model_split_form(const Engine& e, const float* edges, int64_t cols, int num_bins,
                      SplitTrees& s, std::string& err);

// bin_data from host memory into host memory (layout 0 feature-major
// x[f * rows + i], 1 row-major), on `device`.
int bin_data_host(int device, const float* x, int64_t rows, int64_t cols, int layout,
                  const float* edges, int num_bins, const uint8_t* categorical, uint8_t* bins,
                  std::string& err);

// bin_data on device memory, enqueued on `stream` (x feature-major with stride
// ld, or row-major; categorical: cols device bytes or null).
int bin_data_device(int device, const float* x, int64_t rows, int64_t cols, int64_t ld,
                    int layout, const float* edges, int num_bins, const uint8_t* categorical,
                    uint8_t* bins, cudaStream_t stream, std::string& err);

// predict_tree_binned / assign_leaves for trees 0..T-1 from host memory:
// preds class-major (K x rows) updated in place, leaf_idx tree-major (T x rows).
int tree_binned_host(int device, const uint8_t* bins, int64_t rows, int64_t cols, int num_bins,
                     int T, const int64_t* tree_off, const int32_t* feature,
                     const uint32_t* sbin, const uint32_t* flags, const uint32_t* catmask,
                     const float* leaf, int max_depth, int K, float* preds, int32_t* leaf_idx,
                     std::string& err);

// The same on device memory, enqueued on `stream` (no host copies).  A split
// naming a feature or a child outside the arrays sets `status` (device word).
int tree_binned_device(int device, const uint8_t* bins, int64_t rows, int64_t cols, int num_bins,
                       int T, const int64_t* tree_off, const int32_t* feature,
                       const uint32_t* sbin, const uint32_t* flags, const uint32_t* catmask,
                       const float* leaf, int max_depth, int K, float* preds, int32_t* leaf_idx,
                       unsigned* status, cudaStream_t stream, std::string& err);

// Binner.computeEdges (Sources/MacBoost/Binner.swift:26-55): per numeric
// feature of feature-major x, a strided sample (step max(1, rows / 200000))
// without NaN, sorted (stably, as Swift's sort), and the values at indices
// min(m - 1, (k + 1) m / (numBins - 1)) for k < numBins - 2; categorical and
// all-NaN features keep zero edges.
void compute_edges(const float* x, int64_t rows, int64_t cols, int num_bins,
                   const std::vector<char>& categorical, std::vector<float>& edges);

// MacBooster.makeDataset (Booster.swift:392-440): validates labels (finite)
// and categorical ids (integers in 0..<numBins-1 or NaN), computes edges,
// bins on `device`.  x is feature-major host memory.
int make_dataset(int device, const float* x, int64_t rows, int64_t cols, const float* labels,
                 int num_bins, const std::vector<int64_t>& categorical,
                 const std::vector<std::string>* names, Dataset& d, std::string& err);

// BinnedDataset.save (Dataset.swift:26-39).
bool save_mbds(const Dataset& d, const char* path, std::string& err);

// runDataset (Sources/MacBoostCLI/main.swift:134-154): read a table, split
// off the label column, bin the features, write `output_path`.
bool cli_dataset(const char* data_path, int format, const char* label, const char* categorical,
                 int num_bins, int device, const char* output_path, int64_t* rows_out,
                 int64_t* cols_out, std::string& err);

// A model's output of `kind` on every row of a dataset (rows sharded over
// `devices`), row-major like engine_predict_host.
int predict_dataset(Engine& e, const Dataset& d, int kind, const std::vector<int>& devices,
                    void* out, std::string& err);

}  // namespace mb
