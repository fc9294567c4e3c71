// Host engine: per-model state, per-device replicas and the predict pipelines.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "forest.h"
#include "kernels.h"
#include "model.h"
#include "shap.h"

namespace mb {

// One model replicated on one GPU, plus that GPU's staging buffers.
struct DeviceState {
  int device = -1;
  int num_sms = 0;
  int grid_ctas = 0;                    // persistent CTAs for this model
  cudaStream_t stream[2] = {nullptr, nullptr};
  // model replica
  unsigned char* blob = nullptr;
  unsigned long long* block_off = nullptr;
  unsigned* block_rec_base = nullptr;
  int* stage_feature = nullptr;        // staged slot -> feature
  int* conv_src = nullptr;             // -Inf plane fills
  int* conv_dst = nullptr;
  int* code_src = nullptr;             // category-code fills
  int* code_dst = nullptr;
  float* search = nullptr;             // binned codes: threshold search tables
  int* bin_plan = nullptr;             // binned codes: per staged slot conversions
  unsigned* masks = nullptr;
  int* leaf_heap = nullptr;
  float* base = nullptr;
  unsigned* err = nullptr;              // kernel error word
  // Row-chunk counters of the per-warp pipeline, one pair per stream that
  // launches on this replica (launches on one stream run one after another;
  // each launch leaves its pair at zero): kSchedSlots x {next, done}.
  unsigned long long* sched = nullptr;
  std::vector<cudaStream_t> sched_streams;
  std::mutex sched_mu;
  // staging for host-memory inputs (double-buffered chunks)
  float* xbuf[2] = {nullptr, nullptr};  // feature-major chunk
  size_t xcap[2] = {0, 0};
  float* xraw[2] = {nullptr, nullptr};  // row-major chunk before transposition
  size_t rcap[2] = {0, 0};
  void* obuf[2] = {nullptr, nullptr};
  size_t ocap[2] = {0, 0};
  size_t smem_optin = 0;                // shared memory a block may opt in to
  // TreeSHAP tables, uploaded on the first contributions call
  bool shap_ready = false;
  void* shap_paths = nullptr;
  void* shap_uniq = nullptr;
  unsigned* shap_masks = nullptr;
  unsigned* shap_block_path = nullptr;
  unsigned* shap_block_uniq = nullptr;
  unsigned* shap_class_block = nullptr;
  double* shap_coef = nullptr;
  int* shap_feature_slot = nullptr;
  int* shap_slot_feature = nullptr;
  float* shap_bias = nullptr;
  double* shap_scratch = nullptr;       // accumulators when they do not fit in shared memory
  int shap_R = 0;
  bool shap_in_smem = true;
  bool shap_dense = false;              // the 128-register build (global accumulators)
  size_t shap_smem = 0;
  int shap_grid = 0;
  std::mutex mu;                        // one predict at a time per (model, device)
  ~DeviceState();
};

struct Engine {
  Model model;
  FlatForest flat;
  std::unique_ptr<TopRecords> top;      // complete layout: first two levels as a kernel parameter
  std::string description;
  std::mutex mu;                        // guards `devices`
  std::map<int, std::unique_ptr<DeviceState>> devices;
  // TreeSHAP path tables, built on the first contributions call
  std::mutex shap_mu;
  int shap_state = 0;                   // 0 not built, 1 built, -1 failed (shap_err)
  std::string shap_err;
  ShapForest shap;
};

// Global count of forest-kernel launches (for benchmarking claims).
extern std::atomic<unsigned long long> g_kernel_launches;

Engine* engine_load(const std::string& path, std::string& err);
Engine* engine_from_json(const char* text, size_t len, std::string& err);

// Output elements per row for `kind` (K, max(K,2) for proba, T for leaf).
int64_t output_cols(const Engine& e, int kind);

// Upload the model to `device` (idempotent).  Returns the device state.
DeviceState* engine_prepare(Engine& e, int device, std::string& err);

// Predict from host memory, rows sharded over `devices`.
int engine_predict_host(Engine& e, const float* x, int64_t rows, int64_t cols, int layout,
                        int kind, const std::vector<int>& devices, void* out, std::string& err);

// Enqueue a predict on device memory (asynchronous on `stream`).
int engine_predict_device(Engine& e, int device, const float* x, int64_t rows, int64_t cols,
                          int64_t ld, int layout, int kind, void* out, cudaStream_t stream,
                          std::string& err);

// TreeSHAP contributions from host memory (rows x K x (cols + 1) float32),
// rows sharded over `devices` like engine_predict_host.
int engine_contrib_host(Engine& e, const float* x, int64_t rows, int64_t cols, int layout,
                        const std::vector<int>& devices, float* out, std::string& err);

// TreeSHAP contributions from device memory on `device`, enqueued on
// `stream` (feature-major x[f * ld + i], or row-major; row-major input and
// models too wide for shared-memory accumulators make the call wait).
int engine_contrib_device(Engine& e, int device, const float* x, int64_t rows, int64_t cols,
                          int64_t ld, int layout, float* out, cudaStream_t stream,
                          std::string& err);

// Synchronise `device` and report any kernel-side error since the last check.
int engine_check_device(Engine& e, int device, std::string& err);

// Resolve the no-alloc entry point's scratch on `device` (noalloc.cu); run
// by macboost_prepare for each device it prepares.
int noalloc_setup(int device, std::string& err);

// Enqueue the forest kernel on a device where the model is already resident
// (engine_prepare ran before), reporting kernel-side errors into the caller's
// `status` word and taking row chunks from the caller's `sched` counters (two
// zeroed 64-bit words that only launches serialised with this one use; null:
// a fixed chunk order).  Allocates nothing; fails if the model is not
// resident.  `x` is feature-major with stride ld; `use_stage_map`: x holds
// every model feature (false: only the staged features, in slot order).
int engine_launch_resident(Engine& e, int device, const float* x, int64_t rows, int64_t ld,
                           bool use_stage_map, int kind, void* out, unsigned* status,
                           unsigned long long* sched, cudaStream_t stream, std::string& err);

}  // namespace mb
