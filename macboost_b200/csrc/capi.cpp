// extern "C" boundary of libmacboostc.so (declared in include/macboost_c.h).
//
// Error behaviour follows Sources/MacBoostC/CAPI.swift: failures return -1
// (NULL for constructors) and, when `err` is non-NULL, store a strdup'ed
// message that the caller frees with macboost_free_string (CAPI.swift:77-80).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/macboost_c.h"
#include "binned.h"
#include "engine.h"
#include "table.h"

namespace {

void set_error(char** err, const std::string& msg) {
  if (err) *err = strdup(msg.c_str());
}

mb::Engine* engine(void* h) { return static_cast<mb::Engine*>(h); }

// Devices for the reference-signature predict: MACBOOST_DEVICES="0,2,..."
// when set, else the calling thread's current device.
std::vector<int> default_devices() {
  std::vector<int> d;
  if (const char* s = std::getenv("MACBOOST_DEVICES")) {
    const char* p = s;
    while (*p) {
      char* end = nullptr;
      long v = std::strtol(p, &end, 10);
      if (end == p) break;
      d.push_back(int(v));
      p = end;
      while (*p == ',' || *p == ' ') ++p;
    }
  }
  return d;
}

constexpr const char* kNoTraining = "not supported by this inference engine";

}  // namespace

extern "C" {

void* macboost_load(const char* path, char** err) {
  if (!path) {
    set_error(err, "null path");
    return nullptr;
  }
  std::string e;
  mb::Engine* h = mb::engine_load(path, e);
  if (!h) set_error(err, e);
  return h;
}

void* macboost_load_json(const char* json, int64_t len, char** err) {
  if (!json || len < 0) {
    set_error(err, "null or empty JSON");
    return nullptr;
  }
  std::string e;
  mb::Engine* h = mb::engine_from_json(json, size_t(len), e);
  if (!h) set_error(err, e);
  return h;
}

int32_t macboost_predict(void* handle, const float* x, int64_t rows, int64_t cols, float* out,
                         char** err) {
  if (!handle || !x || !out) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::engine_predict_host(*engine(handle), x, rows, cols, 0, mb::kKindPredict,
                              default_devices(), out, e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_ex(void* handle, const float* x, int64_t rows, int64_t cols,
                            int32_t layout, int32_t kind, const int32_t* devices, int32_t ndev,
                            void* out, char** err) {
  if (!handle || !x || !out || (ndev > 0 && !devices) || ndev < 0) {
    set_error(err, "null argument");
    return -1;
  }
  std::vector<int> devs(devices, devices + ndev);
  std::string e;
  if (mb::engine_predict_host(*engine(handle), x, rows, cols, layout, kind, devs, out, e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_device(void* handle, int32_t device, const float* x_dev, int64_t rows,
                                int64_t cols, int64_t ld, int32_t layout, int32_t kind,
                                void* out_dev, void* stream, char** err) {
  if (!handle || !x_dev || !out_dev) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::engine_predict_device(*engine(handle), device, x_dev, rows, cols, ld, layout, kind,
                                out_dev, static_cast<cudaStream_t>(stream), e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_prepare(void* handle, const int32_t* devices, int32_t ndev, char** err) {
  if (!handle || (ndev > 0 && !devices) || ndev < 0) {
    set_error(err, "null argument");
    return -1;
  }
  std::vector<int> devs(devices, devices + ndev);
  if (devs.empty()) {
    int cur = 0;
    cudaGetDevice(&cur);
    devs.push_back(cur);
  }
  for (int d : devs) {
    std::string e;
    if (!mb::engine_prepare(*engine(handle), d, e) || mb::noalloc_setup(d, e) != 0) {
      set_error(err, e);
      return -1;
    }
  }
  return 0;
}

int32_t macboost_check_device(void* handle, int32_t device, char** err) {
  if (!handle) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::engine_check_device(*engine(handle), device, e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int64_t macboost_num_classes(void* handle) {
  return handle ? int64_t(engine(handle)->model.K) : -1;
}

int64_t macboost_num_trees(void* handle) {
  return handle ? int64_t(engine(handle)->model.trees.size()) : -1;
}

int64_t macboost_num_features(void* handle) {
  return handle ? engine(handle)->model.num_features : -1;
}

int64_t macboost_best_iteration(void* handle) { return handle ? 0 : -1; }

char* macboost_warnings(void* /*handle*/) { return nullptr; }

int64_t macboost_output_cols(void* handle, int32_t kind) {
  if (!handle || kind < mb::kKindPredict || kind > mb::kKindCli) return -1;
  return mb::output_cols(*engine(handle), kind);
}

// MacBooster.featureImportance (Booster.swift:1926-1940): per feature, the
// number of reachable splits or their summed gain, visiting each tree's nodes
// in the reference's stack order so the float32 sums round identically.
int32_t macboost_feature_importance(void* handle, int32_t type, float* out) {
  if (!handle || !out) return -1;
  const mb::Model& m = engine(handle)->model;
  std::vector<float> imp(size_t(m.num_features), 0.0f);
  for (const mb::Tree& t : m.trees) {
    std::vector<int64_t> stack{0};
    while (!stack.empty()) {
      const int64_t n = stack.back();
      stack.pop_back();
      if (t.feature[size_t(n)] < 0) continue;
      const size_t f = size_t(t.feature[size_t(n)]);
      if (type == 1)
        imp[f] += 1.0f;
      else
        imp[f] += size_t(n) < t.gain.size() ? t.gain[size_t(n)] : 0.0f;
      stack.push_back(2 * n + 1);
      stack.push_back(2 * n + 2);
    }
  }
  std::memcpy(out, imp.data(), imp.size() * sizeof(float));
  return 0;
}

int32_t macboost_save(void* handle, const char* path, char** err) {
  if (!handle || !path) {
    set_error(err, "null argument");
    return -1;
  }
  const std::string text = mb::model_to_json(engine(handle)->model);
  FILE* f = std::fopen(path, "wb");
  if (!f) {
    set_error(err, std::string("cannot write '") + path + "'");
    return -1;
  }
  const bool ok = std::fwrite(text.data(), 1, text.size(), f) == text.size();
  const bool closed = std::fclose(f) == 0;
  if (!ok || !closed) {
    set_error(err, std::string("error writing '") + path + "'");
    return -1;
  }
  return 0;
}

void macboost_free(void* handle) { delete engine(handle); }

void macboost_free_string(char* s) { std::free(s); }

char* macboost_describe(void* handle) {
  if (!handle) return nullptr;
  return strdup(engine(handle)->description.c_str());
}

int32_t macboost_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

uint64_t macboost_kernel_launches(void) { return mb::g_kernel_launches.load(); }

void* macboost_host_alloc(int64_t bytes) {
  void* p = nullptr;
  if (bytes <= 0 || cudaHostAlloc(&p, size_t(bytes), cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

void macboost_host_free(void* p) {
  if (p) cudaFreeHost(p);
}

void* macboost_train(const char*, const float*, int64_t, int64_t, int32_t, const float*,
                     const float*, const float*, int64_t, const float*, char** err) {
  set_error(err, std::string("training is ") + kNoTraining);
  return nullptr;
}

int32_t macboost_select_features(const char*, const float*, int64_t, int64_t, const float*,
                                 const float*, int32_t, int32_t, float, int64_t, int32_t*,
                                 int32_t*, float*, char** err) {
  set_error(err, std::string("feature selection is ") + kNoTraining);
  return 1;
}

int32_t macboost_predict_contrib(void* handle, const float* x, int64_t rows, int64_t cols,
                                 float* out, char** err) {
  if (!handle || !x || !out) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::engine_contrib_host(*engine(handle), x, rows, cols, 0, default_devices(), out, e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_contrib_ex(void* handle, const float* x, int64_t rows, int64_t cols,
                                    int32_t layout, const int32_t* devices, int32_t ndev,
                                    float* out, char** err) {
  if (!handle || !x || !out || (ndev > 0 && !devices) || ndev < 0) {
    set_error(err, "null argument");
    return -1;
  }
  std::vector<int> devs(devices, devices + ndev);
  std::string e;
  if (mb::engine_contrib_host(*engine(handle), x, rows, cols, layout, devs, out, e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_contrib_device(void* handle, int32_t device, const float* x_dev,
                                        int64_t rows, int64_t cols, int64_t ld, int32_t layout,
                                        float* out_dev, void* stream, char** err) {
  if (!handle || !x_dev || !out_dev) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::engine_contrib_device(*engine(handle), device, x_dev, rows, cols, ld, layout, out_dev,
                                static_cast<cudaStream_t>(stream), e) != 0) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int64_t macboost_num_feature_names(void* handle) {
  if (!handle) return -1;
  const mb::Model& m = engine(handle)->model;
  return m.has_feature_names ? int64_t(m.feature_names.size()) : -1;
}

const char* macboost_feature_name(void* handle, int64_t i) {
  if (!handle) return nullptr;
  const mb::Model& m = engine(handle)->model;
  if (!m.has_feature_names || i < 0 || i >= int64_t(m.feature_names.size())) return nullptr;
  return m.feature_names[size_t(i)].c_str();
}

void* macboost_table_read(const char* path, int32_t format, char** err) {
  if (!path) {
    set_error(err, "null path");
    return nullptr;
  }
  auto* t = new (std::nothrow) mb::Table();
  if (!t) {
    set_error(err, "out of host memory");
    return nullptr;
  }
  std::string e;
  if (!mb::read_table(path, format, mb::ColumnChooser(), false, *t, e)) {
    delete t;
    set_error(err, e);
    return nullptr;
  }
  return t;
}

int64_t macboost_table_rows(void* table) {
  return table ? static_cast<mb::Table*>(table)->rows : -1;
}

int64_t macboost_table_cols(void* table) {
  return table ? static_cast<mb::Table*>(table)->width() : -1;
}

const char* macboost_table_column_name(void* table, int64_t col) {
  if (!table) return nullptr;
  const mb::Table& t = *static_cast<mb::Table*>(table);
  if (col < 0 || col >= t.width()) return nullptr;
  return t.header[size_t(t.columns[size_t(col)])].c_str();
}

const float* macboost_table_data(void* table) {
  return table ? static_cast<mb::Table*>(table)->data : nullptr;
}

void macboost_table_free(void* table) { delete static_cast<mb::Table*>(table); }

int32_t macboost_write_predictions(const float* preds, int64_t rows, int64_t k, const char* path,
                                   char** err) {
  std::string e;
  if (!mb::write_predictions(preds, rows, k, path, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_cli_predict(void* handle, const char* data_path, int32_t format, int32_t raw,
                             const int32_t* devices, int32_t ndev, const char* output_path,
                             int64_t* rows_out, char** err) {
  if (!handle || !data_path || !output_path || (ndev > 0 && !devices) || ndev < 0) {
    set_error(err, "null argument");
    return -1;
  }
  std::vector<int> devs(devices, devices + ndev);
  if (devs.empty()) devs = default_devices();
  std::string e;
  if (!mb::cli_predict(*engine(handle), data_path, format, raw != 0, devs, output_path, rows_out,
                       e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

// ---- binned data -----------------------------------------------------------

int32_t macboost_bin_data(const float* x, int64_t rows, int64_t cols, int32_t layout,
                          const float* edges, int32_t num_bins, const uint8_t* categorical,
                          int32_t device, uint8_t* bins, char** err) {
  if ((rows > 0 && cols > 0) && (!x || !bins || (!edges && num_bins > 2))) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::bin_data_host(device, x, rows, cols, layout, edges, num_bins, categorical, bins, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_bin_data_device(const float* x, int64_t rows, int64_t cols, int64_t ld,
                                 int32_t layout, const float* edges, int32_t num_bins,
                                 const uint8_t* categorical, int32_t device, uint8_t* bins,
                                 void* stream, char** err) {
  if ((rows > 0 && cols > 0) && (!x || !bins || !edges)) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::bin_data_device(device, x, rows, cols, ld, layout, edges, num_bins, categorical, bins,
                          static_cast<cudaStream_t>(stream), e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_tree_binned(const uint8_t* bins, int64_t rows, int64_t cols,
                                     int32_t num_bins, int32_t num_trees,
                                     const int64_t* tree_offsets, const int32_t* split_feature,
                                     const uint32_t* split_bin, const uint32_t* split_flags,
                                     const uint32_t* cat_mask, const float* leaf_values,
                                     int32_t max_depth, int32_t num_classes, int32_t device,
                                     float* preds, int32_t* leaf_idx, char** err) {
  if (num_trees > 0 && rows > 0 &&
      (!bins || !tree_offsets || !split_feature || !split_bin || !split_flags || !cat_mask ||
       !leaf_values)) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::tree_binned_host(device, bins, rows, cols, num_bins, num_trees, tree_offsets,
                           split_feature, split_bin, split_flags, cat_mask, leaf_values,
                           max_depth, num_classes, preds, leaf_idx, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_tree_binned_device(
    const uint8_t* bins, int64_t rows, int64_t cols, int32_t num_bins, int32_t num_trees,
    const int64_t* tree_offsets, const int32_t* split_feature, const uint32_t* split_bin,
    const uint32_t* split_flags, const uint32_t* cat_mask, const float* leaf_values,
    int32_t max_depth, int32_t num_classes, int32_t device, float* preds, int32_t* leaf_idx,
    uint32_t* status, void* stream, char** err) {
  if (num_trees > 0 && rows > 0 &&
      (!bins || !tree_offsets || !split_feature || !split_bin || !split_flags || !cat_mask ||
       !leaf_values || !status)) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (mb::tree_binned_device(device, bins, rows, cols, num_bins, num_trees, tree_offsets,
                             split_feature, split_bin, split_flags, cat_mask, leaf_values,
                             max_depth, num_classes, preds, leaf_idx, status,
                             static_cast<cudaStream_t>(stream), e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

void* macboost_dataset_load(const char* path, char** err) {
  if (!path) {
    set_error(err, "null path");
    return nullptr;
  }
  auto* d = new (std::nothrow) mb::Dataset();
  if (!d) {
    set_error(err, "out of host memory");
    return nullptr;
  }
  std::string e;
  if (!mb::load_mbds(path, *d, e)) {
    delete d;
    set_error(err, e);
    return nullptr;
  }
  return d;
}

static mb::Dataset* dataset(void* d) { return static_cast<mb::Dataset*>(d); }

int64_t macboost_dataset_rows(void* ds) { return ds ? dataset(ds)->rows : -1; }
int64_t macboost_dataset_cols(void* ds) { return ds ? dataset(ds)->cols : -1; }
int32_t macboost_dataset_num_bins(void* ds) { return ds ? dataset(ds)->num_bins : -1; }
const uint8_t* macboost_dataset_bins(void* ds) { return ds ? dataset(ds)->bins.data() : nullptr; }
const float* macboost_dataset_edges(void* ds) { return ds ? dataset(ds)->edges.data() : nullptr; }
const float* macboost_dataset_labels(void* ds) {
  return ds ? dataset(ds)->labels.data() : nullptr;
}
int64_t macboost_dataset_num_categorical(void* ds) {
  return ds ? int64_t(dataset(ds)->categorical.size()) : -1;
}
int64_t macboost_dataset_categorical(void* ds, int64_t i) {
  if (!ds || i < 0 || i >= int64_t(dataset(ds)->categorical.size())) return -1;
  return dataset(ds)->categorical[size_t(i)];
}
int64_t macboost_dataset_num_feature_names(void* ds) {
  if (!ds) return -1;
  return dataset(ds)->has_names ? int64_t(dataset(ds)->names.size()) : -1;
}
const char* macboost_dataset_feature_name(void* ds, int64_t i) {
  if (!ds || !dataset(ds)->has_names || i < 0 || i >= int64_t(dataset(ds)->names.size()))
    return nullptr;
  return dataset(ds)->names[size_t(i)].c_str();
}
void macboost_dataset_free(void* ds) { delete dataset(ds); }

void* macboost_dataset_make(const float* x, int64_t rows, int64_t cols, const float* labels,
                            int32_t num_bins, const int64_t* categorical, int64_t n_categorical,
                            const char* const* feature_names, int32_t device, char** err) {
  if (n_categorical < 0 || (n_categorical > 0 && !categorical)) {
    set_error(err, "null argument");
    return nullptr;
  }
  std::vector<int64_t> cats(categorical, categorical + n_categorical);
  std::vector<std::string> names;
  if (feature_names)
    for (int64_t f = 0; f < cols; ++f) names.emplace_back(feature_names[f] ? feature_names[f] : "");
  auto* d = new (std::nothrow) mb::Dataset();
  if (!d) {
    set_error(err, "out of host memory");
    return nullptr;
  }
  std::string e;
  if (mb::make_dataset(device, x, rows, cols, labels, num_bins, cats,
                       feature_names ? &names : nullptr, *d, e)) {
    delete d;
    set_error(err, e);
    return nullptr;
  }
  return d;
}

int32_t macboost_dataset_save(void* ds, const char* path, char** err) {
  if (!ds || !path) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (!mb::save_mbds(*dataset(ds), path, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_cli_dataset(const char* data_path, int32_t format, const char* label,
                             const char* categorical, int32_t num_bins, int32_t device,
                             const char* output_path, int64_t* rows_out, int64_t* cols_out,
                             char** err) {
  if (!data_path || !output_path) {
    set_error(err, "null argument");
    return -1;
  }
  std::string e;
  if (!mb::cli_dataset(data_path, format, label, categorical, num_bins, device, output_path,
                       rows_out, cols_out, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

int32_t macboost_predict_dataset(void* handle, void* ds, int32_t kind, const int32_t* devices,
                                 int32_t ndev, void* out, char** err) {
  if (!handle || !ds || (ndev > 0 && !devices) || ndev < 0) {
    set_error(err, "null argument");
    return -1;
  }
  std::vector<int> devs(devices, devices + ndev);
  if (devs.empty()) devs = default_devices();
  std::string e;
  if (mb::predict_dataset(*engine(handle), *dataset(ds), kind, devs, out, e)) {
    set_error(err, e);
    return -1;
  }
  return 0;
}

}  // extern "C"
