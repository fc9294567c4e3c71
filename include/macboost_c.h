/*
 * macboost_c.h -- C ABI of the B200 batch-inference engine for MacBoost models.
 *
 * libmacboostc.so exports the inference subset of MacBoost's own C ABI
 * (Sources/MacBoostC/CAPI.swift) with the same names, argument meanings and
 * error behaviour, so MacBoost's Python ctypes bridge (python/macboost/_core.py)
 * and Swift callers bind to it unchanged, plus additive entry points for
 * output kinds, device lists, row-major input and device-resident buffers.
 *
 * Conventions (as in the reference):
 *  - a model handle is an opaque pointer from macboost_load, released with
 *    macboost_free;
 *  - matrices are float32; `x` is feature-major, x[f * rows + i], unless an
 *    entry point takes a `layout` argument;
 *  - functions returning int32 return 0 on success and non-zero on failure;
 *    when `err` is non-NULL it then receives a malloc'ed message that the
 *    caller releases with macboost_free_string;
 *  - getters return -1 for a NULL handle.
 * Every predict runs on NVIDIA sm_100a GPUs; there is no CPU fallback: on a
 * machine without such a GPU the predict entry points fail with a message.
 * Handles may be used from several threads; predicts on one handle and one
 * GPU are serialised.
 * A kernel that waits longer than MACBOOST_WAIT_LIMIT_US microseconds (default
 * 2,000,000) for a shared-memory transfer gives up; the call (or the next
 * macboost_check_device) then fails with "gave up waiting".
 */
#ifndef MACBOOST_C_H
#define MACBOOST_C_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible entry points --------------------------------- */

/* Load a MacBoost JSON model file.  Replaces macboost_load,
 * Sources/MacBoostC/CAPI.swift:257-271 (MacBooster.load, Booster.swift:2144-2162).
 * Parses, validates and flattens the forest on the host; GPU replicas are
 * created on first use (or by macboost_prepare).  Returns NULL on failure. */
void *macboost_load(const char *path, char **err);

/* Predict `rows` rows of feature-major x (rows*cols floats) into out
 * (rows * num_classes floats, row-major).  Replaces macboost_predict,
 * CAPI.swift:185-203: MacBooster.predict semantics (Booster.swift:1993-1999),
 * i.e. raw margins, exp() for the poisson/tweedie objectives.  Fails for NULL
 * arguments or cols != num_features.  Runs on the devices named by the
 * MACBOOST_DEVICES environment variable ("0,1,..."), else the current one. */
int32_t macboost_predict(void *handle, const float *x, int64_t rows, int64_t cols, float *out,
                         char **err);

/* Classes scored (outputs per row).  Replaces CAPI.swift:204-208. */
int64_t macboost_num_classes(void *handle);
/* Trees in the model.  Replaces CAPI.swift:272-277. */
int64_t macboost_num_trees(void *handle);
/* Features the model expects.  Replaces CAPI.swift:278-283. */
int64_t macboost_num_features(void *handle);
/* Best iteration; always 0 for a model read from a file.  Replaces CAPI.swift:284-289. */
int64_t macboost_best_iteration(void *handle);
/* Training warnings; always NULL for a model read from a file.  Replaces CAPI.swift:292-297. */
char *macboost_warnings(void *handle);
/* Feature importance (type 0 gain, 1 split count) into out[num_features].
 * Replaces CAPI.swift:211-220 (MacBooster.featureImportance, Booster.swift:1926-1940). */
int32_t macboost_feature_importance(void *handle, int32_t type, float *out);
/* Write the model back as MacBoost JSON.  Replaces CAPI.swift:242-255. */
int32_t macboost_save(void *handle, const char *path, char **err);
/* Release a handle (NULL is ignored).  Replaces CAPI.swift:299-303. */
void macboost_free(void *handle);
/* Release a string returned through `err` or by macboost_warnings.
 * Replaces CAPI.swift:305-308. */
void macboost_free_string(char *s);

/* TreeSHAP feature contributions of feature-major x into out (rows x K x
 * (cols + 1) floats; per row and class the cols contributions then the
 * expected value; K = macboost_num_classes).  Replaces
 * macboost_predict_contrib, CAPI.swift:222-240 (MacBooster.predictContributions,
 * SHAP.swift:39-52): path-dependent TreeSHAP with node covers as the
 * background, evaluated on the GPU in float64 and rounded to float32; per
 * class, contributions plus expected value sum to the raw margin.  Trees
 * without covers add nothing (their expectation is not part of the bias).
 * Fails for NULL arguments, cols != num_features, a cover array whose length
 * is not the tree's node count, or a path through more than 32 distinct
 * features.  Devices as macboost_predict. */
int32_t macboost_predict_contrib(void *handle, const float *x, int64_t rows, int64_t cols,
                                 float *out, char **err);

/* Training-side entry points of the reference ABI (CAPI.swift:86-135,
 * 138-183).  This library is an inference engine: they exist so that
 * bindings written for the full ABI load it unchanged, and they fail with a
 * message ("not supported by this inference engine"). */
void *macboost_train(const char *params_json, const float *x, int64_t rows, int64_t cols,
                     int32_t row_major, const float *y, const float *w, const float *x_valid,
                     int64_t valid_rows, const float *y_valid, char **err);
int32_t macboost_select_features(const char *params_json, const float *x, int64_t rows,
                                 int64_t cols, const float *y, const float *w, int32_t rounds,
                                 int32_t trees, float alpha, int64_t seed, int32_t *out_hits,
                                 int32_t *out_decision, float *out_gain_ratio, char **err);

/* ---- additive entry points (no counterpart in the reference ABI) -------- */

enum {
  MACBOOST_KIND_PREDICT = 0, /* as macboost_predict */
  MACBOOST_KIND_RAW = 1,     /* raw fp32 margins, rows x K */
  MACBOOST_KIND_PROBA = 2,   /* predict_proba (__init__.py:433-445): rows x 2 [1-p, p] for
                                one class, softmax rows x K otherwise; evaluated in float64,
                                rounded to float32 */
  MACBOOST_KIND_LEAF = 3,    /* int32 heap index of the leaf reached, rows x num_trees */
  MACBOOST_KIND_CLI = 4      /* what `macboost predict` writes (MacBoostCLI/main.swift:344-364):
                                float32 softmax for K > 1, sigmoid for the binary objective,
                                else MACBOOST_KIND_PREDICT; rows x K */
};
enum { MACBOOST_LAYOUT_FEATURE_MAJOR = 0, MACBOOST_LAYOUT_ROW_MAJOR = 1 };

/* Visible CUDA devices (0 if none or no driver). */
int32_t macboost_device_count(void);

/* Elements per output row for `kind` (-1 for a NULL handle / unknown kind). */
int64_t macboost_output_cols(void *handle, int32_t kind);

/* Predict from host memory.  Rows are split into contiguous shards over
 * devices[0..ndev) (ndev == 0: current device), one model replica per GPU, no
 * inter-GPU communication.  `out` holds rows * macboost_output_cols(kind)
 * float32 (int32 for MACBOOST_KIND_LEAF).  Page-locked (pinned) x / out give
 * overlapped transfers. */
int32_t macboost_predict_ex(void *handle, const float *x, int64_t rows, int64_t cols,
                            int32_t layout, int32_t kind, const int32_t *devices, int32_t ndev,
                            void *out, char **err);

/* Predict from device memory on `device`, enqueued on `stream` (a
 * cudaStream_t; NULL = the legacy default stream) and returning before the
 * work completes.  Feature-major x_dev is x_dev[f * ld + i] (ld >= rows);
 * row-major x_dev is x_dev[i * cols + f] (ld ignored; this form waits for
 * completion).  16-byte aligned x_dev with ld % 4 == 0 enables bulk staging.
 * Kernel-side faults are reported by macboost_check_device.  Calls on different
 * streams may run at once: the kernel's row-chunk counters are kept per
 * (handle, device, stream), so launches that overlap must come from different
 * streams (the per-thread default stream takes a fixed chunk order instead). */
int32_t macboost_predict_device(void *handle, int32_t device, const float *x_dev, int64_t rows,
                                int64_t cols, int64_t ld, int32_t layout, int32_t kind,
                                void *out_dev, void *stream, char **err);

/* macboost_predict_contrib with a layout (MACBOOST_LAYOUT_*) and a device
 * list (ndev == 0: the current device); rows shard over the devices. */
int32_t macboost_predict_contrib_ex(void *handle, const float *x, int64_t rows, int64_t cols,
                                    int32_t layout, const int32_t *devices, int32_t ndev,
                                    float *out, char **err);

/* TreeSHAP contributions from device memory on `device`, enqueued on `stream`
 * (a cudaStream_t; NULL = legacy default stream): x_dev as in
 * macboost_predict_device, out_dev rows x K x (cols + 1) floats.  Row-major
 * input, and models whose accumulators do not fit in shared memory, make the
 * call wait for its work; otherwise kernel-side errors are reported by
 * macboost_check_device. */
int32_t macboost_predict_contrib_device(void *handle, int32_t device, const float *x_dev,
                                        int64_t rows, int64_t cols, int64_t ld, int32_t layout,
                                        float *out_dev, void *stream, char **err);

/* Upload the model to the listed devices now (otherwise done on first use). */
int32_t macboost_prepare(void *handle, const int32_t *devices, int32_t ndev, char **err);

/* Synchronise `device` and report kernel-side errors raised since the last check. */
int32_t macboost_check_device(void *handle, int32_t device, char **err);

/* Load a model from JSON text in memory (same rules as macboost_load). */
void *macboost_load_json(const char *json, int64_t len, char **err);

/* JSON description of the flattened forest and launch plan (free with
 * macboost_free_string). */
char *macboost_describe(void *handle);

/* Forest-kernel launches issued by this process so far. */
uint64_t macboost_kernel_launches(void);

/* Page-locked host allocation for inputs and outputs (NULL on failure), and
 * its release. */
void *macboost_host_alloc(int64_t bytes);
void macboost_host_free(void *p);

/* Predict from device memory without allocating any device memory.  No
 * counterpart in the reference ABI.  For callers that cannot let a library
 * call cudaMalloc: hosts that reserve (most of) the GPU's memory in their own
 * pool, where an extra allocation would fail or fragment it, and pipelines
 * where cudaMalloc/cudaFree would synchronise the device and stall other
 * streams.  Arguments as macboost_predict_device; the model must already be
 * resident on `device` (macboost_prepare, done once at set-up, allocates it).
 * The scratch it needs -- a status word and, for row-major input, a
 * feature-major copy of x_dev of at most 16 MiB (4,194,304 values,
 * round_up(rows, 4) * cols) -- is one fixed array inside the library that a
 * GPU reserves when macboost_prepare sets the model up on it (prepare looks up
 * the array's address there, which loads the library's module that holds it)
 * and keeps until the process exits; larger row-major inputs are rejected with
 * an error (split them, or pass feature-major input, which needs no copy).
 * Every call shares that array: calls that overlap on the GPU race, so
 * serialise them.  The call waits for its work on `stream` to finish and
 * reports kernel-side errors itself. */
int32_t macboost_predict_device_noalloc(void *handle, int32_t device, const float *x_dev,
                                        int64_t rows, int64_t cols, int64_t ld, int32_t layout,
                                        int32_t kind, void *out_dev, void *stream, char **err);

/* ---- text input and the `macboost predict` command (additive) ----------- */

/* Feature names stored in the model file (`featureNames`, Booster.swift:2126,
 * 2158): their count, or -1 when the file has none / for a NULL handle; and
 * name i (owned by the handle, NULL when out of range). */
int64_t macboost_num_feature_names(void *handle);
const char *macboost_feature_name(void *handle, int64_t i);

enum { MACBOOST_FORMAT_CSV = 0, MACBOOST_FORMAT_LIBSVM = 1, MACBOOST_FORMAT_AUTO = 2 };

/* Read a text table into host memory with the rules of MacBoost's CLI
 * readers.  MACBOOST_FORMAT_CSV replaces CSV.read (Sources/MacBoostCLI/
 * CSV.swift:48-118): a header row, tab-delimited when the header holds a tab
 * else comma-delimited, names trimmed of white space; blank lines and lines
 * starting with '\r' skipped; each field read with strtof in place, empty or
 * non-numeric fields NaN; extra fields ignored; a row with fewer fields than
 * the header fails ("Malformed CSV: row N has fewer fields than the header
 * (C)", N the first such data row, from 1).  MACBOOST_FORMAT_LIBSVM replaces
 * CSV.readLibSVM (CSV.swift:126-217): "label idx:value ..." lines, '#'
 * comments, non-"idx:" tokens (qid:...) skipped, 0- or 1-based indices
 * detected from the smallest index, absent features 0, columns named
 * label,f0,f1,...; a negative index fails.  MACBOOST_FORMAT_AUTO picks LibSVM
 * for the .svm / .libsvm extensions (MacBoostCLI/main.swift:98-110).
 * Returns a table handle (release with macboost_table_free) or NULL. */
void *macboost_table_read(const char *path, int32_t format, char **err);
int64_t macboost_table_rows(void *table);
int64_t macboost_table_cols(void *table);
/* Name of column `col` (owned by the table; NULL when out of range). */
const char *macboost_table_column_name(void *table, int64_t col);
/* The values, row-major rows x cols float32 (owned by the table). */
const float *macboost_table_data(void *table);
void macboost_table_free(void *table);

/* Write a prediction file as the CLI does: CSV.writePredictions
 * (CSV.swift:219-224) for k == 1 (header "prediction", one value per line),
 * else the multiclass branch of runPredict (main.swift:357-361, header
 * class_0,...,class_{k-1}, one comma-separated row per line).  Values are
 * printed as Swift prints a Float: shortest round-trip digits, exponent form
 * ("1e-05", "1.2345679e+08") below 1e-4 or above 2^24, else positional with
 * at least one fractional digit ("1.0", "0.25"); "nan", "inf", "-inf".
 * The file is written beside `path` and renamed over it. */
int32_t macboost_write_predictions(const float *preds, int64_t rows, int64_t k, const char *path,
                                   char **err);

/* `macboost predict --model M --data D --output O [--raw]`: replaces runPredict,
 * MacBoostCLI/main.swift:317-371, on this engine.  Reads `data_path`
 * (`format` as macboost_table_read; the reference reads CSV/TSV), maps the
 * model's features to columns by name when the model stores names, else takes
 * the first num_features columns; predicts on devices[0..ndev) (ndev == 0:
 * MACBOOST_DEVICES, else the current device); writes MACBOOST_KIND_CLI
 * output, or MACBOOST_KIND_PREDICT when `raw` is non-zero, to `output_path`
 * with macboost_write_predictions; stores the row count in *rows_out.  Errors
 * use the reference's messages ("Malformed CSV: column 'x' required by the
 * model is missing", "model expects N features, CSV has C columns", the
 * reader's), reported after the whole file has been read. */
int32_t macboost_cli_predict(void *handle, const char *data_path, int32_t format, int32_t raw,
                             const int32_t *devices, int32_t ndev, const char *output_path,
                             int64_t *rows_out, char **err);

/* ---- binned data: the trainer's side of the path (additive) ------------ */

/* Bin raw values into the trainer's tiled layout on `device`.  Replaces the
 * bin_data kernel, Sources/MacBoost/Shaders.swift:41-76.  Layout of `bins`
 * (bin_index, Shaders.swift:37-39): ceil(cols / 8) tiles of 8 features; bin
 * (f, i) at (f / 8) * rows * 8 + i * 8 + f % 8; padding features are 0.  A
 * NaN goes to the missing bin num_bins - 1; a categorical feature
 * (categorical[f] == 1; NULL: none) to clamp(rint(v), 0, num_bins - 2); a
 * numeric one to the first of its num_bins - 2 upper edges (edges[f *
 * (num_bins - 2) + k], ascending) that is >= v, or num_bins - 2.  x is
 * feature-major x[f * rows + i] (layout 0) or row-major (layout 1), host
 * memory. */
int32_t macboost_bin_data(const float *x, int64_t rows, int64_t cols, int32_t layout,
                          const float *edges, int32_t num_bins, const uint8_t *categorical,
                          int32_t device, uint8_t *bins, char **err);

/* macboost_bin_data on device memory, enqueued on `stream` (a cudaStream_t;
 * NULL = legacy default stream) without waiting: x, edges, categorical (cols
 * flags, required) and bins are device pointers; feature-major x is x[f * ld
 * + i] with ld >= rows; row-major x ignores ld. */
int32_t macboost_bin_data_device(const float *x, int64_t rows, int64_t cols, int64_t ld,
                                 int32_t layout, const float *edges, int32_t num_bins,
                                 const uint8_t *categorical, int32_t device, uint8_t *bins,
                                 void *stream, char **err);

/* Walk trees in the trainer's split form over binned rows.  Replaces
 * predict_tree_binned and assign_leaves, Shaders.swift:1741-1781, for
 * num_trees trees at once (one call per finished tree reproduces the
 * reference's per-iteration use).  Tree t owns nodes tree_offsets[t] ..
 * tree_offsets[t + 1] - 1 (implicit heap, children 2n+1 / 2n+2); per node
 * split_feature (< 0: leaf), split_bin, split_flags (bit0 missing goes left,
 * bit1 categorical) and 8 cat_mask words; leaf_values per node.  A row goes
 * left when its bin is set in the mask (categorical), else when it is the
 * missing bin and bit0 is set, else when bin <= split_bin; at most max_depth
 * splits are taken.  preds (class-major, num_classes x rows, NULL: none) gets
 * preds[(t % num_classes) * rows + i] += leaf, tree after tree, in float32;
 * leaf_idx (tree-major, num_trees x rows, NULL: none) the final heap index.
 * Host memory, on `device`.  A split that names a feature >= cols or a child
 * outside its tree fails the call. */
int32_t macboost_predict_tree_binned(const uint8_t *bins, int64_t rows, int64_t cols,
                                     int32_t num_bins, int32_t num_trees,
                                     const int64_t *tree_offsets, const int32_t *split_feature,
                                     const uint32_t *split_bin, const uint32_t *split_flags,
                                     const uint32_t *cat_mask, const float *leaf_values,
                                     int32_t max_depth, int32_t num_classes, int32_t device,
                                     float *preds, int32_t *leaf_idx, char **err);

/* The same with every array in device memory, enqueued on `stream` (a
 * cudaStream_t; NULL = legacy default stream) without waiting: the form a
 * GPU training loop calls once per tree.  A bad split ORs 2 into the
 * device word *status instead of failing the call. */
int32_t macboost_predict_tree_binned_device(
    const uint8_t *bins, int64_t rows, int64_t cols, int32_t num_bins, int32_t num_trees,
    const int64_t *tree_offsets, const int32_t *split_feature, const uint32_t *split_bin,
    const uint32_t *split_flags, const uint32_t *cat_mask, const float *leaf_values,
    int32_t max_depth, int32_t num_classes, int32_t device, float *preds, int32_t *leaf_idx,
    uint32_t *status, void *stream, char **err);

/* Load a MacBoost binned dataset (.mbds).  Replaces BinnedDataset.load,
 * Sources/MacBoost/Dataset.swift:41-83 (little-endian "MBDS", version 1,
 * tile width 8; the same "Invalid input: ..." messages).  Returns a handle
 * (macboost_dataset_free) or NULL.  Getters return -1 / NULL for a NULL
 * handle; arrays are owned by the handle. */
void *macboost_dataset_load(const char *path, char **err);
int64_t macboost_dataset_rows(void *dataset);
int64_t macboost_dataset_cols(void *dataset);
int32_t macboost_dataset_num_bins(void *dataset);
const uint8_t *macboost_dataset_bins(void *dataset);  /* tiled, as macboost_bin_data */
const float *macboost_dataset_edges(void *dataset);   /* cols x (num_bins - 2) */
const float *macboost_dataset_labels(void *dataset);  /* rows */
int64_t macboost_dataset_num_categorical(void *dataset);
int64_t macboost_dataset_categorical(void *dataset, int64_t i);
int64_t macboost_dataset_num_feature_names(void *dataset); /* -1 when the file has none */
const char *macboost_dataset_feature_name(void *dataset, int64_t i);
void macboost_dataset_free(void *dataset);

/* Bin a feature matrix into a dataset handle on `device`.  Replaces
 * MacBooster.makeDataset, Sources/MacBoost/Booster.swift:392-434: the same
 * checks and messages in the same order (numBins in 4...256 as
 * MacBooster(params:), Booster.swift:263-265; shapes; finite labels;
 * categorical ids, Booster.swift:1810-1826, features in ascending order),
 * the same quantile edges (Binner.computeEdges, Sources/MacBoost/
 * Binner.swift:25-60: every max(1, rows / 200000)-th non-NaN value, sorted,
 * edge k = sample[min(m - 1, (k + 1) * m / (num_bins - 1))]; zeros for
 * categorical and all-NaN features) and macboost_bin_data for the bins.  x
 * is feature-major x[f * rows + i] and labels[rows], host memory;
 * categorical lists n_categorical feature indices; feature_names holds cols
 * strings, or NULL for a dataset without names.  Returns a handle
 * (macboost_dataset_free) or NULL. */
void *macboost_dataset_make(const float *x, int64_t rows, int64_t cols, const float *labels,
                            int32_t num_bins, const int64_t *categorical, int64_t n_categorical,
                            const char *const *feature_names, int32_t device, char **err);

/* Write a dataset to `path` in MacBoost's .mbds format.  Replaces
 * BinnedDataset.save, Sources/MacBoost/Dataset.swift:26-39 (byte for byte:
 * little-endian header, sorted categorical indices, feature names as
 * JSONEncoder's compact array, then edges, labels and bins with u64
 * counts). */
int32_t macboost_dataset_save(void *dataset, const char *path, char **err);

/* `macboost dataset`: runDataset, Sources/MacBoostCLI/main.swift:134-154.
 * Reads `data_path` (`format` as macboost_table_read), takes the column
 * named `label` (NULL: "label") as labels and every other column as a
 * feature, marks the comma-separated feature names in `categorical` (NULL:
 * none), bins with num_bins on `device` and writes `output_path`; stores the
 * row and feature counts.  Errors use the reference's messages ("label
 * column 'y' not found; columns: a, b", "categorical column 'c' not found
 * among features", the reader's and makeDataset's). */
int32_t macboost_cli_dataset(const char *data_path, int32_t format, const char *label,
                             const char *categorical, int32_t num_bins, int32_t device,
                             const char *output_path, int64_t *rows_out, int64_t *cols_out,
                             char **err);

/* A model's output of `kind` (MACBOOST_KIND_*) on every row of a binned
 * dataset, rows sharded over devices[0..ndev) (ndev == 0: MACBOOST_DEVICES,
 * else the current device); `out` as macboost_predict_ex.  Each numeric
 * threshold is mapped to the bin edge it was trained at (the trainer writes
 * threshold = edges[f * (numBins - 2) + bin], Booster.swift:938), so rows
 * route exactly as macboost_predict_ex routes the values they were binned
 * from (categorical ids inside 0..numBins-2).  Fails when a threshold is no
 * edge of the dataset or the model's numFeatures / numBins differ. */
int32_t macboost_predict_dataset(void *handle, void *dataset, int32_t kind,
                                 const int32_t *devices, int32_t ndev, void *out, char **err);

#ifdef __cplusplus
}
#endif

#endif /* MACBOOST_C_H */
