// Text tables and prediction files of MacBoost's command line interface.
//
// Host-side readers for the on-disk input formats of `macboost predict`:
// headered CSV / TSV (Sources/MacBoostCLI/CSV.swift:48-118) and LibSVM sparse
// text (CSV.swift:126-217), the prediction-file writer (CSV.swift:219-224,
// main.swift:349-364) with Swift's shortest round-trip float text, and the
// predict command itself (main.swift:317-371) on the GPU engine.
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace mb {

struct Engine;

enum TableFormat : int32_t { kFormatCsv = 0, kFormatLibsvm = 1, kFormatAuto = 2 };

// A parsed table: `columns` (indices into `header`) of `rows` data rows,
// row-major float32 in `data` (page-locked when the CUDA runtime could pin
// it, else ordinary heap memory).
struct Table {
  std::vector<std::string> header;  // every column name of the file, in file order
  std::vector<int64_t> columns;     // file columns held, in order (repeats allowed)
  int64_t rows = 0;
  float* data = nullptr;
  bool pinned = false;

  Table() = default;
  Table(const Table&) = delete;
  Table& operator=(const Table&) = delete;
  ~Table();
  int64_t width() const { return int64_t(columns.size()); }
};

// Picks the held columns once the header is known; an empty function holds
// every column.  It may return an empty list (parse and validate only).
using ColumnChooser = std::function<std::vector<int64_t>(const std::vector<std::string>&)>;

// strtof (C locale) with a fast exact path for plain decimal numbers; the
// result and end pointer always equal strtof's.
float parse_f32(const char* s, char** end);

// CSV.read / CSV.readLibSVM on a file; `format` kFormatAuto picks LibSVM for
// the .svm / .libsvm extensions (main.swift:98-110).
bool read_table(const char* path, int format, const ColumnChooser& choose, bool pin, Table& t,
                std::string& err);

// Swift's `Float.description`: shortest round-trip digits, "nan", "inf".
// `out` holds at least 32 bytes; returns the length written (no NUL).
size_t format_float(float v, char* out);

// CSV.writePredictions / the multiclass branch of runPredict: a header line
// ("prediction", or class_0..class_{k-1} when k > 1), then one row per line.
bool write_predictions(const float* p, int64_t rows, int64_t k, const char* path,
                       std::string& err);

// runPredict (main.swift:317-371): read `data_path`, map the model's features
// to columns by name (or take the first num_features columns), predict on
// `devices`, apply the CLI transform unless `raw`, write `output_path`.
bool cli_predict(Engine& e, const char* data_path, int format, bool raw,
                 const std::vector<int>& devices, const char* output_path, int64_t* rows_out,
                 std::string& err);

}  // namespace mb
