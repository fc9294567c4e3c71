// `macboost` command line front end of the B200 inference engine.
//
// Mirrors the inference-side commands of MacBoost's CLI (Sources/MacBoostCLI/
// main.swift): `predict` (runPredict, :317-371), `dataset` (runDataset,
// :134-154), `importance` (:378-397), `version` and `help`, with the same flag syntax (parseFlags, :82-96), the
// same output files and messages, and exit status 1 with "error: ..." on
// stderr for every failure.  It uses only the C ABI of libmacboostc.so.
#include <algorithm>
#include <chrono>
#include <climits>
#include <cstdio>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/macboost_c.h"

namespace {

const char* kUsage =
    "macboost -- MacBoost model inference on NVIDIA B200 GPUs\n"
    "\n"
    "USAGE:\n"
    "  macboost predict --model <model.json> --data <test.csv> [options]\n"
    "  macboost dataset --data <train.csv> --output <train.mbds> [options]\n"
    "  macboost importance --model <model.json>\n"
    "  macboost version\n"
    "\n"
    "PREDICT OPTIONS:\n"
    "  --model <path>     MacBoost JSON model                          [required]\n"
    "  --data <path>      input table; columns are matched to the model's feature\n"
    "                     names, else the first numFeatures columns are used [required]\n"
    "  --output <path>    predictions CSV                        [default: predictions.csv]\n"
    "  --raw              raw scores: no sigmoid (binary) or softmax (multiclass)\n"
    "  --format <f>       csv | tsv | libsvm | auto (libsvm for .svm/.libsvm)\n"
    "                     [default: csv; the delimiter is sniffed from the header]\n"
    "  --devices <list>   GPUs to shard rows over, e.g. 0,1,2,3\n"
    "                     [default: MACBOOST_DEVICES, else the current GPU]\n"
    "\n"
    "DATASET OPTIONS (a binned .mbds file, as MacBoost's trainer reads it):\n"
    "  --data <path>      training table                                 [required]\n"
    "  --output <path>    .mbds file to write                            [required]\n"
    "  --label <name>     label column name                        [default: label]\n"
    "  --bins <n>         histogram bins incl. missing bin (4-256)   [default: 256]\n"
    "  --categorical <cols>  comma-separated categorical column names\n"
    "  --format <f>       csv | tsv | libsvm | auto              [default: auto]\n"
    "  --device <n>       GPU that bins the values\n"
    "                     [default: first of MACBOOST_DEVICES, else 0]\n"
    "\n"
    "Empty fields and non-numeric tokens (NA, nan, ...) are missing values and\n"
    "follow each split's learned default direction.  Training (`train`) is not\n"
    "part of this inference engine.\n";

[[noreturn]] void fail(const std::string& message) {
  std::fprintf(stderr, "error: %s\n", message.c_str());
  std::exit(1);
}

std::string take_error(char* e) {
  std::string s = e ? e : "unknown error";
  macboost_free_string(e);
  return s;
}

// parseFlags (main.swift:82-96): "--key value" pairs, boolean --raw / --goss
// / --feature-selection.
std::map<std::string, std::string> parse_flags(int argc, char** argv, int first) {
  std::map<std::string, std::string> out;
  for (int i = first; i < argc;) {
    const std::string a = argv[i];
    if (a.compare(0, 2, "--") != 0) fail("unexpected argument '" + a + "'");
    const std::string key = a.substr(2);
    if (key == "raw" || key == "goss" || key == "feature-selection") {
      out[key] = "1";
      ++i;
      continue;
    }
    if (i + 1 >= argc) fail("missing value for --" + key);
    out[key] = argv[i + 1];
    i += 2;
  }
  return out;
}

void* load_model(const std::string& path) {
  char* e = nullptr;
  void* h = macboost_load(path.c_str(), &e);
  if (!h) fail(take_error(e));
  return h;
}

std::vector<int32_t> parse_devices(const std::string& s) {
  std::vector<int32_t> d;
  const char* p = s.c_str();
  while (*p) {
    char* end = nullptr;
    const long v = std::strtol(p, &end, 10);
    if (end == p || v < 0) fail("--devices expects a comma-separated list of GPU indices");
    d.push_back(int32_t(v));
    p = end;
    while (*p == ',' || *p == ' ') ++p;
  }
  return d;
}

// --format values of loadTable (main.swift:98-110).
int32_t parse_format(const std::string& f) {
  if (f == "csv" || f == "tsv") return MACBOOST_FORMAT_CSV;
  if (f == "libsvm") return MACBOOST_FORMAT_LIBSVM;
  if (f == "auto") return MACBOOST_FORMAT_AUTO;
  fail("unknown --format '" + f + "' (auto | csv | tsv | libsvm)");
}

// Swift's Int(String): optional sign, then decimal digits only, in range.
bool parse_swift_int(const std::string& s, long long* v) {
  size_t i = (!s.empty() && (s[0] == '+' || s[0] == '-')) ? 1 : 0;
  if (i == s.size()) return false;
  for (size_t j = i; j < s.size(); ++j)
    if (s[j] < '0' || s[j] > '9') return false;
  errno = 0;
  *v = std::strtoll(s.c_str(), nullptr, 10);
  return errno == 0;
}

int run_predict(const std::map<std::string, std::string>& flags) {
  auto get = [&](const char* k) -> const std::string* {
    auto it = flags.find(k);
    return it == flags.end() ? nullptr : &it->second;
  };
  const std::string* model = get("model");
  if (!model) fail("--model is required");
  const std::string* data = get("data");
  if (!data) fail("--data is required");
  const std::string output = get("output") ? *get("output") : "predictions.csv";
  int32_t format = MACBOOST_FORMAT_CSV;
  if (const std::string* f = get("format")) format = parse_format(*f);
  std::vector<int32_t> devices;
  if (const std::string* d = get("devices")) devices = parse_devices(*d);
  void* h = load_model(*model);
  char* e = nullptr;
  int64_t rows = 0;
  if (macboost_cli_predict(h, data->c_str(), format, get("raw") ? 1 : 0,
                           devices.empty() ? nullptr : devices.data(), int32_t(devices.size()),
                           output.c_str(), &rows, &e) != 0) {
    const std::string msg = take_error(e);
    macboost_free(h);
    fail(msg);
  }
  macboost_free(h);
  std::printf("wrote %lld predictions to %s\n", static_cast<long long>(rows), output.c_str());
  return 0;
}

// `macboost dataset` (runDataset, main.swift:134-154).
int run_dataset(const std::map<std::string, std::string>& flags) {
  auto get = [&](const char* k) -> const std::string* {
    auto it = flags.find(k);
    return it == flags.end() ? nullptr : &it->second;
  };
  const std::string* data = get("data");
  if (!data) fail("--data is required");
  const std::string* output = get("output");
  if (!output) fail("--output is required (e.g. train.mbds)");
  long long bins = 256;
  if (const std::string* b = get("bins"))
    if (!parse_swift_int(*b, &bins)) bins = 256;
  const int32_t format = get("format") ? parse_format(*get("format")) : MACBOOST_FORMAT_AUTO;
  int32_t device = 0;
  if (const std::string* d = get("device")) {
    const std::vector<int32_t> v = parse_devices(*d);
    if (v.size() != 1) fail("--device expects one GPU index");
    device = v[0];
  } else if (const char* env = std::getenv("MACBOOST_DEVICES")) {
    const std::vector<int32_t> v = parse_devices(env);
    if (!v.empty()) device = v[0];
  }
  const auto t0 = std::chrono::steady_clock::now();
  // out-of-range counts reach the library as an out-of-range int32; the
  // message then names the value given
  const int32_t nb = int32_t(std::clamp<long long>(bins, INT_MIN, INT_MAX));
  char* e = nullptr;
  int64_t rows = 0, cols = 0;
  if (macboost_cli_dataset(data->c_str(), format, get("label") ? get("label")->c_str() : nullptr,
                           get("categorical") ? get("categorical")->c_str() : nullptr, nb,
                           device, output->c_str(), &rows, &cols, &e) != 0) {
    std::string msg = take_error(e);
    const std::string clamped = "got " + std::to_string(nb);
    if (nb != bins && msg.size() >= clamped.size() &&
        msg.compare(msg.size() - clamped.size(), clamped.size(), clamped) == 0)
      msg = msg.substr(0, msg.size() - clamped.size()) + "got " + std::to_string(bins);
    fail(msg);
  }
  const double secs =
      std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::printf("binned %lld rows x %lld features into %s in %.2fs\n", static_cast<long long>(rows),
              static_cast<long long>(cols), output->c_str(), secs);
  return 0;
}

// Pads to `w` characters (UTF-8 code points) with trailing blanks.
std::string pad(const std::string& s, size_t w) {
  size_t n = 0;
  for (unsigned char c : s) n += (c >> 6) != 2;
  return n >= w ? s : s + std::string(w - n, ' ');
}

// `macboost importance` (main.swift:378-397): features by gain, descending.
int run_importance(const std::map<std::string, std::string>& flags) {
  auto it = flags.find("model");
  if (it == flags.end()) fail("--model is required");
  void* h = load_model(it->second);
  const int64_t F = macboost_num_features(h);
  std::vector<float> gain(size_t(std::max<int64_t>(F, 0))), split(gain.size());
  if (F > 0 && (macboost_feature_importance(h, 0, gain.data()) != 0 ||
                macboost_feature_importance(h, 1, split.data()) != 0))
    fail("feature importance failed");
  const int64_t nn = macboost_num_feature_names(h);
  std::vector<std::string> names;
  for (int64_t i = 0; i < F; ++i) {
    const char* n = i < nn ? macboost_feature_name(h, i) : nullptr;
    names.push_back(n ? n : "f" + std::to_string(i));
  }
  std::vector<int64_t> order(static_cast<size_t>(F));
  for (int64_t i = 0; i < F; ++i) order[size_t(i)] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int64_t a, int64_t b) { return gain[size_t(a)] > gain[size_t(b)]; });
  std::printf("%s\n", (pad("feature", 24) + pad("gain", 14) + "splits").c_str());
  char g[64], s[64];
  for (int64_t i : order) {
    std::snprintf(g, sizeof(g), "%.1f", double(gain[size_t(i)]));
    std::snprintf(s, sizeof(s), "%.0f", double(split[size_t(i)]));
    std::printf("%s\n", (pad(names[size_t(i)], 24) + pad(g, 14) + s).c_str());
  }
  macboost_free(h);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  const std::string cmd = argc > 1 ? argv[1] : "";
  if (cmd == "predict") return run_predict(parse_flags(argc, argv, 2));
  if (cmd == "importance") return run_importance(parse_flags(argc, argv, 2));
  if (cmd == "dataset") return run_dataset(parse_flags(argc, argv, 2));
  if (cmd == "train") fail("`macboost train` is not supported by this inference engine");
  if (cmd == "--version" || cmd == "version") {
    std::printf("macboost 1.0.0\n");
    return 0;
  }
  if (argc < 2 || cmd == "--help" || cmd == "-h" || cmd == "help") {
    std::printf("%s\n", kUsage);
    return 0;
  }
  fail("unknown command '" + cmd + "' — expected train or predict (see macboost --help)");
}
