// MacBoost model file: parsing, validation and serialisation.
//
// The file format is MacBoost's `ModelFile` (Sources/MacBoost/Booster.swift:2119-2130)
// holding implicit-heap `Tree`s (Booster.swift:119-146).  Loading follows
// `MacBooster.load` (Booster.swift:2144-2162) and `PyModel.__init__`
// (python/macboost/_pyinfer.py:22-46).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace mb {

constexpr uint32_t kFlagDefaultLeft = 1u;  // Booster.swift:148
constexpr uint32_t kFlagCategorical = 2u;  // Booster.swift:149

// Objective raw values, Booster.swift:5-13.
enum Objective : int32_t {
  kRegression = 0,
  kBinaryLogistic = 1,
  kMAE = 2,
  kHuber = 3,
  kQuantile = 4,
  kPoisson = 5,
  kTweedie = 6,
  kMulticlass = 7,
};

struct Tree {
  std::vector<int32_t> feature;    // < 0 marks a leaf
  std::vector<float> threshold;    // go left if x <= threshold
  std::vector<float> leaf;         // leaf values (learning rate applied)
  std::vector<uint8_t> flags;      // bit0 default-left, bit1 categorical
  std::vector<uint32_t> cat_mask;  // 8 words per node, or empty
  std::vector<float> gain;         // optional
  std::vector<float> cover;        // optional
  int32_t depth = 0;               // deepest reachable leaf (root = 0)
};

struct Model {
  int32_t version = 1;
  int32_t objective = 0;
  int32_t num_bins = 256;
  float base_score = 0.f;
  int64_t num_features = 0;
  std::vector<int64_t> categorical;
  bool has_feature_names = false;
  std::vector<std::string> feature_names;
  std::vector<Tree> trees;
  bool has_num_classes = false;
  int64_t num_classes_file = 0;    // value stored in the file (if any)
  bool has_base_scores = false;
  std::vector<float> base_scores_file;

  // Derived at load.
  int32_t K = 1;                   // classes scored (trainedNumClasses)
  std::vector<float> base_scores;  // K starting margins
  int32_t max_depth = 0;           // over all trees
  bool any_cat = false;            // any reachable categorical node with a mask
  int64_t reachable_nodes = 0;

  bool uses_log_link() const { return objective == kPoisson || objective == kTweedie; }
};

// Parse and validate a model file.  Returns false and sets `err` on failure.
bool load_model_file(const std::string& path, Model& m, std::string& err);
bool parse_model_json(const char* text, size_t len, Model& m, std::string& err);

// A JSON array of strings (feature-name lists).
bool parse_json_string_array(const char* text, size_t len, std::vector<std::string>& out,
                             std::string& err);

// Serialise back to MacBoost JSON (ModelFile keys, Booster.swift:2132-2142).
std::string model_to_json(const Model& m);

}  // namespace mb
