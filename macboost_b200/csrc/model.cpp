// MacBoost model file loader (see model.h for the format references).
//
// A schema-directed recursive-descent JSON reader: numeric arrays are parsed
// straight into typed vectors, so multi-megabyte forests (500 leaf-wise trees
// of 8,191 heap slots) load without building a document tree.
//
// Number conversion matches the reference readers: JSON numbers are parsed to
// the nearest float64 (std::from_chars, locale independent) and rounded to
// float32, as PyModel does through json.load + np.asarray(dtype=float32)
// (_pyinfer.py:36-39).  Values that overflow float32 are rejected, as Swift's
// JSONDecoder rejects them for `Float` fields; NaN / Infinity literals are not
// JSON and are rejected too.
#include "model.h"

#include <algorithm>
#include <cerrno>
#include <charconv>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string_view>

namespace mb {
namespace {

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Reader {
 public:
  Reader(const char* p, size_t n) : beg_(p), p_(p), end_(p + n) {}

  [[noreturn]] void fail(const std::string& what) const {
    throw ParseError("malformed model JSON at byte " + std::to_string(p_ - beg_) + ": " + what);
  }

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool at(char c) {
    ws();
    return p_ < end_ && *p_ == c;
  }
  void expect(char c) {
    ws();
    if (p_ >= end_ || *p_ != c) fail(std::string("expected '") + c + "'");
    ++p_;
  }
  bool eat(char c) {
    if (at(c)) {
      ++p_;
      return true;
    }
    return false;
  }
  bool eof() {
    ws();
    return p_ >= end_;
  }

  bool null_literal() {
    ws();
    if (end_ - p_ >= 4 && std::memcmp(p_, "null", 4) == 0) {
      p_ += 4;
      return true;
    }
    return false;
  }

  std::string str() {
    expect('"');
    std::string s;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      char c = *p_++;
      if (c == '"') break;
      if (c == '\\') {
        if (p_ >= end_) fail("bad escape");
        char e = *p_++;
        switch (e) {
          case '"': s += '"'; break;
          case '\\': s += '\\'; break;
          case '/': s += '/'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            if (end_ - p_ < 4) fail("bad \\u escape");
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p_++;
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= unsigned(h - '0');
              else if (h >= 'a' && h <= 'f') cp |= unsigned(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') cp |= unsigned(h - 'A' + 10);
              else fail("bad \\u escape");
            }
            if (cp >= 0xD800 && cp <= 0xDBFF && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
              unsigned lo = 0;
              for (int i = 2; i < 6; ++i) {
                char h = p_[i];
                lo <<= 4;
                if (h >= '0' && h <= '9') lo |= unsigned(h - '0');
                else if (h >= 'a' && h <= 'f') lo |= unsigned(h - 'a' + 10);
                else if (h >= 'A' && h <= 'F') lo |= unsigned(h - 'A' + 10);
              }
              if (lo >= 0xDC00 && lo <= 0xDFFF) {
                p_ += 6;
                cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
              }
            }
            if (cp < 0x80) {
              s += char(cp);
            } else if (cp < 0x800) {
              s += char(0xC0 | (cp >> 6));
              s += char(0x80 | (cp & 0x3F));
            } else if (cp < 0x10000) {
              s += char(0xE0 | (cp >> 12));
              s += char(0x80 | ((cp >> 6) & 0x3F));
              s += char(0x80 | (cp & 0x3F));
            } else {
              s += char(0xF0 | (cp >> 18));
              s += char(0x80 | ((cp >> 12) & 0x3F));
              s += char(0x80 | ((cp >> 6) & 0x3F));
              s += char(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        s += c;
      }
    }
    return s;
  }

  // Scan one JSON number token; returns [begin, end) and whether it is an
  // integer literal (no fraction / exponent).
  std::string_view number_token(bool& integral) {
    ws();
    const char* b = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) fail("expected a number");
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    integral = true;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) fail("bad number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) fail("bad exponent");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    return std::string_view(b, size_t(p_ - b));
  }

  double f64() {
    bool integral;
    std::string_view t = number_token(integral);
    double v = 0;
    auto r = std::from_chars(t.data(), t.data() + t.size(), v);
    if (r.ec == std::errc::result_out_of_range) {
      // from_chars reports overflow / underflow; underflow to a subnormal or
      // zero is a valid value, overflow is not representable.
      char* e = nullptr;
      std::string tmp(t);
      v = std::strtod(tmp.c_str(), &e);
      if (std::isinf(v)) fail("number " + tmp + " does not fit in Float");
    } else if (r.ec != std::errc()) {
      fail("bad number");
    }
    return v;
  }

  float f32() {
    const char* b = p_;
    double d = f64();
    float f = static_cast<float>(d);
    if (std::isinf(f)) {
      p_ = b;
      ws();
      fail("number does not fit in Float");
    }
    return f;
  }

  int64_t i64(int64_t lo, int64_t hi, const char* what) {
    bool integral;
    const char* b = p_;
    std::string_view t = number_token(integral);
    int64_t v = 0;
    if (integral) {
      auto r = std::from_chars(t.data(), t.data() + t.size(), v);
      if (r.ec != std::errc()) {
        p_ = b;
        fail(std::string(what) + " out of range");
      }
    } else {
      // Accept integral values written as decimals (1.0, 1e2), as numpy does.
      double d = 0;
      std::from_chars(t.data(), t.data() + t.size(), d);
      if (!(d == std::floor(d)) || d < -9.2e18 || d > 9.2e18) {
        p_ = b;
        fail(std::string(what) + " must be an integer");
      }
      v = static_cast<int64_t>(d);
    }
    if (v < lo || v > hi) {
      p_ = b;
      fail(std::string(what) + " out of range");
    }
    return v;
  }

  template <class Fn>
  void array(Fn&& fn) {
    expect('[');
    if (eat(']')) return;
    do {
      fn();
    } while (eat(','));
    expect(']');
  }

  template <class Fn>
  void object(Fn&& fn) {
    expect('{');
    if (eat('}')) return;
    do {
      std::string key = str();
      expect(':');
      fn(key);
    } while (eat(','));
    expect('}');
  }

  void skip() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    char c = *p_;
    if (c == '{') {
      object([&](const std::string&) { skip(); });
    } else if (c == '[') {
      array([&] { skip(); });
    } else if (c == '"') {
      str();
    } else if (c == 't' && end_ - p_ >= 4 && std::memcmp(p_, "true", 4) == 0) {
      p_ += 4;
    } else if (c == 'f' && end_ - p_ >= 5 && std::memcmp(p_, "false", 5) == 0) {
      p_ += 5;
    } else if (null_literal()) {
    } else {
      bool integral;
      number_token(integral);
    }
  }

 private:
  const char* beg_;
  const char* p_;
  const char* end_;
};

template <class T>
void read_int_array(Reader& r, std::vector<T>& out, int64_t lo, int64_t hi, const char* what) {
  out.clear();
  r.array([&] { out.push_back(static_cast<T>(r.i64(lo, hi, what))); });
}

void read_f32_array(Reader& r, std::vector<float>& out) {
  out.clear();
  r.array([&] { out.push_back(r.f32()); });
}

void read_tree(Reader& r, Tree& t) {
  bool has_f = false, has_t = false, has_l = false, has_fl = false;
  r.object([&](const std::string& key) {
    if (key == "feature") {
      read_int_array(r, t.feature, INT32_MIN, INT32_MAX, "feature index");
      has_f = true;
    } else if (key == "threshold") {
      read_f32_array(r, t.threshold);
      has_t = true;
    } else if (key == "leaf") {
      read_f32_array(r, t.leaf);
      has_l = true;
    } else if (key == "flags") {
      read_int_array(r, t.flags, 0, 255, "flags");
      has_fl = true;
    } else if (key == "catMask") {
      if (!r.null_literal()) read_int_array(r, t.cat_mask, 0, UINT32_MAX, "catMask word");
    } else if (key == "gain") {
      if (!r.null_literal()) read_f32_array(r, t.gain);
    } else if (key == "cover") {
      if (!r.null_literal()) read_f32_array(r, t.cover);
    } else {
      r.skip();
    }
  });
  if (!(has_f && has_t && has_l && has_fl))
    r.fail("tree lacks one of feature / threshold / leaf / flags");
}

// Validate one tree and compute its depth.  Only nodes the walk can reach are
// checked, because the reference walks (_pyinfer.py:62-70,
// Booster.swift:2047-2067) never touch the others.
void validate_tree(Tree& t, size_t ti, const Model& m, bool& any_cat, int64_t& reach) {
  const size_t n = t.feature.size();
  auto where = [&] { return "tree " + std::to_string(ti) + ": "; };
  if (n == 0) throw ParseError(where() + "empty tree");
  if (t.threshold.size() != n || t.leaf.size() != n || t.flags.size() != n)
    throw ParseError(where() + "feature/threshold/leaf/flags lengths differ");
  if (!t.cat_mask.empty() && t.cat_mask.size() != 8 * n)
    throw ParseError(where() + "catMask must hold 8 words per node");
  int32_t depth = 0;
  std::vector<std::pair<int64_t, int32_t>> stack{{0, 0}};
  while (!stack.empty()) {
    auto [i, d] = stack.back();
    stack.pop_back();
    ++reach;
    if (t.feature[i] < 0) {
      depth = std::max(depth, d);
      continue;
    }
    if (t.feature[i] >= m.num_features)
      throw ParseError(where() + "node " + std::to_string(i) + " splits on feature " +
                       std::to_string(t.feature[i]) + " but the model has " +
                       std::to_string(m.num_features) + " features");
    if (2 * i + 2 >= int64_t(n))
      throw ParseError(where() + "node " + std::to_string(i) +
                       " has children outside the tree (length " + std::to_string(n) + ")");
    if ((t.flags[i] & kFlagCategorical) && !t.cat_mask.empty()) any_cat = true;
    if (d + 1 > 62) throw ParseError(where() + "tree deeper than 62 levels");
    stack.push_back({2 * i + 2, d + 1});
    stack.push_back({2 * i + 1, d + 1});
  }
  t.depth = depth;
}

}  // namespace

bool parse_model_json(const char* text, size_t len, Model& m, std::string& err) {
  m = Model();
  try {
    Reader r(text, len);
    bool has_version = false, has_obj = false, has_bins = false, has_base = false,
         has_nf = false, has_trees = false;
    int64_t version = 0, objective = 0, bins = 0;
    r.object([&](const std::string& key) {
      if (key == "version") {
        version = r.i64(INT64_MIN, INT64_MAX, "version");
        has_version = true;
      } else if (key == "objective") {
        objective = r.i64(INT64_MIN, INT64_MAX, "objective");
        has_obj = true;
      } else if (key == "numBins") {
        bins = r.i64(INT64_MIN, INT64_MAX, "numBins");
        has_bins = true;
      } else if (key == "baseScore") {
        m.base_score = r.f32();
        has_base = true;
      } else if (key == "numFeatures") {
        m.num_features = r.i64(0, (int64_t(1) << 27) - 1, "numFeatures");
        has_nf = true;
      } else if (key == "categorical") {
        if (!r.null_literal()) read_int_array(r, m.categorical, INT64_MIN, INT64_MAX, "categorical");
      } else if (key == "featureNames") {
        if (!r.null_literal()) {
          m.has_feature_names = true;
          r.array([&] { m.feature_names.push_back(r.str()); });
        }
      } else if (key == "trees") {
        has_trees = true;
        r.array([&] {
          m.trees.emplace_back();
          read_tree(r, m.trees.back());
        });
      } else if (key == "numClasses") {
        if (!r.null_literal()) {
          m.has_num_classes = true;
          m.num_classes_file = r.i64(INT64_MIN, INT64_MAX, "numClasses");
        }
      } else if (key == "baseScores") {
        if (!r.null_literal()) {
          m.has_base_scores = true;
          read_f32_array(r, m.base_scores_file);
        }
      } else {
        r.skip();
      }
    });
    if (!r.eof()) r.fail("trailing data after the model object");
    if (!has_version || !has_obj || !has_bins || !has_base || !has_nf || !has_trees)
      throw ParseError(
          "model file lacks one of version / objective / numBins / baseScore / numFeatures / "
          "trees");
    // Booster.swift:2146-2148: version 1 and a known objective.
    if (version != 1) throw ParseError("unsupported model file version " + std::to_string(version));
    if (objective < 0 || objective > 7)
      throw ParseError("unsupported model file: unknown objective " + std::to_string(objective));
    // MacBooster(params:) validation, Booster.swift:263-265.
    if (bins < 4 || bins > 256)
      throw ParseError("numBins must be in 4...256, got " + std::to_string(bins));
    m.version = int32_t(version);
    m.objective = int32_t(objective);
    m.num_bins = int32_t(bins);

    // Classes scored: `numClasses` of the file, 1 when absent (Booster.swift:2157,
    // _pyinfer.py:31 -- which also maps 0 to 1).
    int64_t K = m.has_num_classes ? m.num_classes_file : 1;
    if (K == 0) K = 1;
    if (K < 1 || K > 128) throw ParseError("numClasses must be in 1...128, got " + std::to_string(K));
    if (m.objective == kMulticlass && std::max<int64_t>(K, 3) > 128)
      throw ParseError("multiclass requires numClasses <= 128");
    m.K = int32_t(K);
    // Starting margins: `baseScores`, else [baseScore] (Booster.swift:2158,
    // _pyinfer.py:32-33).  Both reference predictors index it by class.
    if (m.has_base_scores && !m.base_scores_file.empty()) {
      if (int64_t(m.base_scores_file.size()) != K)
        throw ParseError("baseScores has " + std::to_string(m.base_scores_file.size()) +
                         " entries for " + std::to_string(K) + " classes");
      m.base_scores = m.base_scores_file;
    } else {
      if (K != 1) throw ParseError("a model with several classes needs baseScores per class");
      m.base_scores = {m.base_score};
    }
    m.max_depth = 0;
    bool any_cat = false;
    for (size_t ti = 0; ti < m.trees.size(); ++ti) {
      validate_tree(m.trees[ti], ti, m, any_cat, m.reachable_nodes);
      m.max_depth = std::max(m.max_depth, m.trees[ti].depth);
    }
    m.any_cat = any_cat;
  } catch (const ParseError& e) {
    err = e.what();
    return false;
  } catch (const std::bad_alloc&) {
    err = "out of host memory while reading the model";
    return false;
  }
  return true;
}

bool parse_json_string_array(const char* text, size_t len, std::vector<std::string>& out,
                             std::string& err) {
  out.clear();
  try {
    Reader r(text, len);
    r.expect('[');
    if (!r.eat(']')) {
      do {
        out.push_back(r.str());
      } while (r.eat(','));
      r.expect(']');
    }
    if (!r.eof()) r.fail("trailing characters");
    return true;
  } catch (const ParseError& e) {
    err = e.what();
    return false;
  }
}

bool load_model_file(const std::string& path, Model& m, std::string& err) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) {
    err = "cannot open model file '" + path + "': " + std::strerror(errno);
    return false;
  }
  std::string buf;
  char tmp[1 << 16];
  size_t got;
  while ((got = std::fread(tmp, 1, sizeof(tmp), f)) > 0) buf.append(tmp, got);
  bool io_err = std::ferror(f) != 0;
  std::fclose(f);
  if (io_err) {
    err = "error reading model file '" + path + "'";
    return false;
  }
  return parse_model_json(buf.data(), buf.size(), m, err);
}

namespace {

void put_f32(std::string& s, float v) {
  // Exact decimal of the float64 value of v: every float64-then-float32 reader
  // (including this one and PyModel) recovers v bit for bit.
  char b[64];
  auto r = std::to_chars(b, b + sizeof(b), double(v));
  std::string_view t(b, size_t(r.ptr - b));
  s.append(t);
  if (t.find_first_of(".eEn") == std::string_view::npos) s.append(".0");
}

template <class T>
void put_ints(std::string& s, const std::vector<T>& v) {
  s += '[';
  for (size_t i = 0; i < v.size(); ++i) {
    if (i) s += ',';
    s += std::to_string(int64_t(v[i]));
  }
  s += ']';
}

void put_floats(std::string& s, const std::vector<float>& v) {
  s += '[';
  for (size_t i = 0; i < v.size(); ++i) {
    if (i) s += ',';
    put_f32(s, v[i]);
  }
  s += ']';
}

void put_str(std::string& s, const std::string& v) {
  s += '"';
  for (unsigned char c : v) {
    if (c == '"' || c == '\\') {
      s += '\\';
      s += char(c);
    } else if (c < 0x20) {
      char b[8];
      std::snprintf(b, sizeof(b), "\\u%04x", c);
      s += b;
    } else {
      s += char(c);
    }
  }
  s += '"';
}

}  // namespace

std::string model_to_json(const Model& m) {
  std::string s;
  s.reserve(1 << 20);
  s += "{\"version\":" + std::to_string(m.version);
  s += ",\"objective\":" + std::to_string(m.objective);
  s += ",\"numBins\":" + std::to_string(m.num_bins);
  s += ",\"baseScore\":";
  put_f32(s, m.base_score);
  s += ",\"numFeatures\":" + std::to_string(m.num_features);
  s += ",\"categorical\":";
  put_ints(s, m.categorical);
  if (m.has_feature_names) {
    s += ",\"featureNames\":[";
    for (size_t i = 0; i < m.feature_names.size(); ++i) {
      if (i) s += ',';
      put_str(s, m.feature_names[i]);
    }
    s += ']';
  }
  s += ",\"trees\":[";
  for (size_t ti = 0; ti < m.trees.size(); ++ti) {
    const Tree& t = m.trees[ti];
    if (ti) s += ',';
    s += "{\"feature\":";
    put_ints(s, t.feature);
    s += ",\"threshold\":";
    put_floats(s, t.threshold);
    s += ",\"leaf\":";
    put_floats(s, t.leaf);
    s += ",\"flags\":";
    put_ints(s, t.flags);
    s += ",\"catMask\":";
    put_ints(s, t.cat_mask);
    if (!t.gain.empty()) {
      s += ",\"gain\":";
      put_floats(s, t.gain);
    }
    if (!t.cover.empty()) {
      s += ",\"cover\":";
      put_floats(s, t.cover);
    }
    s += '}';
  }
  s += ']';
  s += ",\"numClasses\":" + std::to_string(m.has_num_classes ? m.num_classes_file : m.K);
  s += ",\"baseScores\":";
  put_floats(s, m.base_scores);
  s += '}';
  return s;
}

}  // namespace mb
