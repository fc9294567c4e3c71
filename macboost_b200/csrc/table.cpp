// Text tables, prediction files and the predict command of MacBoost's CLI.
//
// Reader rules follow Sources/MacBoostCLI/CSV.swift byte for byte (which
// bytes end a field or a line, which lines are skipped, strtof on each field
// in place, the first short row reported); rows are parsed by all host cores
// into one float32 buffer that holds only the columns asked for.
#include "table.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <locale.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cfloat>
#include <charconv>
#include <climits>
#include <limits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "engine.h"

namespace mb {

Table::~Table() {
  if (!data) return;
  if (pinned)
    cudaFreeHost(data);
  else
    std::free(data);
}

namespace {

// ---- threads --------------------------------------------------------------

int host_threads() {
  const unsigned hc = std::thread::hardware_concurrency();
  return hc ? int(hc) : 1;
}

// Runs fn(lo, hi) over [0, n) split into contiguous ranges of at least
// `grain` items, one host thread per range.  Returns false if a range threw.
template <class F>
bool parallel_ranges(int64_t n, int64_t grain, F&& fn) {
  if (n <= 0) return true;
  const int64_t want = (n + grain - 1) / grain;
  const int nt = int(std::max<int64_t>(1, std::min<int64_t>(want, host_threads())));
  std::atomic<bool> ok{true};
  auto body = [&](int64_t lo, int64_t hi) {
    try {
      fn(lo, hi);
    } catch (...) {
      ok = false;
    }
  };
  if (nt == 1) {
    body(0, n);
    return ok;
  }
  std::vector<std::thread> th;
  th.reserve(size_t(nt));
  for (int t = 0; t < nt; ++t) th.emplace_back(body, n * t / nt, n * (t + 1) / nt);
  for (auto& x : th) x.join();
  return ok;
}

void atomic_min(std::atomic<int64_t>& a, int64_t v) {
  int64_t cur = a.load();
  while (v < cur && !a.compare_exchange_weak(cur, v)) {
  }
}

// ---- number parsing ---------------------------------------------------------

locale_t c_locale() {
  static locale_t loc = newlocale(LC_ALL_MASK, "C", locale_t(0));
  return loc;
}

float strtof_c(const char* s, char** end) {
  locale_t loc = c_locale();
  return loc ? strtof_l(s, end, loc) : std::strtof(s, end);
}

// ---- file and header --------------------------------------------------------

// The file's bytes followed by '\n' and NUL, as CSV.swift:50-54 appends them.
bool read_file(const char* path, std::vector<char>& buf, std::string& err) {
  const std::string io = std::string("CSV I/O error: cannot read ") + path;
  FILE* f = std::fopen(path, "rb");
  if (!f) {
    err = io;
    return false;
  }
  struct stat st;
  if (fstat(fileno(f), &st) != 0 || !S_ISREG(st.st_mode)) {
    std::fclose(f);
    err = io;
    return false;
  }
  try {
    buf.resize(size_t(st.st_size) + 2);
  } catch (...) {
    std::fclose(f);
    err = io;
    return false;
  }
  const size_t got = std::fread(buf.data(), 1, size_t(st.st_size), f);
  std::fclose(f);
  if (got != size_t(st.st_size)) {
    err = io;
    return false;
  }
  buf[got] = '\n';
  buf[got + 1] = '\0';
  return true;
}

// Unicode White_Space (Swift's CharacterSet.whitespacesAndNewlines).
bool is_space_cp(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F ||
         c == 0x205F || c == 0x3000;
}

// Decodes the UTF-8 code point starting at s[i] (length in *len); invalid
// sequences decode as one non-space unit.
uint32_t decode_at(const std::string& s, size_t i, size_t* len) {
  const unsigned char c = static_cast<unsigned char>(s[i]);
  int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
  if (n == 0 || i + size_t(n) > s.size()) {
    *len = 1;
    return 0xFFFFFFFFu;
  }
  uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
  for (int k = 1; k < n; ++k) {
    const unsigned char d = static_cast<unsigned char>(s[i + size_t(k)]);
    if ((d >> 6) != 2) {
      *len = 1;
      return 0xFFFFFFFFu;
    }
    cp = (cp << 6) | (d & 0x3F);
  }
  *len = size_t(n);
  return cp;
}

std::string trim_unicode_space(const std::string& s) {
  size_t b = 0;
  while (b < s.size()) {
    size_t len = 1;
    if (!is_space_cp(decode_at(s, b, &len))) break;
    b += len;
  }
  size_t e = s.size();
  while (e > b) {
    size_t st = e - 1;
    while (st > b && (static_cast<unsigned char>(s[st]) >> 6) == 2) --st;
    size_t len = 1;
    const uint32_t cp = decode_at(s, st, &len);
    if (st + len != e || !is_space_cp(cp)) break;
    e = st;
  }
  return s.substr(b, e - b);
}

// Line starts: the candidates are `first` and every position after a '\n'
// at or beyond `first` (below n); a candidate is kept unless its byte is in
// `skip` (CSV.swift:72-78 and 140-145).
std::vector<int64_t> line_starts(const char* b, int64_t first, int64_t n, const char* skip) {
  std::vector<int64_t> out;
  if (first >= n) return out;
  const int64_t span = n - first;
  const int64_t grain = int64_t(1) << 22;
  const int nt = int(std::max<int64_t>(1, std::min<int64_t>((span + grain - 1) / grain,
                                                            host_threads())));
  std::vector<std::vector<int64_t>> parts(static_cast<size_t>(nt));
  auto keep = [&](int64_t p) { return std::strchr(skip, b[p]) == nullptr; };
  bool ok = parallel_ranges(nt, 1, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t lo = first + span * t / nt, hi = first + span * (t + 1) / nt;
      std::vector<int64_t>& v = parts[size_t(t)];
      if (t == 0 && keep(first)) v.push_back(first);
      const char* p = b + lo;
      const char* e = b + hi;
      while (p < e) {
        const void* nl = std::memchr(p, '\n', size_t(e - p));
        if (!nl) break;
        const int64_t q = static_cast<const char*>(nl) - b;
        if (q + 1 < n && keep(q + 1)) v.push_back(q + 1);
        p = static_cast<const char*>(nl) + 1;
      }
    }
  });
  if (!ok) throw std::bad_alloc();
  size_t total = 0;
  for (auto& v : parts) total += v.size();
  out.reserve(total);
  for (auto& v : parts) out.insert(out.end(), v.begin(), v.end());
  return out;
}

// ---- the held-column buffer ---------------------------------------------------

bool alloc_table(Table& t, int64_t rows, bool pin, std::string& err) {
  t.rows = rows;
  const size_t bytes = size_t(rows) * size_t(std::max<int64_t>(t.width(), 0)) * sizeof(float);
  if (bytes == 0) return true;
  if (pin) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) == cudaSuccess) {
      t.data = static_cast<float*>(p);
      t.pinned = true;
      return true;
    }
    cudaGetLastError();  // no driver / device: ordinary memory serves the same
  }
  t.data = static_cast<float*>(std::malloc(bytes));
  if (!t.data) {
    err = "cannot allocate " + std::to_string(bytes) + " bytes for the table";
    return false;
  }
  return true;
}

// For each file column, the first held slot reading it (-1: not held), and
// the (slot, source slot) pairs of columns held more than once.
struct SlotMap {
  std::vector<int64_t> first;
  std::vector<std::pair<int64_t, int64_t>> repeats;
};

bool make_slots(const Table& t, int64_t file_cols, SlotMap& m, std::string& err) {
  m.first.assign(size_t(file_cols), -1);
  for (int64_t j = 0; j < t.width(); ++j) {
    const int64_t c = t.columns[size_t(j)];
    if (c < 0 || c >= file_cols) {
      err = "column " + std::to_string(c) + " is out of range";
      return false;
    }
    if (m.first[size_t(c)] < 0)
      m.first[size_t(c)] = j;
    else
      m.repeats.push_back({j, m.first[size_t(c)]});
  }
  return true;
}

// ---- CSV / TSV (CSV.swift:48-118) -----------------------------------------------

bool parse_csv(std::vector<char>& buf, const ColumnChooser& choose, bool pin, Table& t,
               std::string& err) {
  const char* b = buf.data();
  const int64_t n = int64_t(buf.size()) - 1;  // bytes before the NUL
  int64_t pos = 0;
  while (pos < n && b[pos] != '\n') ++pos;
  if (pos >= n) {
    err = "Malformed CSV: no header line";
    return false;
  }
  const std::string line(b, size_t(pos));
  const char delim = line.find('\t') != std::string::npos ? '\t' : ',';
  t.header.clear();
  size_t s = 0;
  while (true) {
    const size_t e = line.find(delim, s);
    t.header.push_back(trim_unicode_space(line.substr(s, e == std::string::npos ? e : e - s)));
    if (e == std::string::npos) break;
    s = e + 1;
  }
  const int64_t C = int64_t(t.header.size());
  const std::vector<int64_t> starts = line_starts(b, pos + 1, n, "\n\r");
  const int64_t rows = int64_t(starts.size());
  if (rows == 0) {
    err = "Malformed CSV: no data rows";
    return false;
  }
  if (choose) {
    t.columns = choose(t.header);
  } else {
    t.columns.resize(size_t(C));
    for (int64_t c = 0; c < C; ++c) t.columns[size_t(c)] = c;
  }
  SlotMap sm;
  if (!make_slots(t, C, sm, err) || !alloc_table(t, rows, pin, err)) return false;
  const int64_t W = t.width();
  float* out = t.data;
  std::atomic<int64_t> bad{INT64_MAX};
  const float nan = std::numeric_limits<float>::quiet_NaN();
  const bool ok = parallel_ranges(rows, 4096, [&](int64_t r0, int64_t r1) {
    for (int64_t i = r0; i < r1; ++i) {
      float* row = out ? out + i * W : nullptr;
      for (int64_t j = 0; j < W; ++j) row[j] = nan;
      int64_t q = starts[size_t(i)];
      for (int64_t c = 0; c < C; ++c) {
        const int64_t fs = q;
        bool is_end = false;
        while (true) {
          const char ch = b[q];
          if (ch == delim) break;
          if (ch == '\n' || ch == '\r') {
            is_end = true;
            break;
          }
          ++q;
        }
        const int64_t slot = sm.first[size_t(c)];
        if (q > fs && slot >= 0) {
          char* end = nullptr;
          const float v = parse_f32(b + fs, &end);
          if (end - b > fs) row[slot] = v;  // else non-numeric: stays NaN
        }
        if (is_end) {
          if (c + 1 < C) atomic_min(bad, i);
          break;
        }
        ++q;  // past the delimiter
      }
      for (const auto& r : sm.repeats) row[r.first] = row[r.second];
    }
  });
  if (!ok) {
    err = "out of host memory while parsing";
    return false;
  }
  if (bad.load() != INT64_MAX) {
    err = "Malformed CSV: row " + std::to_string(bad.load() + 1) +
          " has fewer fields than the header (" + std::to_string(C) + ")";
    return false;
  }
  return true;
}

// ---- LibSVM (CSV.swift:126-217) ----------------------------------------------------

// Walks one line's "idx:value" pairs (CSV.swift:156-181): returns the label
// and calls body(idx, value) for each pair, skipping tokens that are not
// "integer:" (qid:..., stray words) up to the next blank.
template <class F>
float for_each_pair(const char* b, int64_t start, F&& body) {
  char* end = nullptr;
  const float label = parse_f32(b + start, &end);
  int64_t q = end - b;
  while (true) {
    while (b[q] == ' ' || b[q] == '\t') ++q;
    if (b[q] == '\n' || b[q] == '\r' || b[q] == '#') break;
    char* e = nullptr;
    const long idx = std::strtol(b + q, &e, 10);
    const int64_t idx_end = e - b;
    if (idx_end == q || b[idx_end] != ':') {
      int64_t skip = q;
      while (b[skip] != ' ' && b[skip] != '\t' && b[skip] != '\n' && b[skip] != '\r') ++skip;
      q = skip;
      continue;
    }
    char* ve = nullptr;
    const float v = parse_f32(b + idx_end + 1, &ve);
    q = ve - b;
    body(int64_t(idx), v);
  }
  return label;
}

bool parse_libsvm(std::vector<char>& buf, const ColumnChooser& choose, bool pin, Table& t,
                  std::string& err) {
  const char* b = buf.data();
  const int64_t n = int64_t(buf.size()) - 1;
  const std::vector<int64_t> starts = line_starts(b, 0, n, "\n\r#");
  const int64_t rows = int64_t(starts.size());
  if (rows == 0) {
    err = "Malformed CSV: no data rows";
    return false;
  }
  // pass A: index range
  std::atomic<int64_t> mn{INT64_MAX};
  std::atomic<int64_t> mx_neg{INT64_MAX};  // -max, so atomic_min serves both
  bool ok = parallel_ranges(rows, 4096, [&](int64_t r0, int64_t r1) {
    int64_t lmax = -1, lmin = INT64_MAX;
    for (int64_t i = r0; i < r1; ++i)
      for_each_pair(b, starts[size_t(i)], [&](int64_t idx, float) {
        lmax = std::max(lmax, idx);
        lmin = std::min(lmin, idx);
      });
    atomic_min(mn, lmin);
    atomic_min(mx_neg, -lmax);
  });
  if (!ok) {
    err = "out of host memory while parsing";
    return false;
  }
  const int64_t max_idx = -mx_neg.load(), min_idx = mn.load();
  if (max_idx < 0) {
    err = "Malformed CSV: no idx:value pairs found";
    return false;
  }
  if (min_idx < 0) {
    err = "Malformed CSV: negative feature index " + std::to_string(min_idx);
    return false;
  }
  const int64_t base = min_idx == 0 ? 0 : 1;  // sklearn-style detection, CSV.swift:199
  const int64_t features = max_idx - base + 1;
  if (features > (int64_t(1) << 31)) {
    err = "Malformed CSV: feature index " + std::to_string(max_idx) + " is too large";
    return false;
  }
  const int64_t C = features + 1;
  t.header.clear();
  t.header.reserve(size_t(C));
  t.header.push_back("label");
  for (int64_t f = 0; f < features; ++f) t.header.push_back("f" + std::to_string(f));
  if (choose) {
    t.columns = choose(t.header);
  } else {
    t.columns.resize(size_t(C));
    for (int64_t c = 0; c < C; ++c) t.columns[size_t(c)] = c;
  }
  SlotMap sm;
  if (!make_slots(t, C, sm, err) || !alloc_table(t, rows, pin, err)) return false;
  const int64_t W = t.width();
  float* out = t.data;
  // pass B: absent features are 0 (the LibSVM convention)
  ok = parallel_ranges(rows, 4096, [&](int64_t r0, int64_t r1) {
    for (int64_t i = r0; i < r1; ++i) {
      float* row = out ? out + i * W : nullptr;
      for (int64_t j = 0; j < W; ++j) row[j] = 0.0f;
      const float label = for_each_pair(b, starts[size_t(i)], [&](int64_t idx, float v) {
        const int64_t slot = sm.first[size_t(1 + idx - base)];
        if (slot >= 0) row[slot] = v;
      });
      if (sm.first[0] >= 0) row[sm.first[0]] = label;
      for (const auto& r : sm.repeats) row[r.first] = row[r.second];
    }
  });
  if (!ok) {
    err = "out of host memory while parsing";
    return false;
  }
  return true;
}

bool has_libsvm_extension(const char* path) {
  const char* dot = std::strrchr(path, '.');
  const char* slash = std::strrchr(path, '/');
  if (!dot || (slash && slash > dot)) return false;
  std::string ext(dot + 1);
  for (char& c : ext) c = char(std::tolower(static_cast<unsigned char>(c)));
  return ext == "svm" || ext == "libsvm";
}

}  // namespace

// Decimal strings of at most 19 significant digits whose value m * 10^e
// (m < 2^53, |e| <= 22) lands in float32's normal range are converted with
// one correctly rounded double multiply or divide (Clinger's fast path) and
// one rounding to float32.  That second rounding can differ from rounding
// the exact value only when the double lies exactly halfway between two
// float32 values; such strings, and every other form (hex, inf, nan,
// leading blanks, long mantissas, subnormal or overflowing values), go to
// strtof itself.
float parse_f32(const char* s, char** end) {
  static const double kPow10[23] = {1e0,  1e1,  1e2,  1e3,  1e4,  1e5,  1e6,  1e7,
                                    1e8,  1e9,  1e10, 1e11, 1e12, 1e13, 1e14, 1e15,
                                    1e16, 1e17, 1e18, 1e19, 1e20, 1e21, 1e22};
  const char* p = s;
  bool neg = false;
  if (*p == '+' || *p == '-') {
    neg = *p == '-';
    ++p;
  }
  if (p[0] == '0' && (p[1] == 'x' || p[1] == 'X')) return strtof_c(s, end);
  uint64_t m = 0;
  int digits = 0, e10 = 0;
  bool any = false;
  for (; *p >= '0' && *p <= '9'; ++p) {
    any = true;
    if (m == 0 && *p == '0') continue;
    if (digits == 19) return strtof_c(s, end);
    m = m * 10 + uint64_t(*p - '0');
    ++digits;
  }
  if (*p == '.') {
    for (++p; *p >= '0' && *p <= '9'; ++p) {
      any = true;
      if (m == 0 && *p == '0') {
        --e10;
        continue;
      }
      if (digits == 19) return strtof_c(s, end);
      m = m * 10 + uint64_t(*p - '0');
      ++digits;
      --e10;
    }
  }
  if (!any) return strtof_c(s, end);
  if (*p == 'e' || *p == 'E') {
    const char* q = p + 1;
    bool eneg = false;
    if (*q == '+' || *q == '-') {
      eneg = *q == '-';
      ++q;
    }
    if (*q >= '0' && *q <= '9') {
      int ev = 0, ed = 0;
      for (; *q >= '0' && *q <= '9'; ++q, ++ed)
        if (ed < 6) ev = ev * 10 + (*q - '0');
      if (ed >= 6) return strtof_c(s, end);
      e10 += eneg ? -ev : ev;
      p = q;
    }
  }
  if (m == 0) {
    *end = const_cast<char*>(p);
    return neg ? -0.0f : 0.0f;
  }
  if (m > (uint64_t(1) << 53) || e10 < -22 || e10 > 22) return strtof_c(s, end);
  const double d = e10 >= 0 ? double(m) * kPow10[e10] : double(m) / kPow10[-e10];
  const float f = float(d);
  if (!(f >= FLT_MIN) || std::isinf(f)) return strtof_c(s, end);
  if (double(f) != d) {
    const float g = std::nextafter(f, d > double(f) ? INFINITY : 0.0f);
    if (d == (double(f) + double(g)) * 0.5) return strtof_c(s, end);
  }
  *end = const_cast<char*>(p);
  return neg ? -f : f;
}

bool read_table(const char* path, int format, const ColumnChooser& choose, bool pin, Table& t,
                std::string& err) {
  if (format != kFormatCsv && format != kFormatLibsvm && format != kFormatAuto) {
    err = "unknown table format " + std::to_string(format) + " (0 csv/tsv, 1 libsvm, 2 auto)";
    return false;
  }
  std::vector<char> buf;
  if (!read_file(path, buf, err)) return false;
  const bool libsvm = format == kFormatLibsvm || (format == kFormatAuto && has_libsvm_extension(path));
  try {
    return libsvm ? parse_libsvm(buf, choose, pin, t, err) : parse_csv(buf, choose, pin, t, err);
  } catch (const std::bad_alloc&) {
    err = "out of host memory while parsing";
    return false;
  }
}

// Swift prints a Float (`description`, SwiftDtoa) with the shortest digit
// string that reads back to the same value, as "d.ddde-05" when the decimal
// exponent is below -4 or the magnitude exceeds 2^24, else in positional form
// with at least one fractional digit ("1.0", "0.0001", "123.25"); every NaN
// prints "nan".  The digits come from std::to_chars (shortest round trip,
// nearest on ties), the layout is assembled here.
size_t format_float(float v, char* out) {
  if (std::isnan(v)) {
    std::memcpy(out, "nan", 3);
    return 3;
  }
  if (std::isinf(v)) {
    if (v < 0) {
      std::memcpy(out, "-inf", 4);
      return 4;
    }
    std::memcpy(out, "inf", 3);
    return 3;
  }
  size_t k = 0;
  if (std::signbit(v)) out[k++] = '-';
  if (v == 0.0f) {
    std::memcpy(out + k, "0.0", 3);
    return k + 3;
  }
  char sci[48];
  const auto r = std::to_chars(sci, sci + sizeof(sci), std::fabs(v), std::chars_format::scientific);
  char digits[16] = {};
  int nd = 0;
  const char* p = sci;
  for (; p < r.ptr && *p != 'e'; ++p)
    if (*p != '.') digits[nd++] = *p;
  // exponent: "e", a sign, digits (to_chars writes no terminating NUL)
  int exp10 = 0;  // value = d.ddd x 10^exp10
  const bool eneg = p + 1 < r.ptr && p[1] == '-';
  for (const char* q = p + 2; q < r.ptr; ++q) exp10 = exp10 * 10 + (*q - '0');
  if (eneg) exp10 = -exp10;
  const int dexp = exp10 + 1;           // value = 0.dddd x 10^dexp
  if (dexp < -3 || std::fabs(v) > 16777216.0f) {
    out[k++] = digits[0];
    if (nd > 1) {
      out[k++] = '.';
      for (int i = 1; i < nd; ++i) out[k++] = digits[i];
    }
    out[k++] = 'e';
    out[k++] = exp10 < 0 ? '-' : '+';
    const int a = exp10 < 0 ? -exp10 : exp10;
    if (a >= 100) out[k++] = char('0' + a / 100);
    out[k++] = char('0' + (a / 10) % 10);
    out[k++] = char('0' + a % 10);
    return k;
  }
  if (dexp <= 0) {
    out[k++] = '0';
    out[k++] = '.';
    for (int i = 0; i < -dexp; ++i) out[k++] = '0';
    for (int i = 0; i < nd; ++i) out[k++] = digits[i];
  } else if (dexp >= nd) {
    for (int i = 0; i < nd; ++i) out[k++] = digits[i];
    for (int i = nd; i < dexp; ++i) out[k++] = '0';
    out[k++] = '.';
    out[k++] = '0';
  } else {
    for (int i = 0; i < dexp; ++i) out[k++] = digits[i];
    out[k++] = '.';
    for (int i = dexp; i < nd; ++i) out[k++] = digits[i];
  }
  return k;
}

bool write_predictions(const float* p, int64_t rows, int64_t k, const char* path,
                       std::string& err) {
  if (!path || rows < 0 || k < 1 || (rows > 0 && !p)) {
    err = "null or invalid argument";
    return false;
  }
  std::string head;
  if (k > 1) {
    for (int64_t c = 0; c < k; ++c) head += (c ? ",class_" : "class_") + std::to_string(c);
  } else {
    head = "prediction";
  }
  head += '\n';
  const int64_t grain = 65536;
  const int64_t nchunks = std::max<int64_t>(1, (rows + grain - 1) / grain);
  std::vector<std::string> parts(static_cast<size_t>(nchunks));
  const bool ok = parallel_ranges(nchunks, 1, [&](int64_t c0, int64_t c1) {
    char tmp[40];
    for (int64_t c = c0; c < c1; ++c) {
      std::string& s = parts[size_t(c)];
      const int64_t r0 = c * grain, r1 = std::min(rows, r0 + grain);
      s.reserve(size_t((r1 - r0) * k * 13));
      for (int64_t i = r0; i < r1; ++i)
        for (int64_t j = 0; j < k; ++j) {
          const size_t len = format_float(p[i * k + j], tmp);
          s.append(tmp, len);
          s += j + 1 < k ? ',' : '\n';
        }
    }
  });
  if (!ok) {
    err = "out of host memory while formatting";
    return false;
  }
  // written to a fresh file beside the target, then renamed over it, as an
  // atomic Foundation write does
  static std::atomic<unsigned> serial{0};
  const std::string tmp = std::string(path) + ".tmp" + std::to_string(getpid()) + "." +
                          std::to_string(serial.fetch_add(1));
  const int fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_EXCL | O_CLOEXEC, 0666);
  if (fd < 0) {
    err = std::string("cannot write '") + path + "': " + std::strerror(errno);
    return false;
  }
  bool good = true;
  auto put = [&](const std::string& s) {
    size_t off = 0;
    while (good && off < s.size()) {
      const ssize_t w = ::write(fd, s.data() + off, s.size() - off);
      if (w < 0 && errno == EINTR) continue;
      if (w <= 0) good = false;
      else off += size_t(w);
    }
  };
  put(head);
  for (const auto& s : parts) put(s);
  if (::close(fd) != 0) good = false;
  if (!good || std::rename(tmp.c_str(), path) != 0) {
    const int e = errno;
    ::unlink(tmp.c_str());
    err = std::string("cannot write '") + path + "': " + std::strerror(e);
    return false;
  }
  return true;
}

bool cli_predict(Engine& e, const char* data_path, int format, bool raw,
                 const std::vector<int>& devices, const char* output_path, int64_t* rows_out,
                 std::string& err) {
  const Model& m = e.model;
  std::string map_err;
  // main.swift:327-342: by name when the model stores names, else the first
  // numFeatures columns.  The reader validates every row before this error
  // is reported, as the reference reads the whole table first.
  ColumnChooser choose = [&](const std::vector<std::string>& header) {
    std::vector<int64_t> cols;
    if (m.has_feature_names) {
      for (const std::string& name : m.feature_names) {
        const auto it = std::find(header.begin(), header.end(), name);
        if (it == header.end()) {
          map_err = "Malformed CSV: column '" + name + "' required by the model is missing";
          return std::vector<int64_t>();
        }
        cols.push_back(int64_t(it - header.begin()));
      }
    } else {
      if (int64_t(header.size()) < m.num_features) {
        map_err = "model expects " + std::to_string(m.num_features) + " features, CSV has " +
                  std::to_string(header.size()) + " columns";
        return std::vector<int64_t>();
      }
      for (int64_t f = 0; f < m.num_features; ++f) cols.push_back(f);
    }
    return cols;
  };
  Table t;
  if (!read_table(data_path, format, choose, true, t, err)) return false;
  if (!map_err.empty()) {
    err = map_err;
    return false;
  }
  const int kind = raw ? kKindPredict : kKindCli;
  const int64_t k = output_cols(e, kind);
  std::vector<float> out;
  try {
    out.resize(size_t(t.rows) * size_t(k));
  } catch (...) {
    err = "out of host memory for the predictions";
    return false;
  }
  if (engine_predict_host(e, t.data, t.rows, t.width(), /*row-major*/ 1, kind, devices,
                          out.data(), err) != 0)
    return false;
  if (!write_predictions(out.data(), t.rows, k, output_path, err)) return false;
  if (rows_out) *rows_out = t.rows;
  return true;
}

}  // namespace mb
