// Binned data: .mbds files, binning, and binned tree walks (see binned.h).
#include "binned.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

#include "engine.h"
#include "kernels.h"
#include "model.h"
#include "table.h"

namespace mb {

namespace {

std::string cuda_msg(const char* what, cudaError_t e) {
  return std::string(what) + ": " + cudaGetErrorString(e);
}

#define BN_CUDA(call, what)     \
  do {                          \
    cudaError_t e_ = (call);    \
    if (e_ != cudaSuccess) {    \
      err = cuda_msg(what, e_); \
      return -1;                \
    }                           \
  } while (0)

struct Guard {
  int prev = -1;
  explicit Guard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~Guard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Device allocation released with the owner.
struct DevBuf {
  void* p = nullptr;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int alloc(size_t bytes, std::string& err) {
    BN_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc (binned data)");
    return 0;
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

template <class T>
int upload(DevBuf& b, const T* src, size_t n, std::string& err) {
  if (b.alloc(n * sizeof(T), err)) return -1;
  if (n) BN_CUDA(cudaMemcpy(b.p, src, n * sizeof(T), cudaMemcpyHostToDevice), "cudaMemcpy (binned)");
  return 0;
}

int check_device(int device, std::string& err) {
  int n = 0;
  const cudaError_t ce = cudaGetDeviceCount(&n);
  if (ce != cudaSuccess || n == 0) {
    cudaGetLastError();
    err = ce != cudaSuccess ? cuda_msg("no CUDA device available", ce)
                            : std::string("no CUDA device available");
    return -1;
  }
  if (device < 0 || device >= n) {
    err = "device " + std::to_string(device) + " does not exist (" + std::to_string(n) +
          " visible)";
    return -1;
  }
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (major != 10) {
    err = "device " + std::to_string(device) + " is not an sm_100a (B200) GPU";
    return -1;
  }
  return 0;
}

// Little-endian reader over the file's bytes.
struct Bytes {
  const uint8_t* p;
  size_t n, pos = 0;
  bool take(void* dst, size_t k) {
    if (k > n - pos) return false;
    if (k) std::memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  template <class T>
  bool get(T& v) {
    return take(&v, sizeof(T));
  }
};

}  // namespace

bool load_mbds(const char* path, Dataset& d, std::string& err) {
  std::vector<uint8_t> buf;
  {
    FILE* f = std::fopen(path, "rb");
    if (!f) {
      err = std::string("cannot read '") + path + "'";
      return false;
    }
    std::fseek(f, 0, SEEK_END);
    const long sz = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (sz < 0) {
      std::fclose(f);
      err = std::string("cannot read '") + path + "'";
      return false;
    }
    try {
      buf.resize(size_t(sz));
    } catch (...) {
      std::fclose(f);
      err = "out of host memory reading the dataset";
      return false;
    }
    const size_t got = std::fread(buf.data(), 1, buf.size(), f);
    std::fclose(f);
    if (got != buf.size()) {
      err = std::string("cannot read '") + path + "'";
      return false;
    }
  }
  // Dataset.swift:41-83
  const std::string trunc = "Invalid input: truncated .mbds file";
  Bytes r{buf.data(), buf.size()};
  uint32_t magic = 0, version = 0, tile = 0, cols = 0, nb = 0, ncat = 0, namelen = 0;
  uint64_t rows = 0;
  if (!r.get(magic)) {
    err = trunc;
    return false;
  }
  if (magic != 0x4D424453u) {
    err = "Invalid input: not a MacBoost dataset (.mbds) file";
    return false;
  }
  if (!r.get(version)) {
    err = trunc;
    return false;
  }
  if (version != 1) {
    err = "Invalid input: unsupported .mbds version";
    return false;
  }
  if (!r.get(tile)) {
    err = trunc;
    return false;
  }
  if (tile != 8) {
    err = "Invalid input: .mbds tile width mismatch";
    return false;
  }
  if (!r.get(rows) || !r.get(cols) || !r.get(nb) || !r.get(ncat)) {
    err = trunc;
    return false;
  }
  d = Dataset();
  for (uint32_t c = 0; c < ncat; ++c) {
    uint32_t v = 0;
    if (!r.get(v)) {
      err = trunc;
      return false;
    }
    d.categorical.push_back(int64_t(v));
  }
  std::sort(d.categorical.begin(), d.categorical.end());
  if (!r.get(namelen) || namelen > r.n - r.pos) {
    err = trunc;
    return false;
  }
  if (namelen > 0) {
    std::string why;
    if (!parse_json_string_array(reinterpret_cast<const char*>(buf.data() + r.pos), namelen,
                                 d.names, why)) {
      err = "Invalid input: .mbds feature names: " + why;
      return false;
    }
    d.has_names = true;
    r.pos += namelen;
  }
  auto arr = [&](auto& vec) -> bool {
    uint64_t count = 0;
    if (!r.get(count)) return false;
    using T = typename std::decay_t<decltype(vec)>::value_type;
    if (count > (r.n - r.pos) / sizeof(T)) return false;
    vec.resize(size_t(count));
    return r.take(vec.data(), size_t(count) * sizeof(T));
  };
  if (!arr(d.edges) || !arr(d.labels) || !arr(d.bins)) {
    err = trunc;
    return false;
  }
  const uint64_t tiles = (uint64_t(cols) + 7) / 8;
  if (d.labels.size() != rows || d.bins.size() != rows * tiles * 8 || nb < 2 ||
      d.edges.size() != uint64_t(cols) * (nb - 2)) {
    err = "Invalid input: .mbds sizes are inconsistent";
    return false;
  }
  if (nb < 4 || nb > 256) {
    err = "Invalid input: .mbds numBins must be in 4...256, got " + std::to_string(nb);
    return false;
  }
  for (int64_t c : d.categorical)
    if (c >= int64_t(cols)) {
      err = "Invalid input: .mbds categorical feature " + std::to_string(c) + " out of range";
      return false;
    }
  d.rows = int64_t(rows);
  d.cols = int64_t(cols);
  d.num_bins = int32_t(nb);
  return true;
}

bool model_split_form(const Engine& e, const float* edges, int64_t cols, int num_bins,
                      SplitTrees& s, std::string& err) {
  const Model& m = e.model;
  if (m.num_features != cols) {
    err = "model expects " + std::to_string(m.num_features) + " features, the dataset has " +
          std::to_string(cols);
    return false;
  }
  if (m.num_bins != num_bins) {
    err = "model was trained with numBins " + std::to_string(m.num_bins) +
          ", the dataset has " + std::to_string(num_bins);
    return false;
  }
  const int ne = num_bins - 2;
  // edge rows in ascending order allow a binary search for the first match
  std::vector<int8_t> sorted(size_t(cols), -1);
  auto first_edge = [&](int64_t f, float th) -> int {
    const float* row = edges + size_t(f) * size_t(ne);
    if (sorted[size_t(f)] < 0) sorted[size_t(f)] = std::is_sorted(row, row + ne) ? 1 : 0;
    if (sorted[size_t(f)]) {
      const float* it = std::lower_bound(row, row + ne, th);
      return (it != row + ne && *it == th) ? int(it - row) : -1;
    }
    for (int b = 0; b < ne; ++b)
      if (row[b] == th) return b;
    return -1;
  };
  s = SplitTrees();
  s.tree_off.push_back(0);
  for (size_t t = 0; t < m.trees.size(); ++t) {
    const Tree& tr = m.trees[t];
    const bool masked = !tr.cat_mask.empty();
    for (size_t g = 0; g < tr.feature.size(); ++g) {
      const int32_t f = tr.feature[g];
      s.feature.push_back(f);
      s.leaf.push_back(tr.leaf[g]);
      uint32_t fl = tr.flags[g];
      uint32_t b = 0;
      if (f >= 0) {
        if ((fl & kFlagCategorical) && masked) {
          for (int w = 0; w < 8; ++w) s.catmask.push_back(tr.cat_mask[g * 8 + size_t(w)]);
        } else {
          fl &= ~kFlagCategorical;  // numeric routing, as the float predictor
          const int hit = first_edge(f, tr.threshold[g]);
          if (hit < 0) {
            char th[48];
            std::snprintf(th, sizeof(th), "%.9g", double(tr.threshold[g]));
            err = "tree " + std::to_string(t) + " node " + std::to_string(g) + ": threshold " +
                  th + " of feature " + std::to_string(f) + " is not one of the dataset's bin edges";
            return false;
          }
          b = uint32_t(hit);
        }
      }
      if (f < 0 || !((fl & kFlagCategorical) && masked))
        for (int w = 0; w < 8; ++w) s.catmask.push_back(0u);
      s.sbin.push_back(b);
      s.flags.push_back(fl);
    }
    s.tree_off.push_back((long long)s.feature.size());
  }
  s.max_depth = m.max_depth;
  return true;
}

int bin_data_host(int device, const float* x, int64_t rows, int64_t cols, int layout,
                  const float* edges, int num_bins, const uint8_t* categorical, uint8_t* bins,
                  std::string& err) {
  if (rows < 0 || cols < 0 || (layout != 0 && layout != 1) || num_bins < 4 || num_bins > 256) {
    err = "invalid argument (rows, cols >= 0; layout 0 or 1; num_bins in 4...256)";
    return -1;
  }
  if (rows == 0 || cols == 0) return 0;
  if (check_device(device, err)) return -1;
  Guard gd(device);
  const int64_t groups = (cols + 7) / 8;
  std::vector<uint8_t> cat(size_t(cols), 0);
  if (categorical) std::memcpy(cat.data(), categorical, size_t(cols));
  DevBuf dedges, dcat, dx, dbins;
  if (upload(dedges, edges, size_t(cols) * size_t(num_bins - 2), err) ||
      upload(dcat, cat.data(), cat.size(), err))
    return -1;
  // chunks of rows with at most 256 MB of input
  int64_t C = std::max<int64_t>((int64_t(256) << 20) / (cols * 4), 256);
  C = std::min(C, rows);
  if (dx.alloc(size_t(C) * size_t(cols) * 4, err) || dbins.alloc(size_t(groups) * C * 8, err))
    return -1;
  for (int64_t r0 = 0; r0 < rows; r0 += C) {
    const int64_t nr = std::min(C, rows - r0);
    if (layout == 0)
      BN_CUDA(cudaMemcpy2D(dx.p, size_t(nr) * 4, x + r0, size_t(rows) * 4, size_t(nr) * 4,
                           size_t(cols), cudaMemcpyHostToDevice),
              "cudaMemcpy2D (values)");
    else
      BN_CUDA(cudaMemcpy(dx.p, x + r0 * cols, size_t(nr) * size_t(cols) * 4,
                         cudaMemcpyHostToDevice),
              "cudaMemcpy (values)");
    BN_CUDA(launch_bin_data(dx.as<float>(), nr, cols, nr, layout, dedges.as<float>(), num_bins,
                            dcat.as<unsigned char>(), dbins.as<unsigned char>(), 0),
            "bin_data launch");
    g_kernel_launches.fetch_add(1);
    // chunk tile g (nr rows) -> rows [r0, r0 + nr) of tile g in the rows-row matrix
    BN_CUDA(cudaMemcpy2D(bins + r0 * 8, size_t(rows) * 8, dbins.p, size_t(nr) * 8,
                         size_t(nr) * 8, size_t(groups), cudaMemcpyDeviceToHost),
            "cudaMemcpy2D (bins)");
  }
  BN_CUDA(cudaDeviceSynchronize(), "bin_data");
  return 0;
}

int bin_data_device(int device, const float* x, int64_t rows, int64_t cols, int64_t ld,
                    int layout, const float* edges, int num_bins, const uint8_t* categorical,
                    uint8_t* bins, cudaStream_t stream, std::string& err) {
  if (rows < 0 || cols < 0 || (layout != 0 && layout != 1) || num_bins < 4 || num_bins > 256 ||
      (layout == 0 && ld < rows) || !categorical) {
    err = "invalid argument (rows, cols >= 0; layout 0 or 1 with ld >= rows; num_bins in "
          "4...256; categorical flags in device memory)";
    return -1;
  }
  if (rows == 0 || cols == 0) return 0;
  if (check_device(device, err)) return -1;
  Guard gd(device);
  BN_CUDA(launch_bin_data(x, rows, cols, layout == 0 ? ld : cols, layout, edges, num_bins,
                          categorical, bins, stream),
          "bin_data launch");
  g_kernel_launches.fetch_add(1);
  return 0;
}

namespace {

// Upload trees in split form; validates nothing on the device side (the
// kernel checks features and children as it walks).
struct DevTrees {
  DevBuf off, feature, sbin, flags, mask, leaf;
  long long nodes = 0;
  int put(int T, const int64_t* tree_off, const int32_t* f, const uint32_t* b,
          const uint32_t* fl, const uint32_t* cm, const float* lv, std::string& err) {
    const size_t N = size_t(tree_off[T]);
    nodes = (long long)(N - size_t(tree_off[0]));
    std::vector<long long> o(tree_off, tree_off + T + 1);
    return upload(off, o.data(), o.size(), err) || upload(feature, f, N, err) ||
                   upload(sbin, b, N, err) || upload(flags, fl, N, err) ||
                   upload(mask, cm, N * 8, err) || upload(leaf, lv, N, err)
               ? -1
               : 0;
  }
};

BinnedArgs tree_args(const DevTrees& t, int T, int64_t rows, int64_t cols, int num_bins,
                     int max_depth, int K) {
  BinnedArgs a{};
  a.n = rows;
  a.cols = cols;
  a.num_bins = num_bins;
  a.T = T;
  a.tree_off = t.off.as<long long>();
  a.feature = t.feature.as<int>();
  a.sbin = t.sbin.as<unsigned>();
  a.flags = t.flags.as<unsigned>();
  a.catmask = t.mask.as<unsigned>();
  a.leaf = t.leaf.as<float>();
  a.max_depth = max_depth;
  a.K = K;
  a.node_hint = t.nodes;
  return a;
}

int check_status(const unsigned* dstatus, std::string& err) {
  unsigned w = 0;
  BN_CUDA(cudaMemcpy(&w, dstatus, sizeof(w), cudaMemcpyDeviceToHost), "reading kernel status");
  if (w & kErrBadTree) {
    err = "a split names a feature outside the bin matrix or a child outside its tree";
    return -1;
  }
  return 0;
}

bool check_trees(int T, const int64_t* tree_off, std::string& err) {
  if (T < 0 || (T > 0 && !tree_off) || (T > 0 && tree_off[0] != 0)) {
    err = "tree offsets must start at 0";
    return false;
  }
  for (int t = 0; t < T; ++t)
    if (tree_off[t + 1] <= tree_off[t]) {
      err = "tree " + std::to_string(t) + " has no nodes";
      return false;
    }
  return true;
}

}  // namespace

int tree_binned_host(int device, const uint8_t* bins, int64_t rows, int64_t cols, int num_bins,
                     int T, const int64_t* tree_off, const int32_t* feature,
                     const uint32_t* sbin, const uint32_t* flags, const uint32_t* catmask,
                     const float* leaf, int max_depth, int K, float* preds, int32_t* leaf_idx,
                     std::string& err) {
  if (rows < 0 || cols < 0 || K < 1 || max_depth < 0 || num_bins < 4 || num_bins > 256) {
    err = "invalid argument (rows, cols, max_depth >= 0; num_classes >= 1; num_bins in 4...256)";
    return -1;
  }
  if (!check_trees(T, tree_off, err)) return -1;
  if (rows == 0 || T == 0) return 0;
  if (check_device(device, err)) return -1;
  Guard gd(device);
  const int64_t groups = (cols + 7) / 8;
  DevTrees dt;
  DevBuf dbins, dpreds, dleaf, dstatus;
  if (dt.put(T, tree_off, feature, sbin, flags, catmask, leaf, err) ||
      upload(dbins, bins, size_t(groups) * size_t(rows) * 8, err) ||
      dstatus.alloc(sizeof(unsigned), err))
    return -1;
  BN_CUDA(cudaMemset(dstatus.p, 0, sizeof(unsigned)), "cudaMemset");
  if (preds && upload(dpreds, preds, size_t(K) * size_t(rows), err)) return -1;
  if (leaf_idx && dleaf.alloc(size_t(T) * size_t(rows) * 4, err)) return -1;
  BinnedArgs a = tree_args(dt, T, rows, cols, num_bins, max_depth, K);
  a.bins = dbins.as<unsigned char>();
  a.preds = preds ? dpreds.as<float>() : nullptr;
  a.leaf_idx = leaf_idx ? dleaf.as<int>() : nullptr;
  a.err = dstatus.as<unsigned>();
  BN_CUDA(launch_binned(a, 0), "binned walk launch");
  g_kernel_launches.fetch_add(1);
  BN_CUDA(cudaDeviceSynchronize(), "binned walk");
  if (check_status(dstatus.as<unsigned>(), err)) return -1;
  if (preds)
    BN_CUDA(cudaMemcpy(preds, dpreds.p, size_t(K) * size_t(rows) * 4, cudaMemcpyDeviceToHost),
            "cudaMemcpy (preds)");
  if (leaf_idx)
    BN_CUDA(cudaMemcpy(leaf_idx, dleaf.p, size_t(T) * size_t(rows) * 4, cudaMemcpyDeviceToHost),
            "cudaMemcpy (leaf indices)");
  return 0;
}

int tree_binned_device(int device, const uint8_t* bins, int64_t rows, int64_t cols, int num_bins,
                       int T, const int64_t* tree_off, const int32_t* feature,
                       const uint32_t* sbin, const uint32_t* flags, const uint32_t* catmask,
                       const float* leaf, int max_depth, int K, float* preds, int32_t* leaf_idx,
                       unsigned* status, cudaStream_t stream, std::string& err) {
  if (rows < 0 || cols < 0 || K < 1 || T < 0 || max_depth < 0 || num_bins < 4 ||
      num_bins > 256 || !status) {
    err = "invalid argument";
    return -1;
  }
  if (rows == 0 || T == 0) return 0;
  if (check_device(device, err)) return -1;
  Guard gd(device);
  BinnedArgs a{};
  a.bins = bins;
  a.n = rows;
  a.cols = cols;
  a.num_bins = num_bins;
  a.T = T;
  a.tree_off = reinterpret_cast<const long long*>(tree_off);
  a.feature = feature;
  a.sbin = sbin;
  a.flags = flags;
  a.catmask = catmask;
  a.leaf = leaf;
  a.max_depth = max_depth;
  a.K = K;
  a.preds = preds;
  a.leaf_idx = leaf_idx;
  a.err = status;
  BN_CUDA(launch_binned(a, stream), "binned walk launch");
  g_kernel_launches.fetch_add(1);
  return 0;
}

namespace {

int dataset_slice(Engine& e, const Dataset& d, const SplitTrees& st, int kind, int device,
                  int64_t r0, int64_t r1, void* out, std::string& err) {
  if (r1 <= r0) return 0;
  Guard gd(device);
  const int T = int(st.tree_off.size()) - 1;
  const int K = e.model.K;
  const int64_t groups = (d.cols + 7) / 8;
  const int64_t ocols = output_cols(e, kind);
  DevTrees dt;
  DevBuf dbase, dbins, dout, dstatus;
  const size_t N = st.feature.size();
  std::vector<int64_t> off(st.tree_off.begin(), st.tree_off.end());
  if (dt.put(T, off.data(), st.feature.data(), st.sbin.data(), st.flags.data(),
             st.catmask.data(), st.leaf.data(), err) ||
      upload(dbase, e.model.base_scores.data(), e.model.base_scores.size(), err) ||
      dstatus.alloc(sizeof(unsigned), err))
    return -1;
  (void)N;
  BN_CUDA(cudaMemset(dstatus.p, 0, sizeof(unsigned)), "cudaMemset");
  const int64_t n = r1 - r0;
  int64_t C = std::max<int64_t>((int64_t(256) << 20) / std::max<int64_t>(ocols * 4, groups * 8),
                                1024);
  C = std::min(C, n);
  if (dbins.alloc(size_t(groups) * size_t(C) * 8, err) ||
      dout.alloc(size_t(C) * size_t(ocols) * 4, err))
    return -1;
  BinnedArgs a = tree_args(dt, T, 0, d.cols, d.num_bins, st.max_depth, K);
  a.forest_mode = 1;
  a.base = dbase.as<float>();
  a.err = dstatus.as<unsigned>();
  a.ka.kind = kind;
  a.ka.log_link = e.model.uses_log_link() ? 1 : 0;
  a.ka.binary = e.model.objective == kBinaryLogistic ? 1 : 0;
  a.ka.K = K;
  for (int64_t c0 = r0; c0 < r1; c0 += C) {
    const int64_t nr = std::min(C, r1 - c0);
    // rows [c0, c0 + nr) of every tile of the dataset -> a chunk matrix of nr rows
    BN_CUDA(cudaMemcpy2D(dbins.p, size_t(nr) * 8, d.bins.data() + c0 * 8, size_t(d.rows) * 8,
                         size_t(nr) * 8, size_t(groups), cudaMemcpyHostToDevice),
            "cudaMemcpy2D (bins)");
    a.bins = dbins.as<unsigned char>();
    a.n = nr;
    a.ka.out = kind == kKindLeaf ? nullptr : dout.as<float>();
    a.ka.out_leaf = kind == kKindLeaf ? dout.as<int>() : nullptr;
    BN_CUDA(launch_binned(a, 0), "binned forest launch");
    g_kernel_launches.fetch_add(1);
    BN_CUDA(cudaMemcpy(static_cast<char*>(out) + size_t(c0) * size_t(ocols) * 4, dout.p,
                       size_t(nr) * size_t(ocols) * 4, cudaMemcpyDeviceToHost),
            "cudaMemcpy (outputs)");
  }
  return check_status(dstatus.as<unsigned>(), err);
}

}  // namespace

int predict_dataset(Engine& e, const Dataset& d, int kind, const std::vector<int>& devices_in,
                    void* out, std::string& err) {
  if (kind < kKindPredict || kind > kKindCli) {
    err = "unknown output kind " + std::to_string(kind);
    return -1;
  }
  SplitTrees st;
  if (!model_split_form(e, d.edges.data(), d.cols, d.num_bins, st, err)) return -1;
  if (d.rows == 0) return 0;
  if (!out) {
    err = "null argument";
    return -1;
  }
  std::vector<int> devices = devices_in;
  if (devices.empty()) {
    int cur = 0;
    cudaGetDevice(&cur);
    devices.push_back(cur);
  }
  for (size_t i = 0; i < devices.size(); ++i) {
    if (check_device(devices[i], err)) return -1;
    for (size_t j = 0; j < i; ++j)
      if (devices[j] == devices[i]) {
        err = "device " + std::to_string(devices[i]) + " listed twice";
        return -1;
      }
  }
  const int nd = int(devices.size());
  std::vector<std::string> errs(static_cast<size_t>(nd));
  std::vector<int> rcs(static_cast<size_t>(nd), 0);
  std::vector<std::thread> th;
  for (int g = 0; g < nd; ++g) {
    const int64_t a = d.rows * g / nd, b = d.rows * (g + 1) / nd;
    auto job = [&, g, a, b] {
      rcs[size_t(g)] = dataset_slice(e, d, st, kind, devices[size_t(g)], a, b, out, errs[size_t(g)]);
    };
    if (nd == 1) {
      job();
      break;
    }
    try {
      th.emplace_back(job);
    } catch (...) {
      job();
    }
  }
  for (auto& t : th) t.join();
  for (int g = 0; g < nd; ++g)
    if (rcs[size_t(g)] != 0) {
      err = errs[size_t(g)];
      return -1;
    }
  return 0;
}

// ---- making and saving datasets --------------------------------------------

namespace {

std::string swift_float(float v) {
  char b[40];
  return std::string(b, format_float(v, b));
}

}  // namespace

void compute_edges(const float* x, int64_t rows, int64_t cols, int num_bins,
                   const std::vector<char>& categorical, std::vector<float>& edges) {
  const int data_bins = num_bins - 1;
  const int ne = data_bins - 1;
  const int64_t step = std::max<int64_t>(1, rows / 200000);
  edges.assign(size_t(cols) * size_t(ne), 0.0f);
  auto one = [&](int64_t f) {
    if (categorical[size_t(f)]) return;
    std::vector<float> sample;
    sample.reserve(size_t(rows / step + 1));
    for (int64_t i = 0; i < rows; i += step) {
      const float v = x[size_t(f) * size_t(rows) + size_t(i)];
      if (!std::isnan(v)) sample.push_back(v);
    }
    if (sample.empty()) return;  // all-NaN column
    std::stable_sort(sample.begin(), sample.end());
    const int64_t m = int64_t(sample.size());
    for (int k = 0; k < ne; ++k)
      edges[size_t(f) * size_t(ne) + size_t(k)] =
          sample[size_t(std::min(m - 1, (int64_t(k) + 1) * m / data_bins))];
  };
  const int nt = int(std::max<int64_t>(1, std::min<int64_t>(cols, std::thread::hardware_concurrency())));
  std::vector<std::thread> th;
  for (int t = 0; t < nt; ++t)
    th.emplace_back([&, t] {
      for (int64_t f = t; f < cols; f += nt) one(f);
    });
  for (auto& x_ : th) x_.join();
}

int make_dataset(int device, const float* x, int64_t rows, int64_t cols, const float* labels,
                 int num_bins, const std::vector<int64_t>& categorical,
                 const std::vector<std::string>* names, Dataset& d, std::string& err) {
  // MacBooster(params:) (Booster.swift:263-265), then makeDataset's checks in order
  if (num_bins < 4 || num_bins > 256) {
    err = "Invalid input: numBins must be in 4...256, got " + std::to_string(num_bins);
    return -1;
  }
  if (rows <= 0 || cols <= 0 || !x || !labels) {
    const int64_t r = std::max<int64_t>(rows, 0), c = std::max<int64_t>(cols, 0);
    err = "Invalid input: dataset shapes inconsistent (rows=" + std::to_string(rows) +
          ", cols=" + std::to_string(cols) + ", X=" + std::to_string(x ? r * c : 0) +
          ", y=" + std::to_string(labels ? r : 0) + ")";
    return -1;
  }
  for (int64_t i = 0; i < rows; ++i)
    if (!std::isfinite(labels[i])) {
      err = "Invalid input: label at row " + std::to_string(i) + " is " +
            swift_float(labels[i]) + "; labels must be finite";
      return -1;
    }
  std::vector<int64_t> cats(categorical);
  std::sort(cats.begin(), cats.end());
  cats.erase(std::unique(cats.begin(), cats.end()), cats.end());
  const int data_bins = num_bins - 1;
  std::vector<char> is_cat(size_t(cols), 0);
  for (int64_t f : cats) {
    // validateCategoricals (Booster.swift:1810-1826), features in ascending order
    if (f < 0 || f >= cols) {
      err = "Internal error: categorical feature index " + std::to_string(f) + " out of range";
      return -1;
    }
    is_cat[size_t(f)] = 1;
    for (int64_t i = 0; i < rows; ++i) {
      const float v = x[size_t(f) * size_t(rows) + size_t(i)];
      if (std::isnan(v)) continue;
      const float c = std::nearbyint(v);
      if (!(c >= 0.0f) || c >= float(data_bins)) {
        err = "Categorical feature " + std::to_string(f) + " has value " + swift_float(v) +
              "; expected integer ids in 0..<" + std::to_string(data_bins) + " or NaN";
        return -1;
      }
    }
  }
  d = Dataset();
  d.rows = rows;
  d.cols = cols;
  d.num_bins = num_bins;
  d.categorical = cats;
  if (names) {
    d.has_names = true;
    d.names = *names;
  }
  d.labels.assign(labels, labels + rows);
  compute_edges(x, rows, cols, num_bins, is_cat, d.edges);
  const int64_t groups = (cols + 7) / 8;
  d.bins.assign(size_t(groups) * 8 * size_t(rows), 0);
  std::vector<uint8_t> flags(is_cat.begin(), is_cat.end());
  return bin_data_host(device, x, rows, cols, 0, d.edges.data(), num_bins, flags.data(),
                       d.bins.data(), err);
}

bool save_mbds(const Dataset& d, const char* path, std::string& err) {
  std::string out;
  auto put32 = [&](uint32_t v) { out.append(reinterpret_cast<const char*>(&v), 4); };
  auto put64 = [&](uint64_t v) { out.append(reinterpret_cast<const char*>(&v), 8); };
  put32(0x4D424453u);
  put32(1);
  put32(8);
  put64(uint64_t(d.rows));
  put32(uint32_t(d.cols));
  put32(uint32_t(d.num_bins));
  put32(uint32_t(d.categorical.size()));
  for (int64_t c : d.categorical) put32(uint32_t(c));
  // feature names as Foundation's JSONEncoder writes a [String]: compact, with
  // '"', '\\' and '/' escaped and control characters as \b \f \n \r \t or \u00xx
  std::string names;
  if (d.has_names) {
    names = "[";
    for (size_t i = 0; i < d.names.size(); ++i) {
      if (i) names += ',';
      names += '"';
      for (unsigned char ch : d.names[i]) {
        switch (ch) {
          case '"': names += "\\\""; break;
          case '\\': names += "\\\\"; break;
          case '/': names += "\\/"; break;
          case '\b': names += "\\b"; break;
          case '\f': names += "\\f"; break;
          case '\n': names += "\\n"; break;
          case '\r': names += "\\r"; break;
          case '\t': names += "\\t"; break;
          default:
            if (ch < 0x20) {
              char u[8];
              std::snprintf(u, sizeof(u), "\\u%04x", ch);
              names += u;
            } else {
              names += char(ch);
            }
        }
      }
      names += '"';
    }
    names += "]";
  }
  put32(uint32_t(names.size()));
  out += names;
  put64(d.edges.size());
  out.append(reinterpret_cast<const char*>(d.edges.data()), d.edges.size() * 4);
  put64(d.labels.size());
  out.append(reinterpret_cast<const char*>(d.labels.data()), d.labels.size() * 4);
  put64(d.bins.size());
  out.append(reinterpret_cast<const char*>(d.bins.data()), d.bins.size());
  FILE* f = std::fopen(path, "wb");
  if (!f) {
    err = std::string("cannot write '") + path + "'";
    return false;
  }
  const bool ok = std::fwrite(out.data(), 1, out.size(), f) == out.size();
  if (std::fclose(f) != 0 || !ok) {
    err = std::string("error writing '") + path + "'";
    return false;
  }
  return true;
}

bool cli_dataset(const char* data_path, int format, const char* label, const char* categorical,
                 int num_bins, int device, const char* output_path, int64_t* rows_out,
                 int64_t* cols_out, std::string& err) {
  Table t;
  if (!read_table(data_path, format, ColumnChooser(), false, t, err)) return false;
  // prepare (main.swift:112-132)
  const std::string lname = label ? label : "label";
  int64_t lcol = -1;
  for (size_t c = 0; c < t.header.size(); ++c)
    if (t.header[c] == lname) {
      lcol = int64_t(c);
      break;
    }
  if (lcol < 0) {
    std::string cols;
    for (size_t c = 0; c < t.header.size(); ++c) cols += (c ? ", " : "") + t.header[c];
    err = "label column '" + lname + "' not found; columns: " + cols;
    return false;
  }
  const int64_t C = t.width();
  std::vector<int64_t> fcols;
  std::vector<std::string> names;
  for (int64_t c = 0; c < C; ++c)
    if (c != lcol) {
      fcols.push_back(c);
      names.push_back(t.header[size_t(c)]);
    }
  std::vector<int64_t> cats;
  if (categorical) {
    const std::string list(categorical);
    size_t s = 0;
    while (s <= list.size()) {
      const size_t e = list.find(',', s);
      const std::string name = list.substr(s, e == std::string::npos ? std::string::npos : e - s);
      if (!name.empty()) {
        const auto it = std::find(names.begin(), names.end(), name);
        if (it == names.end()) {
          err = "categorical column '" + name + "' not found among features";
          return false;
        }
        cats.push_back(int64_t(it - names.begin()));
      }
      if (e == std::string::npos) break;
      s = e + 1;
    }
  }
  const int64_t rows = t.rows, F = int64_t(fcols.size());
  std::vector<float> X, y(static_cast<size_t>(rows));
  try {
    X.resize(size_t(rows) * size_t(F));
  } catch (...) {
    err = "out of host memory";
    return false;
  }
  for (int64_t i = 0; i < rows; ++i) {
    const float* row = t.data + i * C;
    for (int64_t j = 0; j < F; ++j) X[size_t(j) * size_t(rows) + size_t(i)] = row[fcols[size_t(j)]];
    y[size_t(i)] = row[lcol];
  }
  Dataset d;
  if (make_dataset(device, X.data(), rows, F, y.data(), num_bins, cats, &names, d, err)) return false;
  if (!save_mbds(d, output_path, err)) return false;
  if (rows_out) *rows_out = rows;
  if (cols_out) *cols_out = F;
  return true;
}

}  // namespace mb
