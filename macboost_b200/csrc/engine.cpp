// Host engine (see engine.h).
//
// Predict from host memory, per GPU slice of rows:
//   chunk c (double-buffered, two streams):  H2D copy of the chunk's used
//   feature columns  ->  forest kernel  ->  D2H copy of the chunk's outputs.
// The D2H of chunk c is enqueued after the copy and kernel of chunk c+1, so a
// blocking copy into pageable host memory never stalls the next chunk.  Rows
// shard into contiguous ranges over the GPUs, one host thread per GPU; the
// model is replicated by host-to-device copy at prepare time and no
// collective is needed (rows are independent).
#include "engine.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <thread>

namespace mb {

std::atomic<unsigned long long> g_kernel_launches{0};

namespace {

std::string cuda_msg(const char* what, cudaError_t e) {
  return std::string(what) + ": " + cudaGetErrorString(e);
}

#define MB_CUDA(call, what)                  \
  do {                                       \
    cudaError_t e_ = (call);                 \
    if (e_ != cudaSuccess) {                 \
      err = cuda_msg(what, e_);              \
      return -1;                             \
    }                                        \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <class T>
int upload(T*& dst, const std::vector<T>& src, std::string& err) {
  const size_t bytes = std::max<size_t>(src.size() * sizeof(T), 16);
  MB_CUDA(cudaMalloc(reinterpret_cast<void**>(&dst), bytes), "cudaMalloc (model)");
  if (!src.empty())
    MB_CUDA(cudaMemcpy(dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice),
            "cudaMemcpy (model)");
  return 0;
}

int ensure(void*& buf, size_t& cap, size_t bytes, std::string& err) {
  if (bytes <= cap) return 0;
  if (buf) cudaFree(buf);
  buf = nullptr;
  cap = 0;
  MB_CUDA(cudaMalloc(&buf, bytes), "cudaMalloc (staging)");
  cap = bytes;
  return 0;
}

// Kernel family: 0 complete, 1 explicit, 2 complete with binned codes, 3 complete
// with the default direction carried as the record word (FlatForest::payload).
int layout_code(const FlatForest& f) { return f.codes ? 2 : (f.payload ? 3 : int(f.layout)); }

// Device-wait settings, read at each launch: MACBOOST_WAIT_LIMIT_US bounds
// every mbarrier wait of the forest kernels (2 s when unset or invalid), and
// MACBOOST_TEST_STALL_TILES=1 (a test hook, off by default) makes the row-tile
// waits run out with no copy in flight, to exercise the abort path.
void apply_wait_env(KArgs& a) {
  a.wait_ns = kDefaultWaitNs;
  if (const char* s = std::getenv("MACBOOST_WAIT_LIMIT_US")) {
    char* end = nullptr;
    const long long us = std::strtoll(s, &end, 10);
    if (end != s && us > 0 && us <= 60000000ll) a.wait_ns = (unsigned long long)us * 1000ull;
  }
  const char* st = std::getenv("MACBOOST_TEST_STALL_TILES");
  a.stall_tiles = (st && st[0] == '1') ? 1 : 0;
}

// The per-warp pipeline's chunk counters for launches on `s`: a pair of its
// own per stream, since launches on one stream never overlap and each leaves
// its pair at zero.  The per-thread default stream names a different stream
// on every host thread, so it (and a stream beyond the pool) gets none: the
// kernel then takes chunks in a fixed order.
unsigned long long* sched_for(const Engine& e, DeviceState& d, cudaStream_t s) {
  if (d.sched == nullptr || s == cudaStreamPerThread || !e.flat.plan.claim) return nullptr;
  std::lock_guard<std::mutex> lk(d.sched_mu);
  for (size_t i = 0; i < d.sched_streams.size(); ++i)
    if (d.sched_streams[i] == s) return d.sched + 2 * i;
  if (d.sched_streams.size() >= size_t(kSchedSlots)) return nullptr;
  d.sched_streams.push_back(s);
  return d.sched + 2 * (d.sched_streams.size() - 1);
}

// CTAs of one launch over `ntiles` row tiles: one wave of resident CTAs, or
// fewer under MACBOOST_PLAN "grid".
int grid_for(const FlatForest& f, const DeviceState& d, int64_t ntiles) {
  int64_t g = std::min<int64_t>(ntiles, d.grid_ctas);
  if (f.plan.grid_cap > 0) g = std::min<int64_t>(g, f.plan.grid_cap);
  return int(std::max<int64_t>(g, 1));
}

KArgs make_args(const Engine& e, const DeviceState& d, int kind) {
  const FlatForest& f = e.flat;
  KArgs a{};
  a.blob = d.blob;
  a.block_off = d.block_off;
  a.block_rec_base = d.block_rec_base;
  a.masks = d.masks;
  a.leaf_heap = d.leaf_heap;
  a.base = d.base;
  a.S_stage = f.S_stage;
  a.conv_src = d.conv_src;
  a.conv_dst = d.conv_dst;
  a.n_conv = int(f.conv_src.size());
  a.code_src = d.code_src;
  a.code_dst = d.code_dst;
  a.n_codes = int(f.code_src.size());
  a.K = f.K;
  a.G = f.G;
  a.T = f.T;
  a.D = f.D;
  a.Tb = f.plan.Tb;
  a.nblocks = f.plan.nblocks;
  a.buf_bytes = f.plan.buf_bytes;
  a.leaf_off = f.leaf_off;
  a.tile_bytes = f.plan.tile_bytes;
  a.bin_plan = d.bin_plan;
  a.search = d.search;
  a.search_depth = f.search_depth;
  a.code_tile_bytes = f.code_tile_bytes;
  a.neg_inf_slot = f.neg_inf_slot_bytes;
  a.compact_children = f.compact_children ? 1 : 0;
  a.data_bins = e.model.num_bins - 1;
  a.kind = kind;
  a.log_link = e.model.uses_log_link() ? 1 : 0;
  a.binary = e.model.objective == kBinaryLogistic ? 1 : 0;
  a.R = f.plan.R;
  a.tile_bufs = f.plan.tile_bufs;
  a.err = d.err;
  apply_wait_env(a);
  return a;
}

// Launch the forest kernel over `rows` rows of feature-major `x` (stride ld).
int launch(Engine& e, DeviceState& d, const float* x, int64_t rows, int64_t ld,
           const int* stage_feature, int kind, void* out, cudaStream_t s, std::string& err) {
  if (rows <= 0) return 0;
  KArgs a = make_args(e, d, kind);
  a.x = x;
  a.rows = rows;
  a.ld = ld;
  a.stage_feature = stage_feature;
  a.bulk = (reinterpret_cast<uintptr_t>(x) % 16 == 0 && ld % 4 == 0) ? 1 : 0;
  if (kind == kKindLeaf) {
    a.out = nullptr;
    a.out_leaf = static_cast<int*>(out);
  } else {
    a.out = static_cast<float*>(out);
    a.out_leaf = nullptr;
  }
  a.ntiles = (rows + a.R - 1) / a.R;
  a.sched = sched_for(e, d, s);
  const int grid = grid_for(e.flat, d, a.ntiles);
  cudaError_t ce = launch_forest(layout_code(e.flat), e.flat.plan.planes, e.model.any_cat, a,
                                 e.flat.plan.smem, grid, s, e.flat.code_bytes, e.top.get());
  if (ce != cudaSuccess) {
    err = cuda_msg("forest kernel launch", ce);
    return -1;
  }
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return 0;
}

}  // namespace

DeviceState::~DeviceState() {
  if (device < 0) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  for (auto* p : {static_cast<void*>(blob), static_cast<void*>(block_off),
                  static_cast<void*>(block_rec_base), static_cast<void*>(stage_feature),
                  static_cast<void*>(conv_src), static_cast<void*>(conv_dst),
                  static_cast<void*>(code_src), static_cast<void*>(code_dst),
                  static_cast<void*>(search), static_cast<void*>(bin_plan),
                  static_cast<void*>(masks), static_cast<void*>(leaf_heap),
                  static_cast<void*>(base), static_cast<void*>(err), static_cast<void*>(sched),
                  shap_paths, shap_uniq,
                  static_cast<void*>(shap_masks), static_cast<void*>(shap_block_path),
                  static_cast<void*>(shap_block_uniq), static_cast<void*>(shap_class_block),
                  static_cast<void*>(shap_coef), static_cast<void*>(shap_feature_slot),
                  static_cast<void*>(shap_slot_feature), static_cast<void*>(shap_bias),
                  static_cast<void*>(shap_scratch)})
    if (p) cudaFree(p);
  for (int i = 0; i < 2; ++i) {
    if (xbuf[i]) cudaFree(xbuf[i]);
    if (xraw[i]) cudaFree(xraw[i]);
    if (obuf[i]) cudaFree(obuf[i]);
    if (stream[i]) cudaStreamDestroy(stream[i]);
  }
  if (prev >= 0) cudaSetDevice(prev);
}

static Engine* finish_load(Engine* e, std::string& err) {
  if (!flatten_forest(e->model, e->flat, err)) {
    delete e;
    return nullptr;
  }
  e->description = describe_forest(e->flat);
  if (!e->flat.top_recs.empty() && !e->flat.codes && e->flat.layout == Layout::kComplete) {
    e->top = std::make_unique<TopRecords>();
    std::memset(e->top.get(), 0, sizeof(TopRecords));
    std::memcpy(e->top->rec, e->flat.top_recs.data(), e->flat.top_recs.size() * 8);
  }
  return e;
}

Engine* engine_load(const std::string& path, std::string& err) {
  auto* e = new Engine();
  if (!load_model_file(path, e->model, err)) {
    delete e;
    return nullptr;
  }
  return finish_load(e, err);
}

Engine* engine_from_json(const char* text, size_t len, std::string& err) {
  auto* e = new Engine();
  if (!parse_model_json(text, len, e->model, err)) {
    delete e;
    return nullptr;
  }
  return finish_load(e, err);
}

int64_t output_cols(const Engine& e, int kind) {
  if (kind == kKindLeaf) return e.flat.T;
  if (kind == kKindProba) return std::max(e.model.K, 2);
  return e.model.K;
}

DeviceState* engine_prepare(Engine& e, int device, std::string& err) {
  std::lock_guard<std::mutex> lk(e.mu);
  auto it = e.devices.find(device);
  if (it != e.devices.end()) return it->second.get();
  int ndev = 0;
  cudaError_t ce = cudaGetDeviceCount(&ndev);
  if (ce != cudaSuccess || ndev == 0) {
    err = ce != cudaSuccess ? cuda_msg("no CUDA device available", ce)
                            : std::string("no CUDA device available");
    return nullptr;
  }
  if (device < 0 || device >= ndev) {
    err = "device " + std::to_string(device) + " does not exist (" + std::to_string(ndev) +
          " visible)";
    return nullptr;
  }
  cudaDeviceProp prop{};
  ce = cudaGetDeviceProperties(&prop, device);
  if (ce != cudaSuccess) {
    err = cuda_msg("cudaGetDeviceProperties", ce);
    return nullptr;
  }
  if (prop.major != 10) {
    err = "device " + std::to_string(device) + " is sm_" + std::to_string(prop.major) +
          std::to_string(prop.minor) + "; this engine is built for sm_100a (B200)";
    return nullptr;
  }
  if (size_t(prop.sharedMemPerBlockOptin) < e.flat.plan.smem) {
    err = "device " + std::to_string(device) + " offers " +
          std::to_string(prop.sharedMemPerBlockOptin) + " bytes of shared memory per block, " +
          std::to_string(e.flat.plan.smem) + " needed";
    return nullptr;
  }
  DeviceGuard g(device);
  auto d = std::make_unique<DeviceState>();
  d->device = device;
  d->num_sms = prop.multiProcessorCount;
  d->smem_optin = size_t(prop.sharedMemPerBlockOptin);
  std::vector<float> base = e.model.base_scores;
  std::vector<unsigned long long> boff(e.flat.block_off.begin(), e.flat.block_off.end());
  if (boff.empty()) boff.push_back(0);
  std::vector<unsigned> rec_base(e.flat.block_rec_base.begin(), e.flat.block_rec_base.end());
  if (rec_base.empty()) rec_base.push_back(0);
  const std::vector<uint32_t>& mask_src = e.flat.codes ? e.flat.cat_masks : e.flat.full_masks;
  std::vector<unsigned> masks(mask_src.begin(), mask_src.end());
  std::vector<float> search(e.flat.search.begin(), e.flat.search.end());
  std::vector<int> bin_plan(e.flat.bin_plan.begin(), e.flat.bin_plan.end());
  std::vector<int> slots(e.flat.stage_feature.begin(), e.flat.stage_feature.end());
  std::vector<int> csrc(e.flat.conv_src.begin(), e.flat.conv_src.end());
  std::vector<int> cdst(e.flat.conv_dst.begin(), e.flat.conv_dst.end());
  std::vector<int> ksrc(e.flat.code_src.begin(), e.flat.code_src.end());
  std::vector<int> kdst(e.flat.code_dst.begin(), e.flat.code_dst.end());
  std::vector<int> heap(e.flat.leaf_heap.begin(), e.flat.leaf_heap.end());
  if (upload(d->blob, e.flat.blob, err) || upload(d->block_off, boff, err) ||
      upload(d->block_rec_base, rec_base, err) || upload(d->stage_feature, slots, err) ||
      upload(d->conv_src, csrc, err) || upload(d->conv_dst, cdst, err) ||
      upload(d->code_src, ksrc, err) || upload(d->code_dst, kdst, err) ||
      upload(d->search, search, err) || upload(d->bin_plan, bin_plan, err) ||
      upload(d->masks, masks, err) || upload(d->leaf_heap, heap, err) ||
      upload(d->base, base, err))
    return nullptr;
  if ((ce = cudaMalloc(reinterpret_cast<void**>(&d->err), sizeof(unsigned))) != cudaSuccess ||
      (ce = cudaMemset(d->err, 0, sizeof(unsigned))) != cudaSuccess) {
    err = cuda_msg("cudaMalloc (error word)", ce);
    return nullptr;
  }
  const size_t sched_bytes = size_t(kSchedSlots) * 2 * sizeof(unsigned long long);
  if ((ce = cudaMalloc(reinterpret_cast<void**>(&d->sched), sched_bytes)) != cudaSuccess ||
      (ce = cudaMemset(d->sched, 0, sched_bytes)) != cudaSuccess) {
    err = cuda_msg("cudaMalloc (chunk counters)", ce);
    return nullptr;
  }
  for (int i = 0; i < 2; ++i)
    if ((ce = cudaStreamCreateWithFlags(&d->stream[i], cudaStreamNonBlocking)) != cudaSuccess) {
      err = cuda_msg("cudaStreamCreate", ce);
      return nullptr;
    }
  int ctas = 0;
  ce = forest_occupancy(layout_code(e.flat), e.flat.plan.planes, e.model.any_cat, e.flat.K,
                        e.flat.G, e.flat.plan.R, e.flat.plan.smem, &ctas, e.flat.code_bytes,
                        e.top != nullptr);
  if (ce != cudaSuccess || ctas < 1) {
    err = ce != cudaSuccess ? cuda_msg("occupancy query", ce)
                            : std::string("the forest kernel cannot be resident on an SM");
    return nullptr;
  }
  d->grid_ctas = ctas * d->num_sms;
  if ((ce = cudaDeviceSynchronize()) != cudaSuccess) {
    err = cuda_msg("model upload", ce);
    return nullptr;
  }
  DeviceState* raw = d.get();
  e.devices.emplace(device, std::move(d));
  return raw;
}

namespace {

int check_err_word(DeviceState& d, std::string& err) {
  unsigned w = 0;
  MB_CUDA(cudaMemcpy(&w, d.err, sizeof(w), cudaMemcpyDeviceToHost), "reading kernel status");
  if (w != 0) {
    cudaMemset(d.err, 0, sizeof(unsigned));
    err = "device " + std::to_string(d.device) +
          ": a kernel gave up waiting for a shared-memory transfer (status " +
          std::to_string(w) + ")";
    return -1;
  }
  return 0;
}

// One GPU's share [r_begin, r_end) of a host-memory predict.
int run_slice(Engine& e, DeviceState& d, const float* x, int64_t rows, int64_t cols, int layout,
              int kind, int64_t r_begin, int64_t r_end, void* out, std::string& err) {
  std::lock_guard<std::mutex> lk(d.mu);
  DeviceGuard g(d.device);
  const int64_t n = r_end - r_begin;
  if (n <= 0) return 0;
  const FlatForest& f = e.flat;
  const int64_t S = f.S_stage;
  const int64_t ocols = output_cols(e, kind);
  const size_t oelem = 4;
  const int R = f.plan.R;
  // chunk rows: a multiple of the tile rows, <= 256 MB of staged input and of
  // output per buffer
  const int64_t in_row = std::max<int64_t>(layout == 1 ? cols : S, 1) * 4;
  const int64_t out_row = std::max<int64_t>(ocols, 1) * int64_t(oelem);
  const int64_t budget = int64_t(256) << 20;
  int64_t C = std::min(budget / in_row, budget / out_row);
  C = std::max<int64_t>(C / R * R, R);
  if (f.plan.chunk_rows > 0) C = std::max<int64_t>(f.plan.chunk_rows / 4 * 4, 4);
  if (C > n) C = (n + 3) / 4 * 4;
  const int64_t ldc = (C + 3) / 4 * 4;
  for (int p = 0; p < 2; ++p) {
    if (ensure(reinterpret_cast<void*&>(d.xbuf[p]), d.xcap[p],
               size_t(std::max<int64_t>(layout == 1 ? cols : S, 1)) * ldc * 4, err))
      return -1;
    if (layout == 1 &&
        ensure(reinterpret_cast<void*&>(d.xraw[p]), d.rcap[p], size_t(cols) * C * 4 + 16, err))
      return -1;
    if (ensure(d.obuf[p], d.ocap[p], size_t(ocols) * C * oelem + 16, err)) return -1;
  }
  // runs of consecutive used features (one 2-D copy each)
  std::vector<std::pair<int64_t, int64_t>> runs;  // (first feature, count)
  for (int64_t s = 0; s < S; ++s) {
    const int64_t feat = f.stage_feature[size_t(s)];
    if (!runs.empty() && runs.back().first + runs.back().second == feat)
      ++runs.back().second;
    else
      runs.push_back({feat, 1});
  }
  int64_t prev_r0 = -1, prev_n = 0;
  int prev_p = 0;
  auto drain = [&](int p, int64_t r0, int64_t nr) -> int {
    char* dst = static_cast<char*>(out) + size_t(r0) * ocols * oelem;
    MB_CUDA(cudaMemcpyAsync(dst, d.obuf[p], size_t(nr) * ocols * oelem, cudaMemcpyDeviceToHost,
                            d.stream[p]),
            "cudaMemcpyAsync (output)");
    return 0;
  };
  int c = 0;
  for (int64_t r0 = r_begin; r0 < r_end; r0 += C, ++c) {
    const int p = c & 1;
    const int64_t nr = std::min(C, r_end - r0);
    cudaStream_t s = d.stream[p];
    const int* slot_map = nullptr;
    if (layout == 0) {
      int64_t slot = 0;
      for (auto& run : runs) {
        MB_CUDA(cudaMemcpy2DAsync(d.xbuf[p] + slot * ldc, size_t(ldc) * 4,
                                  x + run.first * rows + r0, size_t(rows) * 4, size_t(nr) * 4,
                                  size_t(run.second), cudaMemcpyHostToDevice, s),
                "cudaMemcpy2DAsync (features)");
        slot += run.second;
      }
    } else {
      MB_CUDA(cudaMemcpyAsync(d.xraw[p], x + r0 * cols, size_t(nr) * cols * 4,
                              cudaMemcpyHostToDevice, s),
              "cudaMemcpyAsync (rows)");
      MB_CUDA(launch_transpose(d.xraw[p], nr, int(cols), d.xbuf[p], ldc, s), "transpose launch");
      slot_map = d.stage_feature;
    }
    if (launch(e, d, d.xbuf[p], nr, ldc, slot_map, kind, d.obuf[p], s, err)) return -1;
    if (prev_r0 >= 0 && drain(prev_p, prev_r0, prev_n)) return -1;
    prev_r0 = r0;
    prev_n = nr;
    prev_p = p;
  }
  if (prev_r0 >= 0 && drain(prev_p, prev_r0, prev_n)) return -1;
  MB_CUDA(cudaStreamSynchronize(d.stream[0]), "predict (stream 0)");
  MB_CUDA(cudaStreamSynchronize(d.stream[1]), "predict (stream 1)");
  return check_err_word(d, err);
}

}  // namespace

int engine_predict_host(Engine& e, const float* x, int64_t rows, int64_t cols, int layout,
                        int kind, const std::vector<int>& devices_in, void* out,
                        std::string& err) {
  if (rows < 0) {
    err = "rows must be >= 0";
    return -1;
  }
  if (cols != e.model.num_features) {
    err = "model expects " + std::to_string(e.model.num_features) + " features, got " +
          std::to_string(cols);
    return -1;
  }
  if (layout != 0 && layout != 1) {
    err = "layout must be 0 (feature-major) or 1 (row-major)";
    return -1;
  }
  if (kind < kKindPredict || kind > kKindCli) {
    err = "unknown output kind " + std::to_string(kind);
    return -1;
  }
  if (rows == 0) return 0;
  if (!x || !out) {
    err = "null argument";
    return -1;
  }
  std::vector<int> devices = devices_in;
  if (devices.empty()) {
    int cur = 0;
    cudaGetDevice(&cur);
    devices.push_back(cur);
  }
  std::vector<DeviceState*> ds;
  for (int dev : devices) {
    DeviceState* d = engine_prepare(e, dev, err);
    if (!d) return -1;
    if (std::find(ds.begin(), ds.end(), d) != ds.end()) {
      err = "device " + std::to_string(dev) + " listed twice";
      return -1;
    }
    ds.push_back(d);
  }
  const int nd = int(ds.size());
  if (nd == 1) return run_slice(e, *ds[0], x, rows, cols, layout, kind, 0, rows, out, err);
  std::vector<std::string> errs(static_cast<size_t>(nd));
  std::vector<int> rcs(static_cast<size_t>(nd), 0);
  std::vector<std::thread> th;
  for (int g = 0; g < nd; ++g) {
    const int64_t a = rows * g / nd, b = rows * (g + 1) / nd;
    try {
      th.emplace_back([&, g, a, b] {
        rcs[size_t(g)] = run_slice(e, *ds[size_t(g)], x, rows, cols, layout, kind, a, b, out,
                                   errs[size_t(g)]);
      });
    } catch (...) {
      rcs[size_t(g)] = run_slice(e, *ds[size_t(g)], x, rows, cols, layout, kind, a, b, out,
                                 errs[size_t(g)]);
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

int engine_predict_device(Engine& e, int device, const float* x, int64_t rows, int64_t cols,
                          int64_t ld, int layout, int kind, void* out, cudaStream_t stream,
                          std::string& err) {
  if (rows < 0) {
    err = "rows must be >= 0";
    return -1;
  }
  if (cols != e.model.num_features) {
    err = "model expects " + std::to_string(e.model.num_features) + " features, got " +
          std::to_string(cols);
    return -1;
  }
  if (kind < kKindPredict || kind > kKindCli) {
    err = "unknown output kind " + std::to_string(kind);
    return -1;
  }
  if (layout == 0 && ld < rows) {
    err = "feature-major input needs ld >= rows";
    return -1;
  }
  if (layout != 0 && layout != 1) {
    err = "layout must be 0 (feature-major) or 1 (row-major)";
    return -1;
  }
  if (rows == 0) return 0;
  if (!x || !out) {
    err = "null argument";
    return -1;
  }
  DeviceState* d = engine_prepare(e, device, err);
  if (!d) return -1;
  DeviceGuard g(device);
  if (layout == 0) return launch(e, *d, x, rows, ld, d->stage_feature, kind, out, stream, err);
  // Row-major device input: transpose into this device's staging buffer first;
  // the staging buffer is private to this call, so the call waits for it.
  std::lock_guard<std::mutex> lk(d->mu);
  const int64_t ldt = (rows + 3) / 4 * 4;
  if (ensure(reinterpret_cast<void*&>(d->xbuf[0]), d->xcap[0],
             size_t(std::max<int64_t>(cols, 1)) * ldt * 4, err))
    return -1;
  MB_CUDA(launch_transpose(x, rows, int(cols), d->xbuf[0], ldt, stream), "transpose launch");
  if (launch(e, *d, d->xbuf[0], rows, ldt, d->stage_feature, kind, out, stream, err)) return -1;
  MB_CUDA(cudaStreamSynchronize(stream), "predict (row-major device input)");
  return 0;
}

int engine_check_device(Engine& e, int device, std::string& err) {
  DeviceState* d = engine_prepare(e, device, err);
  if (!d) return -1;
  DeviceGuard g(device);
  MB_CUDA(cudaDeviceSynchronize(), "device synchronize");
  return check_err_word(*d, err);
}

int engine_launch_resident(Engine& e, int device, const float* x, int64_t rows, int64_t ld,
                           bool use_stage_map, int kind, void* out, unsigned* status,
                           unsigned long long* sched, cudaStream_t stream, std::string& err) {
  DeviceState* d = nullptr;
  {
    std::lock_guard<std::mutex> lk(e.mu);
    auto it = e.devices.find(device);
    if (it != e.devices.end()) d = it->second.get();
  }
  if (!d) {
    err = "the model is not resident on device " + std::to_string(device) +
          ": call macboost_prepare for that device first";
    return -1;
  }
  if (rows <= 0) return 0;
  DeviceGuard g(device);
  KArgs a = make_args(e, *d, kind);
  a.x = x;
  a.rows = rows;
  a.ld = ld;
  a.stage_feature = use_stage_map ? d->stage_feature : nullptr;
  a.bulk = (reinterpret_cast<uintptr_t>(x) % 16 == 0 && ld % 4 == 0) ? 1 : 0;
  a.out = kind == kKindLeaf ? nullptr : static_cast<float*>(out);
  a.out_leaf = kind == kKindLeaf ? static_cast<int*>(out) : nullptr;
  a.err = status;
  a.sched = e.flat.plan.claim ? sched : nullptr;
  a.ntiles = (rows + a.R - 1) / a.R;
  const int grid = grid_for(e.flat, *d, a.ntiles);
  cudaError_t ce = launch_forest(layout_code(e.flat), e.flat.plan.planes, e.model.any_cat, a,
                                 e.flat.plan.smem, grid, stream, e.flat.code_bytes, e.top.get());
  if (ce != cudaSuccess) {
    err = cuda_msg("forest kernel launch", ce);
    return -1;
  }
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return 0;
}

}  // namespace mb

// ---- TreeSHAP contributions -------------------------------------------------

namespace mb {
namespace {

int upload_bytes(void*& dst, const void* src, size_t bytes, std::string& err) {
  MB_CUDA(cudaMalloc(&dst, std::max<size_t>(bytes, 16)), "cudaMalloc (SHAP tables)");
  if (bytes) MB_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy (SHAP)");
  return 0;
}

bool ensure_shap_built(Engine& e, std::string& err) {
  std::lock_guard<std::mutex> lk(e.shap_mu);
  if (e.shap_state == 0) {
    std::string why;
    e.shap_state = build_shap(e.model, e.shap, why) ? 1 : -1;
    e.shap_err = why;
  }
  if (e.shap_state < 0) {
    err = e.shap_err;
    return false;
  }
  return true;
}

// Doubles of one scratch region of global TreeSHAP accumulators: S slots x R
// rows per CTA of the plan's grid.
size_t shap_region(const DeviceState& d, int S) {
  return size_t(d.shap_grid) * size_t(std::max(S, 1)) * size_t(d.shap_R);
}

// Upload the path tables to `d` and pick the launch plan (the row tile and
// where its float64 accumulators live, below).  Called with d.mu held.
int prepare_shap(Engine& e, DeviceState& d, std::string& err) {
  if (d.shap_ready) return 0;
  const ShapForest& s = e.shap;
  const int S = int(s.slot_feature.size());
  const int maxu = std::max(s.max_unique, 1);
  void* p = nullptr;
  if (upload_bytes(d.shap_paths, s.paths.data(), s.paths.size() * sizeof(ShapPathRec), err) ||
      upload_bytes(d.shap_uniq, s.uniq.data(), s.uniq.size() * sizeof(ShapUniqueRec), err))
    return -1;
  if (upload_bytes(p, s.masks.data(), s.masks.size() * 4, err)) return -1;
  d.shap_masks = static_cast<unsigned*>(p);
  if (upload_bytes(p, s.block_path.data(), s.block_path.size() * 4, err)) return -1;
  d.shap_block_path = static_cast<unsigned*>(p);
  if (upload_bytes(p, s.block_uniq.data(), s.block_uniq.size() * 4, err)) return -1;
  d.shap_block_uniq = static_cast<unsigned*>(p);
  if (upload_bytes(p, s.class_block.data(), s.class_block.size() * 4, err)) return -1;
  d.shap_class_block = static_cast<unsigned*>(p);
  if (upload_bytes(p, s.coef.data(), s.coef.size() * 8, err)) return -1;
  d.shap_coef = static_cast<double*>(p);
  if (upload_bytes(p, s.feature_slot.data(), s.feature_slot.size() * 4, err)) return -1;
  d.shap_feature_slot = static_cast<int*>(p);
  if (upload_bytes(p, s.slot_feature.data(), s.slot_feature.size() * 4, err)) return -1;
  d.shap_slot_feature = static_cast<int*>(p);
  if (upload_bytes(p, s.bias.data(), s.bias.size() * 4, err)) return -1;
  d.shap_bias = static_cast<float*>(p);
  // Candidates: row tile and float64 accumulators in shared memory (R = 256
  // ... 32), or, for paths of at most 8 distinct features, accumulators in a
  // global scratch (R = 128 or 64) that the L2 holds (at most
  // kShapScratchBytes), whose CTAs need no shared memory for them and so are
  // limited by registers only.  The plan keeps the most rows resident per SM;
  // shared memory wins ties.  B200, 100-feature models: depth-6 trees (cfg1,
  // cfg4) run 19-22% faster with 3 x 128 rows per SM in global memory than
  // with 1 x 256 in shared memory; the leaf-wise model (cfg5, paths of up to
  // 11 features, more accumulator updates per path) runs 15% slower.
  constexpr size_t kShapScratchBytes = size_t(64) << 20;
  int best_rows = 0;
  const int force_global = plan_shap_global_from_env();  // MACBOOST_PLAN "shapglobal=N"
  for (int R : {256, 128, 64, 32}) {
    if (force_global > 0) break;
    const size_t smem = shap_smem_bytes(maxu, true, S, R);
    if (smem > d.smem_optin) continue;
    int ctas = 0;
    MB_CUDA(shap_occupancy(maxu, true, R, smem, &ctas), "occupancy query (SHAP)");
    if (ctas * R > best_rows) {
      best_rows = ctas * R;
      d.shap_R = R;
      d.shap_smem = smem;
      d.shap_grid = ctas * d.num_sms;
      d.shap_in_smem = true;
    }
  }
  // The dense build (128 registers, four 128-row CTAs per SM) for single-class
  // models: cfg1 model 73.9 -> 66.5 ms; on the 10-class cfg4 model it measured
  // 1% slower than three CTAs of the 154-register build.
  const int dense_env = plan_shap_dense_from_env();
  for (int dense = 0; dense < 2; ++dense) {
    if (dense && (maxu > 12 || dense_env == 0 || (e.model.K > 1 && dense_env < 1))) break;
    for (int R : {128, 64}) {
      if (maxu > 8 && force_global == 0) break;
      if (dense && R != 128) continue;
      const size_t smem = shap_smem_bytes(maxu, false, S, R);
      int ctas = 0;
      MB_CUDA(shap_occupancy(maxu, false, R, smem, &ctas, dense != 0), "occupancy query (SHAP)");
      const size_t per_cta = size_t(std::max(S, 1)) * size_t(R) * sizeof(double);
      const int fit = int(std::min<size_t>(kShapScratchBytes / (per_cta * size_t(d.num_sms)), 64));
      ctas = std::min(ctas, force_global > 0 ? force_global : fit);
      if (ctas >= 1 && ctas * R > best_rows) {
        best_rows = ctas * R;
        d.shap_R = R;
        d.shap_smem = smem;
        d.shap_grid = ctas * d.num_sms;
        d.shap_in_smem = false;
        d.shap_dense = dense != 0;
      }
    }
  }
  if (best_rows == 0) {
    // very wide models: one 64-row CTA per SM with its accumulators in global memory
    const int R = 64;
    const size_t smem = shap_smem_bytes(maxu, false, S, R);
    int ctas = 0;
    MB_CUDA(shap_occupancy(maxu, false, R, smem, &ctas), "occupancy query (SHAP)");
    if (ctas < 1) {
      err = "the contributions kernel cannot be resident on an SM";
      return -1;
    }
    d.shap_R = R;
    d.shap_smem = smem;
    d.shap_grid = d.num_sms;
    d.shap_in_smem = false;
  }
  // two regions: the double-buffered chunks of a host-memory call run on two
  // streams at once, each with its own (the device entry point uses region 0
  // and waits for its kernel)
  if (!d.shap_in_smem)
    MB_CUDA(cudaMalloc(reinterpret_cast<void**>(&d.shap_scratch),
                       2 * shap_region(d, S) * sizeof(double)),
            "cudaMalloc (SHAP accumulators)");
  d.shap_ready = true;
  return 0;
}

// Enqueue the contributions kernel over `rows` rows of feature-major x
// (stride ld; slot_map null: x holds the staged slots in order), with global
// accumulators (when the plan has them) in scratch region `region` (0 or 1).
int launch_shap_on(Engine& e, DeviceState& d, const float* x, int64_t rows, int64_t ld,
                   const int* slot_map, float* out, cudaStream_t st, std::string& err,
                   int region = 0) {
  const ShapForest& s = e.shap;
  ShapArgs a{};
  a.x = x;
  a.rows = rows;
  a.ld = ld;
  a.slot_map = slot_map;
  a.S = int(s.slot_feature.size());
  a.paths = d.shap_paths;
  a.uniq = d.shap_uniq;
  a.masks = d.shap_masks;
  a.block_path = d.shap_block_path;
  a.block_uniq = d.shap_block_uniq;
  a.class_block = d.shap_class_block;
  a.err = d.err;
  a.coef = d.shap_coef;
  a.feature_slot = d.shap_feature_slot;
  a.bias = d.shap_bias;
  a.K = e.model.K;
  a.F = int(e.model.num_features);
  a.data_bins = e.model.num_bins - 1;
  a.out = out;
  a.scratch = d.shap_scratch ? d.shap_scratch + size_t(region) * shap_region(d, a.S) : nullptr;
  a.R = d.shap_R;
  a.ntiles = (rows + a.R - 1) / a.R;
  int64_t grid = std::min<int64_t>(d.shap_grid, a.ntiles);
  if (e.flat.plan.grid_cap > 0) grid = std::min<int64_t>(grid, e.flat.plan.grid_cap);
  MB_CUDA(launch_shap(a, std::max(s.max_unique, 1), d.shap_in_smem, d.shap_smem, int(grid), st,
                      d.shap_dense),
          "contributions kernel launch");
  g_kernel_launches.fetch_add(1);
  return 0;
}

// One GPU's share [r_begin, r_end) of a host-memory contributions call:
// double-buffered chunks as in run_slice (H2D of the used feature columns,
// kernel, D2H of the chunk's rows x K x (F + 1) block).
int run_contrib_slice(Engine& e, DeviceState& d, const float* x, int64_t rows, int64_t cols,
                      int layout, int64_t r_begin, int64_t r_end, float* out, std::string& err) {
  std::lock_guard<std::mutex> lk(d.mu);
  DeviceGuard g(d.device);
  if (prepare_shap(e, d, err)) return -1;
  const int64_t n = r_end - r_begin;
  if (n <= 0) return 0;
  const ShapForest& s = e.shap;
  const int S = int(s.slot_feature.size());
  const int K = e.model.K;
  const int64_t W = cols + 1;
  const int R = d.shap_R;
  const int64_t in_row = std::max<int64_t>(layout == 1 ? cols : S, 1) * 4;
  const int64_t out_row = int64_t(K) * W * 4;
  const int64_t budget = int64_t(256) << 20;
  int64_t C = std::min(budget / in_row, budget / out_row);
  C = std::max<int64_t>(C / R * R, R);
  if (e.flat.plan.chunk_rows > 0) C = std::max<int64_t>(e.flat.plan.chunk_rows / 4 * 4, 4);
  if (C > n) C = (n + 3) / 4 * 4;
  const int64_t ldc = (C + 3) / 4 * 4;
  for (int p = 0; p < 2; ++p) {
    if (ensure(reinterpret_cast<void*&>(d.xbuf[p]), d.xcap[p],
               size_t(std::max<int64_t>(layout == 1 ? cols : S, 1)) * ldc * 4, err))
      return -1;
    if (layout == 1 &&
        ensure(reinterpret_cast<void*&>(d.xraw[p]), d.rcap[p], size_t(cols) * C * 4 + 16, err))
      return -1;
    if (ensure(d.obuf[p], d.ocap[p], size_t(out_row) * C + 16, err)) return -1;
  }
  // runs of slots whose features are consecutive (one 2-D copy each)
  std::vector<std::pair<int64_t, int64_t>> runs;  // (first feature, count)
  for (int sl = 0; sl < S; ++sl) {
    const int64_t feat = s.slot_feature[size_t(sl)];
    if (!runs.empty() && runs.back().first + runs.back().second == feat)
      ++runs.back().second;
    else
      runs.push_back({feat, 1});
  }
  int64_t prev_r0 = -1, prev_n = 0;
  int prev_p = 0;
  auto drain = [&](int p, int64_t r0, int64_t nr) -> int {
    MB_CUDA(cudaMemcpyAsync(out + size_t(r0) * size_t(K * W), d.obuf[p], size_t(nr) * out_row,
                            cudaMemcpyDeviceToHost, d.stream[p]),
            "cudaMemcpyAsync (contributions)");
    return 0;
  };
  int c = 0;
  for (int64_t r0 = r_begin; r0 < r_end; r0 += C, ++c) {
    const int p = c & 1;
    const int64_t nr = std::min(C, r_end - r0);
    cudaStream_t st = d.stream[p];
    const int* slot_map = nullptr;
    if (layout == 0) {
      int64_t slot = 0;
      for (auto& run : runs) {
        MB_CUDA(cudaMemcpy2DAsync(d.xbuf[p] + slot * ldc, size_t(ldc) * 4,
                                  x + run.first * rows + r0, size_t(rows) * 4, size_t(nr) * 4,
                                  size_t(run.second), cudaMemcpyHostToDevice, st),
                "cudaMemcpy2DAsync (features)");
        slot += run.second;
      }
    } else {
      MB_CUDA(cudaMemcpyAsync(d.xraw[p], x + r0 * cols, size_t(nr) * cols * 4,
                              cudaMemcpyHostToDevice, st),
              "cudaMemcpyAsync (rows)");
      MB_CUDA(launch_transpose(d.xraw[p], nr, int(cols), d.xbuf[p], ldc, st), "transpose launch");
      slot_map = d.shap_slot_feature;
    }
    if (launch_shap_on(e, d, d.xbuf[p], nr, ldc, slot_map, static_cast<float*>(d.obuf[p]), st,
                       err, p))
      return -1;
    if (prev_r0 >= 0 && drain(prev_p, prev_r0, prev_n)) return -1;
    prev_r0 = r0;
    prev_n = nr;
    prev_p = p;
  }
  if (prev_r0 >= 0 && drain(prev_p, prev_r0, prev_n)) return -1;
  MB_CUDA(cudaStreamSynchronize(d.stream[0]), "contributions (stream 0)");
  MB_CUDA(cudaStreamSynchronize(d.stream[1]), "contributions (stream 1)");
  return check_err_word(d, err);
}

}  // namespace

int engine_contrib_device(Engine& e, int device, const float* x, int64_t rows, int64_t cols,
                          int64_t ld, int layout, float* out, cudaStream_t stream,
                          std::string& err) {
  if (rows < 0) {
    err = "rows must be >= 0";
    return -1;
  }
  if (cols != e.model.num_features) {
    err = "model expects " + std::to_string(e.model.num_features) + " features, got " +
          std::to_string(cols);
    return -1;
  }
  if (layout != 0 && layout != 1) {
    err = "layout must be 0 (feature-major) or 1 (row-major)";
    return -1;
  }
  if (layout == 0 && ld < rows) {
    err = "feature-major input needs ld >= rows";
    return -1;
  }
  if (!ensure_shap_built(e, err)) return -1;
  if (rows == 0) return 0;
  if (!x || !out) {
    err = "null argument";
    return -1;
  }
  DeviceState* d = engine_prepare(e, device, err);
  if (!d) return -1;
  std::lock_guard<std::mutex> lk(d->mu);
  DeviceGuard g(device);
  if (prepare_shap(e, *d, err)) return -1;
  bool wait = !d->shap_in_smem;  // the global accumulators are one region per device
  if (layout == 0) {
    if (launch_shap_on(e, *d, x, rows, ld, d->shap_slot_feature, out, stream, err)) return -1;
  } else {
    const int64_t ldt = (rows + 3) / 4 * 4;
    if (ensure(reinterpret_cast<void*&>(d->xbuf[0]), d->xcap[0],
               size_t(std::max<int64_t>(cols, 1)) * ldt * 4, err))
      return -1;
    MB_CUDA(launch_transpose(x, rows, int(cols), d->xbuf[0], ldt, stream), "transpose launch");
    if (launch_shap_on(e, *d, d->xbuf[0], rows, ldt, d->shap_slot_feature, out, stream, err))
      return -1;
    wait = true;  // the staging buffer is private to this call
  }
  if (wait) {
    MB_CUDA(cudaStreamSynchronize(stream), "contributions");
    return check_err_word(*d, err);
  }
  return 0;
}

int engine_contrib_host(Engine& e, const float* x, int64_t rows, int64_t cols, int layout,
                        const std::vector<int>& devices_in, float* out, std::string& err) {
  if (rows < 0) {
    err = "rows must be >= 0";
    return -1;
  }
  if (cols != e.model.num_features) {
    err = "model expects " + std::to_string(e.model.num_features) + " features, got " +
          std::to_string(cols);
    return -1;
  }
  if (layout != 0 && layout != 1) {
    err = "layout must be 0 (feature-major) or 1 (row-major)";
    return -1;
  }
  if (!ensure_shap_built(e, err)) return -1;
  if (rows == 0) return 0;
  if (!x || !out) {
    err = "null argument";
    return -1;
  }
  std::vector<int> devices = devices_in;
  if (devices.empty()) {
    int cur = 0;
    cudaGetDevice(&cur);
    devices.push_back(cur);
  }
  std::vector<DeviceState*> ds;
  for (int dev : devices) {
    DeviceState* d = engine_prepare(e, dev, err);
    if (!d) return -1;
    if (std::find(ds.begin(), ds.end(), d) != ds.end()) {
      err = "device " + std::to_string(dev) + " listed twice";
      return -1;
    }
    ds.push_back(d);
  }
  const int nd = int(ds.size());
  std::vector<std::string> errs(static_cast<size_t>(nd));
  std::vector<int> rcs(static_cast<size_t>(nd), 0);
  std::vector<std::thread> th;
  for (int gi = 0; gi < nd; ++gi) {
    const int64_t a = rows * gi / nd, b = rows * (gi + 1) / nd;
    auto job = [&, gi, a, b] {
      rcs[size_t(gi)] =
          run_contrib_slice(e, *ds[size_t(gi)], x, rows, cols, layout, a, b, out, errs[size_t(gi)]);
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
  for (int gi = 0; gi < nd; ++gi)
    if (rcs[size_t(gi)] != 0) {
      err = errs[size_t(gi)];
      return -1;
    }
  return 0;
}

}  // namespace mb
