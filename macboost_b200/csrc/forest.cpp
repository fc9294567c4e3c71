// Forest flattening and launch planning (layouts described in forest.h).
#include "forest.h"

#include "kernels.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>

namespace mb {

std::vector<int> group_options(int K) {
  // (class count, tree group) pairs with a dedicated kernel instantiation
  // (kernels_complete.cu / kernels_explicit.cu); other class counts use the
  // generic kernel (per-thread accumulators in local memory, group 8).
  switch (K) {
    case 1: return {16, 8};
    case 2: case 4: case 8: return {8};
    case 3: case 6: return {6};
    case 5: return {5};
    case 7: return {7};
    case 10: return {10};
    case 12: return {12};
    case 16: return {16};
    default: return {8};
  }
}

int max_threads_for_group(int K, int G) {
  // must match dev::Bounds (kernels_common.cuh); K outside the dedicated
  // instantiations runs the generic kernel (KT = 0)
  const bool dedicated = K >= 1 && K <= 8;  // else the generic kernel (KT = 0)
  if (G >= 12) return 256;
  if (G >= 10) return 384;
  if (!dedicated || K >= 5) return 512;
  return K <= 2 ? 768 : 640;
}

namespace {

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Optional restriction of the planner's choices from the environment, for
// tuning and tests: MACBOOST_PLAN="G=8,R=256,bufs=2,planes=0,grid=2,chunk=4096,claim=0,pay=0"
// (any subset; 0 = free).
struct PlanOverride {
  int G = 0, R = 0, bufs = 0, planes = -1, codes = -1, top = -1, grid = 0, claim = -1,
      shapglobal = 0, shapdense = -1, pay = -1;
  long chunk = 0;
  PlanOverride() {
    const char* s = std::getenv("MACBOOST_PLAN");
    if (!s) return;
    const char* p = s;
    while (*p) {
      const char* eq = std::strchr(p, '=');
      if (!eq) break;
      const std::string key(p, size_t(eq - p));
      char* end = nullptr;
      const long v = std::strtol(eq + 1, &end, 10);
      if (key == "G") G = int(v);
      else if (key == "R") R = int(v);
      else if (key == "bufs") bufs = int(v);
      else if (key == "planes") planes = int(v);
      else if (key == "codes") codes = int(v);
      else if (key == "top") top = int(v);
      else if (key == "grid") grid = int(v);
      else if (key == "claim") claim = int(v);
      else if (key == "shapglobal") shapglobal = int(v);
      else if (key == "shapdense") shapdense = int(v);
      else if (key == "pay") pay = int(v);
      else if (key == "chunk") chunk = v;
      p = end;
      while (*p == ',' || *p == ' ') ++p;
    }
  }
};

struct SlotPlan {
  std::vector<int32_t> stage_feature;   // staged slot -> feature
  std::vector<int32_t> raw_slot;        // feature -> staged slot (or -1)
  std::vector<int32_t> left_slot;       // feature -> -Inf slot (planes) (or -1)
  std::vector<int32_t> conv_src, conv_dst;
  std::vector<int32_t> code_slot;       // feature -> slot of its category codes (or -1)
  std::vector<int32_t> code_src, code_dst;
  int S_stage = 0, S_total = 0;
};

// Which features are read, and by which kinds of split.
void scan_usage(const Model& m, std::vector<char>& used, std::vector<char>& need_raw,
                std::vector<char>& need_left, std::vector<char>& numeric,
                std::vector<char>& categorical) {
  const size_t F = size_t(m.num_features);
  used.assign(F, 0);
  need_raw.assign(F, 0);
  need_left.assign(F, 0);
  numeric.assign(F, 0);
  categorical.assign(F, 0);
  for (const Tree& t : m.trees) {
    std::vector<int64_t> st{0};
    while (!st.empty()) {
      const int64_t o = st.back();
      st.pop_back();
      const int32_t f = t.feature[size_t(o)];
      if (f < 0) continue;
      used[size_t(f)] = 1;
      const uint32_t fl = t.flags[size_t(o)];
      if ((fl & kFlagCategorical) && !t.cat_mask.empty()) {
        need_raw[size_t(f)] = 1;  // categorical code from the raw value
        categorical[size_t(f)] = 1;
      } else {
        numeric[size_t(f)] = 1;
        if (fl & kFlagDefaultLeft)
          need_left[size_t(f)] = 1;
        else
          need_raw[size_t(f)] = 1;
      }
      st.push_back(2 * o + 1);
      st.push_back(2 * o + 2);
    }
  }
}

SlotPlan make_slots(const Model& m, bool planes) {
  std::vector<char> used, need_raw, need_left, numeric, categorical;
  scan_usage(m, used, need_raw, need_left, numeric, categorical);
  SlotPlan p;
  const size_t F = size_t(m.num_features);
  p.raw_slot.assign(F, -1);
  p.left_slot.assign(F, -1);
  for (size_t f = 0; f < F; ++f)
    if (used[f]) {
      p.raw_slot[f] = int32_t(p.stage_feature.size());
      p.stage_feature.push_back(int32_t(f));
    }
  p.S_stage = int(p.stage_feature.size());
  p.S_total = p.S_stage;
  // Category codes: a feature that only categorical splits read has its staged
  // values replaced by their codes; one that numeric splits read too gets a
  // slot of codes beside its values.
  p.code_slot.assign(F, -1);
  for (size_t f = 0; f < F; ++f) {
    if (!used[f] || !categorical[f]) continue;
    p.code_slot[f] = numeric[f] ? p.S_total++ : p.raw_slot[f];
    p.code_src.push_back(p.raw_slot[f]);
    p.code_dst.push_back(p.code_slot[f]);
  }
  if (planes) {
    for (size_t f = 0; f < F; ++f) {
      if (!used[f] || !need_left[f]) continue;
      if (need_raw[f]) {
        p.left_slot[f] = p.S_total++;
      } else {
        p.left_slot[f] = p.raw_slot[f];  // only default-left splits: convert in place
      }
      p.conv_src.push_back(p.raw_slot[f]);
      p.conv_dst.push_back(p.left_slot[f]);
    }
  }
  return p;
}

// Categorical and numeric node encoding.  Codes run over 0..dataBins
// (dataBins = the missing bin, _pyinfer.py:80-86); a mask whose bits 32 to
// dataBins all share one value compresses to word 0 plus that value.
uint2_like encode_split(const Tree& t, int64_t o, const SlotPlan& sp, bool planes, int R,
                        int data_bins, std::vector<uint32_t>& full_masks, bool payload = false) {
  const int32_t f = t.feature[size_t(o)];
  const uint32_t fl = t.flags[size_t(o)];
  const uint32_t row_bytes = uint32_t(R) * 4u;
  if ((fl & kFlagCategorical) && !t.cat_mask.empty()) {
    const uint32_t off = uint32_t(sp.code_slot[size_t(f)]) * row_bytes;  // the codes
    const uint32_t* w = &t.cat_mask[size_t(o) * 8];
    bool uniform = true;
    uint32_t hb = 0;
    if (data_bins >= 32) {
      hb = w[1] & 1u;
      for (int c = 33; c <= data_bins && uniform; ++c)
        uniform = ((w[c >> 5] >> (c & 31)) & 1u) == hb;
    }
    if (uniform) return uint2_like{off | kRecCategorical | (hb ? kRecDefaultLeft : 0u), w[0]};
    const uint32_t idx = uint32_t(full_masks.size() / 8);
    full_masks.insert(full_masks.end(), w, w + 8);
    return uint2_like{off | kRecCategorical | kRecFullMask, idx};
  }
  // Numeric (also a categorical flag in a tree without catMask: PyModel routes
  // it numerically, _pyinfer.py:79).
  uint32_t bits;
  std::memcpy(&bits, &t.threshold[size_t(o)], 4);
  const bool dl = (fl & kFlagDefaultLeft) != 0;
  if (planes) {
    const int32_t s = dl ? sp.left_slot[size_t(f)] : sp.raw_slot[size_t(f)];
    return uint2_like{uint32_t(s) * row_bytes, bits};
  }
  if (payload)
    return uint2_like{uint32_t(sp.raw_slot[size_t(f)]) * row_bytes |
                          (dl ? kRecPayloadLeft : kRecPayloadRight),
                      bits};
  return uint2_like{uint32_t(sp.raw_slot[size_t(f)]) * row_bytes | (dl ? kRecDefaultLeft : 0u),
                    bits};
}

// Group trees into blocks: `bytes(t0, n)` is the size of a block holding trees
// [t0, t0+n) (n a multiple of G).  Returns false if one group does not fit.
bool make_blocks(int ngroups, int G, size_t max_block,
                 const std::function<size_t(int, int)>& bytes,
                 std::vector<std::pair<int, int>>& blocks) {
  blocks.clear();
  int g = 0;
  while (g < ngroups) {
    if (bytes(g * G, G) > max_block) return false;
    int n = 1;
    while (g + n < ngroups && bytes(g * G, (n + 1) * G) <= max_block) ++n;
    blocks.push_back({g * G, n * G});
    g += n;
  }
  return true;
}

}  // namespace

static bool flatten_f32(const Model& m, FlatForest& f, std::string& err, int force_planes);

int plan_grid_cap_from_env() { return std::max(0, PlanOverride().grid); }
int plan_shap_global_from_env() { return std::max(0, PlanOverride().shapglobal); }
int plan_shap_dense_from_env() { return PlanOverride().shapdense; }

bool flatten_forest(const Model& m, FlatForest& f, std::string& err, int force_planes) {
  const PlanOverride ov;
  FlatForest coded;
  std::string why;
  const bool codes_ok = ov.codes != 0 && force_planes != 0 && flatten_codes(m, coded, why, ov.G, ov.R);
  if (codes_ok && ov.codes == 1) {
    f = std::move(coded);
  } else if (!flatten_f32(m, f, err, force_planes)) {
    if (!codes_ok) return false;
    f = std::move(coded);
  } else if (codes_ok && coded.plan.est_clk_per_row < f.plan.est_clk_per_row) {
    f = std::move(coded);
  }
  f.plan.grid_cap = std::max(0, ov.grid);
  f.plan.chunk_rows = std::max(0L, ov.chunk);
  f.plan.claim = ov.claim != 0;
  return true;
}

static bool flatten_f32(const Model& m, FlatForest& f, std::string& err, int force_planes) {
  f = FlatForest();
  f.T = int(m.trees.size());
  f.K = m.K;
  f.max_depth = m.max_depth;
  const int data_bins = m.num_bins - 1;
  const bool complete = std::max(1, m.max_depth) <= kMaxCompleteDepth;
  f.layout = complete ? Layout::kComplete : Layout::kExplicit;
  const int D = std::max(1, std::min(m.max_depth, 30));
  const int NL = 1 << std::min(D, kMaxCompleteDepth);  // complete: slots / leaves per tree

  // explicit layout: reachable nodes per tree and the mean leaf depth
  std::vector<int64_t> tree_nodes(size_t(f.T), 1);
  double avg_depth = D;
  if (!complete) {
    double depth_sum = 0;
    int64_t leaves = 0;
    for (int t = 0; t < f.T; ++t) {
      int64_t c = 0;
      std::vector<std::pair<int64_t, int>> st{{0, 0}};
      while (!st.empty()) {
        auto [o, d] = st.back();
        st.pop_back();
        ++c;
        if (m.trees[size_t(t)].feature[size_t(o)] >= 0) {
          st.push_back({2 * o + 1, d + 1});
          st.push_back({2 * o + 2, d + 1});
        } else {
          depth_sum += d;
          ++leaves;
        }
      }
      if (c > kMaxExplicitNodes) {
        err = "tree " + std::to_string(t) + " has more than 16384 reachable nodes";
        return false;
      }
      tree_nodes[size_t(t)] = c;
    }
    avg_depth = leaves ? depth_sum / double(leaves) : 1.0;
  }

  // --- launch plan: enumerate (group, rows per tile, buffers, planes) ------
  const SlotPlan sp_planes = make_slots(m, true);
  const SlotPlan sp_flat = make_slots(m, false);
  const bool any_left = !sp_planes.conv_dst.empty();
  struct Best {
    LaunchPlan p;
    int G = 0;
    std::vector<std::pair<int, int>> blocks;
    std::vector<size_t> node_prefix;
    double cost = 1e300;
  } best;
  const int Rs[] = {768, 640, 512, 384, 256, 128, 64, 32};
  const PlanOverride ov;
  if (ov.codes == 1) {
    err = "binned codes requested but not applicable";
    return false;
  }
  if (ov.planes >= 0 && force_planes < 0) force_planes = ov.planes;
  for (int G : group_options(m.K)) {
    if (ov.G && G != ov.G) continue;
    const int ngroups = (f.T + G - 1) / G;
    std::vector<size_t> node_prefix;  // explicit: prefix sums over padded trees
    if (!complete) {
      node_prefix.assign(size_t(ngroups) * G + 1, 0);
      for (size_t i = 0; i + 1 < node_prefix.size(); ++i)
        node_prefix[i + 1] = node_prefix[i] + size_t(i < tree_nodes.size() ? tree_nodes[i] : 1);
    }
    auto block_bytes = [&](int t0, int n) -> size_t {
      if (complete)
        return round_up(round_up(size_t(n) * NL * 8, 128) + size_t(n) * NL * 4, 128);
      const size_t head = round_up(16 + 4 * size_t(n + n / G), 16);
      return round_up(head + 8 * (node_prefix[size_t(t0 + n)] - node_prefix[size_t(t0)]), 128);
    };
    for (int pl = 1; pl >= 0; --pl) {
      const bool planes = pl == 1 && any_left;
      if (pl == 0 && !any_left) continue;  // identical to the planes variant
      if (force_planes == 0 && planes) continue;
      if (force_planes == 1 && !planes && any_left) continue;
      const SlotPlan& sp = planes ? sp_planes : sp_flat;
      // explicit layout: one more slot holding -Inf, read by leaf records
      const int S_tile = std::max(sp.S_total, 1) + (complete ? 0 : 1);
      for (int R : Rs) {
        if (R > max_threads_for_group(m.K, G) || (ov.R && R != ov.R)) continue;
        for (int bufs = 2; bufs >= 1; --bufs) {
          if (ov.bufs && bufs != ov.bufs) continue;
          const size_t tile = round_up(size_t(S_tile) * R * 4, 128);
          const size_t used = kSmemHeader + size_t(bufs) * tile;
          if (used > kSmemBudget) continue;
          const size_t avail = kSmemBudget - used;
          LaunchPlan p;
          p.R = R;
          p.tile_bufs = bufs;
          p.planes = planes;
          p.tile_bytes = uint32_t(tile);
          std::vector<std::pair<int, int>> blocks;
          if (ngroups == 0) {
            p.smem = used;
            p.note = "no trees";
          } else {
            const size_t whole = round_up(block_bytes(0, ngroups * G), 128);
            if (whole <= avail) {
              blocks = {{0, ngroups * G}};
              p.Tb = ngroups * G;
              p.nblocks = 1;
              p.buf_bytes = uint32_t(whole);
              p.smem = used + whole;
              p.note = "forest resident in shared memory";
            } else {
              const size_t max_block = (avail / 2) / 128 * 128;
              if (complete) {
                int Tb = 0;
                for (int t = G; t <= ngroups * G && block_bytes(0, t) <= max_block; t += G) Tb = t;
                if (Tb == 0) continue;
                // the block count (>= the minimum) that pads the fewest trees
                const int nb_min = (ngroups * G + Tb - 1) / Tb;
                int nb = nb_min, best_pad = 1 << 30;
                for (int c = nb_min; c <= nb_min + nb_min / 2 + 1; ++c) {
                  const int tb = ((ngroups + c - 1) / c) * G;
                  if (block_bytes(0, tb) > max_block) continue;
                  if (c * tb - f.T < best_pad) {
                    best_pad = c * tb - f.T;
                    nb = c;
                  }
                }
                Tb = ((ngroups + nb - 1) / nb) * G;
                for (int b = 0; b < nb; ++b) blocks.push_back({b * Tb, Tb});
                p.Tb = Tb;
              } else if (!make_blocks(ngroups, G, max_block, block_bytes, blocks)) {
                continue;
              }
              size_t mx = 0;
              for (auto& b : blocks) mx = std::max(mx, block_bytes(b.first, b.second));
              p.nblocks = int(blocks.size());
              p.buf_bytes = uint32_t(round_up(mx, 128));
              p.smem = used + 2 * size_t(p.buf_bytes);
              p.note = "forest streamed in tree blocks";
            }
          }
          // Cost model (SM clocks per row), calibrated on B200 (cfg2-like
          // depth-6 forests): a warp scores one tree in ~24 SM clocks when the
          // shared-memory pipe is saturated (~19 wavefronts: two per 8-byte
          // record load, one per gather, two for the leaf), ~28 without NaN
          // planes (23 on NaN-free row chunks, 29 on chunks with NaN, issue-
          // bound on the default-direction max and compare); saturation needs
          // warps more than per-thread tree groups: efficiency ~ (warps/16)^0.45
          // * (G/8)^0.15.  Staging uses the SM's share of HBM bandwidth
          // (~23 B/clk), hidden when double-buffered; streamed forest blocks
          // add barriers and L2 traffic.
          const int Tpad = blocks.empty() ? 0 : blocks.back().first + blocks.back().second;
          const double levels = complete ? double(D) : avg_depth * 1.15;
          const double per_tree = (planes || !any_left ? 24.0 : 28.0) * levels / 6.0 *
                                  (complete ? 1.0 : 1.3);
          const double warps = double(R) / 32.0;
          const double eff =
              std::min(1.0, std::pow(warps / 16.0, 0.45) * std::pow(double(G) / 8.0, 0.15));
          const double compute = double(Tpad) * per_tree / 32.0 / eff;
          const double load = double(sp.S_stage) * 4.0 / 23.0;
          const double stream =
              p.nblocks > 1
                  ? (double(blocks.size()) * 1500.0 + double(p.buf_bytes) * p.nblocks / 64.0) /
                        double(R)
                  : 0.0;
          // A resident forest runs the per-warp pipeline: a warp waiting for
          // its next chunk leaves the SM to the other warps, so with enough
          // warps (16 or more) one buffer hides the copies too (B200: cfg1 and
          // cfg3 at 4 and 8 warps ran 1.7-3x slower than streamed 16-warp
          // tiles).  Otherwise a single tile buffer exposes the bulk-copy
          // latency of each tile.
          const bool hidden = bufs == 2 || (p.nblocks == 1 && R >= 512);
          const double cost =
              (hidden ? std::max(compute, load) : compute + load + 2500.0 / double(R)) + stream;
          p.est_clk_per_row = cost;
          if (cost < best.cost * 0.999) {
            best.p = p;
            best.G = G;
            best.blocks = blocks;
            best.node_prefix = node_prefix;
            best.cost = cost;
          }
        }
      }
    }
  }
  if (best.p.R == 0) {
    err = "the forest's " + std::to_string(sp_flat.S_stage) +
          " used features do not fit a row tile in shared memory";
    return false;
  }
  f.plan = best.p;
  f.G = best.G;
  const std::vector<std::pair<int, int>>& blocks = best.blocks;
  const std::vector<size_t>& node_prefix = best.node_prefix;
  const int Gsel = best.G;
  auto block_bytes = [&](int t0, int n) -> size_t {
    if (complete)
      return round_up(round_up(size_t(n) * NL * 8, 128) + size_t(n) * NL * 4, 128);
    const size_t head = round_up(16 + 4 * size_t(n + n / Gsel), 16);
    return round_up(head + 8 * (node_prefix[size_t(t0 + n)] - node_prefix[size_t(t0)]), 128);
  };
  const SlotPlan& sp = f.plan.planes ? sp_planes : sp_flat;
  f.S_stage = sp.S_stage;
  f.S_total = sp.S_total;
  f.stage_feature = sp.stage_feature;
  f.conv_src = sp.conv_src;
  f.conv_dst = sp.conv_dst;
  f.code_src = sp.code_src;
  f.code_dst = sp.code_dst;
  const int R = f.plan.R;
  const int nb = int(blocks.size());
  f.Tpad = nb ? blocks.back().first + blocks.back().second : 0;

  // --- emit ------------------------------------------------------------------
  f.block_off.assign(size_t(nb) + 1, 0);
  for (int b = 0; b < nb; ++b)
    f.block_off[size_t(b) + 1] =
        f.block_off[size_t(b)] + block_bytes(blocks[size_t(b)].first, blocks[size_t(b)].second);
  f.blob.assign(size_t(f.block_off[size_t(nb)]), 0);
  const float neg_zero = -0.0f;
  uint32_t nz_bits;
  std::memcpy(&nz_bits, &neg_zero, 4);

  if (complete) {
    f.D = D;
    // Records carry the default direction as the walk's fmax operand (no
    // NaN planes, no categorical splits; B200 cfg4 5.57 -> 5.36 ms per 2M
    // rows).  A default-left record is 0xFF000000 | slot offset, a float at or
    // below -2^127 that replaces NaN (and any value below it) by a value left
    // of every threshold at or above -2^127; a forest with a default-left
    // threshold below that keeps the funnel-shift route.
    {
      const PlanOverride ov;
      bool ok = !f.plan.planes && !m.any_cat && ov.pay != 0;
      for (size_t t = 0; ok && t < m.trees.size(); ++t) {
        const Tree& tr = m.trees[t];
        for (size_t n = 0; ok && n < tr.feature.size(); ++n)
          if (tr.feature[n] >= 0 && (tr.flags[n] & kFlagDefaultLeft) &&
              !(tr.threshold[n] >= -0x1p127f))
            ok = false;
      }
      f.payload = ok;
    }
    const int Tb = f.plan.Tb;
    f.leaf_off = uint32_t(round_up(size_t(Tb) * NL * 8, 128));
    f.leaf_heap.assign(size_t(f.Tpad) * NL, -1);
    for (int t = 0; t < f.Tpad; ++t) {
      const int b = t / Tb, i = t % Tb;
      uint8_t* blk = f.blob.data() + f.block_off[size_t(b)];
      auto* slots = reinterpret_cast<uint2_like*>(blk) + size_t(i) * NL;  // heap n at n + 1
      auto* leaves = reinterpret_cast<float*>(blk + f.leaf_off) + size_t(i) * NL;
      int32_t* heap = f.leaf_heap.data() + size_t(t) * NL;
      if (t >= f.T) {
        for (int n = 0; n < NL; ++n) slots[n] = uint2_like{0u, 0u};
        for (int n = 0; n < NL; ++n) leaves[n] = neg_zero;
        continue;
      }
      const Tree& tr = m.trees[size_t(t)];
      const int NI = NL - 1;
      // (padded heap index p, original index o or -1, original leaf or -1, level)
      std::function<void(int64_t, int64_t, int64_t, int)> fill = [&](int64_t p, int64_t o,
                                                                     int64_t lf, int L) {
        if (L == D) {
          const int64_t src = lf >= 0 ? lf : o;
          leaves[p - NI] = tr.leaf[size_t(src)];
          heap[p - NI] = int32_t(src);
          return;
        }
        if (lf < 0 && tr.feature[size_t(o)] >= 0) {
          slots[p + 1] = encode_split(tr, o, sp, f.plan.planes, R, data_bins, f.full_masks,
                                       f.payload);
          fill(2 * p + 1, 2 * o + 1, -1, L + 1);
          fill(2 * p + 2, 2 * o + 2, -1, L + 1);
        } else {
          // padding split: both subtrees end in the same leaf
          const int64_t leaf_src = lf >= 0 ? lf : o;
          slots[p + 1] = uint2_like{0u, 0u};
          fill(2 * p + 1, -1, leaf_src, L + 1);
          fill(2 * p + 2, -1, leaf_src, L + 1);
        }
      };
      fill(0, 0, -1, 0);
      f.nodes += int64_t(NL) * 2 - 1;
    }
    // Heap nodes 0, 1, 2 (slots 1, 2, 3) of every tree for the kernel
    // parameter.  It removes the first two levels' shared-memory record loads,
    // which pays where those loads bound the walk: with NaN planes (one compare
    // per node), and with a resident forest, whose per-warp pipeline keeps the
    // shared-memory pipe busy (B200, cfg2 without planes: 4% faster).  With
    // streamed blocks and no planes the walk is bound by ALU issue (flag test
    // and compare select per node) and the constant-bank reads and selects only
    // add to it (B200: cfg1/cfg3 4.5% slower).
    const PlanOverride ov;
    if (D >= 2 && f.Tpad <= kTopTrees && ov.top != 0 &&
        (f.plan.planes || f.plan.nblocks == 1 || ov.top == 1)) {
      f.top_recs.resize(size_t(f.Tpad) * 3);
      for (int t = 0; t < f.Tpad; ++t) {
        const int b = t / Tb, i = t % Tb;
        const auto* slots = reinterpret_cast<const uint2_like*>(f.blob.data() + f.block_off[size_t(b)]) +
                            size_t(i) * NL;
        for (int k = 0; k < 3; ++k)
          f.top_recs[size_t(t) * 3 + size_t(k)] =
              uint64_t(slots[k + 1].x) | (uint64_t(slots[k + 1].y) << 32);
      }
    }
  } else {
    f.leaf_heap.assign(node_prefix.back(), -1);
    f.block_rec_base.assign(size_t(nb), 0);
    uint32_t max_delta = 0;
    // Leaf records loop on themselves: they read the constant -Inf slot (the
    // tile slot after all staged and -Inf-plane slots) with the default-left
    // flag, so go_right = (-Inf > leaf value) is 0, and their child distance is
    // 0; every tree of a group can then take the same number of steps (the
    // group's deepest leaf) and end on its leaf, whose value is the record's y.
    const uint32_t leaf_x =
        uint32_t(std::max(sp.S_total, 1)) * uint32_t(R) * 4u | kRecDefaultLeft;
    f.neg_inf_slot_bytes = uint32_t(std::max(sp.S_total, 1)) * uint32_t(R) * 4u;
    for (int b = 0; b < nb; ++b) {
      const int t0 = blocks[size_t(b)].first, n = blocks[size_t(b)].second;
      uint8_t* blk = f.blob.data() + f.block_off[size_t(b)];
      auto* head = reinterpret_cast<uint32_t*>(blk);
      head[0] = uint32_t(n);
      head[1] = uint32_t(t0);
      const size_t rec_off = round_up(16 + 4 * size_t(n + n / Gsel), 16);
      auto* recs = reinterpret_cast<uint2_like*>(blk + rec_off);
      const size_t base = node_prefix[size_t(t0)];
      f.block_rec_base[size_t(b)] = uint32_t(base);
      for (int i = 0; i < n; ++i) {
        const int t = t0 + i;
        const uint32_t start = uint32_t(node_prefix[size_t(t)] - base);
        head[4 + i] = start;
        uint2_like* r = recs + start;
        int32_t* heap = f.leaf_heap.data() + node_prefix[size_t(t)];
        uint32_t& steps = head[4 + n + i / Gsel];  // per group: its deepest leaf
        if (i % Gsel == 0) steps = 0;
        if (t >= f.T) {
          r[0] = uint2_like{leaf_x, nz_bits};
          continue;
        }
        const Tree& tr = m.trees[size_t(t)];
        steps = std::max<uint32_t>(steps, uint32_t(tr.depth));
        std::vector<int64_t> order{0};
        uint32_t next = 1;
        for (size_t q = 0; q < order.size(); ++q) {
          const int64_t o = order[q];
          if (tr.feature[size_t(o)] < 0) {
            uint32_t bits;
            std::memcpy(&bits, &tr.leaf[size_t(o)], 4);
            r[q] = uint2_like{leaf_x, bits};
            heap[q] = int32_t(o);
            continue;
          }
          uint2_like rec = encode_split(tr, o, sp, f.plan.planes, R, data_bins, f.full_masks);
          const uint32_t delta = next - uint32_t(q);
          if (delta > kMaxChildDelta) {
            err = "tree " + std::to_string(t) + " is too wide for the explicit layout";
            return false;
          }
          rec.x |= delta << kRecChildShift;
          max_delta = std::max(max_delta, delta);
          r[q] = rec;
          order.push_back(2 * o + 1);
          order.push_back(2 * o + 2);
          next += 2;
        }
        f.nodes += int64_t(order.size());
      }
    }
    // With every child distance at most kMaxCompactDelta, store 8 x the
    // distance: the walk then adds the field to the record address directly.
    f.compact_children = max_delta <= kMaxCompactDelta;
    if (f.compact_children) {
      for (int b = 0; b < nb; ++b) {
        const int t0 = blocks[size_t(b)].first, n = blocks[size_t(b)].second;
        uint8_t* blk = f.blob.data() + f.block_off[size_t(b)];
        const size_t rec_off = round_up(16 + 4 * size_t(n + n / Gsel), 16);
        auto* recs = reinterpret_cast<uint2_like*>(blk + rec_off);
        const size_t count = node_prefix[size_t(t0 + n)] - node_prefix[size_t(t0)];
        for (size_t q = 0; q < count; ++q) {
          const uint32_t d = recs[q].x >> kRecChildShift;
          recs[q].x = (recs[q].x & ((1u << kRecChildShift) - 1u)) | ((d * 8u) << kRecChildShift);
        }
      }
    }
  }
  if (f.full_masks.empty()) f.full_masks.assign(8, 0u);
  if (f.leaf_heap.empty()) f.leaf_heap.assign(1, -1);
  return true;
}

std::string describe_forest(const FlatForest& f) {
  char est[64];
  std::snprintf(est, sizeof(est), "%.2f", f.plan.est_clk_per_row);
  std::string s = "{";
  s += "\"layout\":\"" + std::string(f.layout == Layout::kComplete ? "complete" : "explicit") + "\"";
  s += ",\"trees\":" + std::to_string(f.T);
  s += ",\"padded_trees\":" + std::to_string(f.Tpad);
  s += ",\"group\":" + std::to_string(f.G);
  s += ",\"classes\":" + std::to_string(f.K);
  s += ",\"slots\":" + std::to_string(f.S_stage);
  s += ",\"tile_slots\":" + std::to_string(f.S_total);
  s += ",\"nan_planes\":" + std::string(f.plan.planes ? "true" : "false");
  s += ",\"codes\":" + std::string(f.codes ? "true" : "false");
  s += ",\"top_params\":" + std::string(f.top_recs.empty() ? "false" : "true");
  s += ",\"payload_records\":" + std::string(f.payload ? "true" : "false");
  if (f.layout == Layout::kExplicit)
    s += ",\"compact_children\":" + std::string(f.compact_children ? "true" : "false");
  if (f.codes) {
    s += ",\"code_bytes\":" + std::to_string(f.code_bytes);
    s += ",\"code_slots\":" + std::to_string(f.S_code);
    s += ",\"search_depth\":" + std::to_string(f.search_depth);
  }
  s += ",\"depth\":" + std::to_string(f.layout == Layout::kComplete ? f.D : f.max_depth);
  s += ",\"rows_per_tile\":" + std::to_string(f.plan.R);
  s += ",\"tile_buffers\":" + std::to_string(f.plan.tile_bufs);
  s += ",\"blocks\":" + std::to_string(f.plan.nblocks);
  s += ",\"block_buffer_bytes\":" + std::to_string(f.plan.buf_bytes);
  s += ",\"smem_bytes\":" + std::to_string(f.plan.smem);
  s += ",\"forest_bytes\":" + std::to_string(f.blob.size());
  s += ",\"full_masks\":" + std::to_string(f.full_masks.size() / 8);
  s += ",\"est_clk_per_row\":" + std::string(est);
  s += ",\"plan\":\"" + f.plan.note + "\"";
  if (f.plan.grid_cap > 0) s += ",\"grid_cap\":" + std::to_string(f.plan.grid_cap);
  if (f.plan.chunk_rows > 0) s += ",\"chunk_rows\":" + std::to_string(f.plan.chunk_rows);
  if (!f.plan.claim) s += ",\"claim\":false";
  s += "}";
  return s;
}

}  // namespace mb
