// Forest flattening and launch planning (layouts described in forest.h).
#include "forest.h"

#include <algorithm>
#include <cstring>
#include <functional>
#include <set>

namespace mb {
namespace {

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Categorical node encoding shared by both layouts.  Codes run over
// 0..dataBins (dataBins = the missing bin, _pyinfer.py:80-86); when every mask
// bit from 32 to dataBins has the same value the mask compresses to word 0
// plus that value.
uint2_like encode_split(const Tree& t, int64_t o, uint32_t slot_field, int data_bins,
                        std::vector<uint32_t>& full_masks) {
  const uint32_t fl = t.flags[size_t(o)];
  if ((fl & kFlagCategorical) && !t.cat_mask.empty()) {
    const uint32_t* w = &t.cat_mask[size_t(o) * 8];
    bool uniform = true;
    uint32_t hb = 0;
    if (data_bins >= 32) {
      hb = w[1] & 1u;
      for (int c = 33; c <= data_bins && uniform; ++c)
        uniform = ((w[c >> 5] >> (c & 31)) & 1u) == hb;
    }
    if (uniform) return uint2_like{slot_field | kRecCategorical | (hb ? kRecDefaultLeft : 0u), w[0]};
    const uint32_t idx = uint32_t(full_masks.size() / 8);
    full_masks.insert(full_masks.end(), w, w + 8);
    return uint2_like{slot_field | kRecCategorical | kRecFullMask, idx};
  }
  // Numeric (also a categorical flag in a tree without catMask: PyModel routes
  // it numerically, _pyinfer.py:79).
  uint32_t bits;
  std::memcpy(&bits, &t.threshold[size_t(o)], 4);
  return uint2_like{slot_field | ((fl & kFlagDefaultLeft) ? kRecDefaultLeft : 0u), bits};
}

struct Candidate {
  int R, bufs;
  bool resident;
};
// Preference: the whole forest resident in shared memory with double-buffered
// row tiles; then resident with a single tile buffer; then the forest streamed
// through two block buffers.
const Candidate kCandidates[] = {{512, 2, true},  {256, 2, true},  {256, 1, true},
                                 {128, 2, true},  {128, 1, true},  {256, 2, false},
                                 {256, 1, false}, {128, 2, false}, {128, 1, false},
                                 {64, 1, false},  {32, 1, false}};

// Group the forest's trees into blocks.  `group_bytes(g0, ntrees)` is the
// byte size of a block holding trees [g0, g0+ntrees) (ntrees a multiple of G;
// trees past T are padding).  Returns false if a single group does not fit.
bool make_blocks(int Tpad_groups, int G, size_t max_block,
                 const std::function<size_t(int, int)>& block_bytes,
                 std::vector<std::pair<int, int>>& blocks) {
  blocks.clear();
  int g = 0;
  while (g < Tpad_groups) {
    int n = 1;
    if (block_bytes(g * G, G) > max_block) return false;
    while (g + n < Tpad_groups && block_bytes(g * G, (n + 1) * G) <= max_block) ++n;
    blocks.push_back({g * G, n * G});
    g += n;
  }
  return true;
}

}  // namespace

bool flatten_forest(const Model& m, FlatForest& f, std::string& err) {
  f = FlatForest();
  f.T = int(m.trees.size());
  f.K = m.K;
  f.G = group_size(m.K);
  f.max_depth = m.max_depth;
  const int data_bins = m.num_bins - 1;

  // Slots: the features some reachable split reads, in increasing order.
  std::vector<int32_t> slot_of(size_t(m.num_features), -1);
  {
    std::vector<char> used(size_t(m.num_features), 0);
    for (const Tree& t : m.trees) {
      std::vector<int64_t> st{0};
      while (!st.empty()) {
        int64_t o = st.back();
        st.pop_back();
        if (t.feature[size_t(o)] < 0) continue;
        used[size_t(t.feature[size_t(o)])] = 1;
        st.push_back(2 * o + 1);
        st.push_back(2 * o + 2);
      }
    }
    for (int64_t i = 0; i < m.num_features; ++i)
      if (used[size_t(i)]) {
        slot_of[size_t(i)] = int32_t(f.slot_feature.size());
        f.slot_feature.push_back(int32_t(i));
      }
  }
  f.S = int(f.slot_feature.size());

  const bool complete = std::max(1, m.max_depth) <= kMaxCompleteDepth;
  f.layout = complete ? Layout::kComplete : Layout::kExplicit;
  const int Tgroups = (f.T + f.G - 1) / f.G;

  // --- per-layout sizes --------------------------------------------------
  const int D = std::max(1, m.max_depth);
  const int NI = (1 << std::min(D, 30)) - 1, NL = 1 << std::min(D, 30);
  std::vector<int64_t> tree_nodes;  // explicit: records per tree (padding trees: 1)
  std::vector<size_t> node_prefix;  // explicit: prefix sums over padded trees
  if (!complete) {
    if (f.S > kMaxExplicitSlots) {
      err = "explicit layout supports at most 4096 used features";
      return false;
    }
    tree_nodes.assign(size_t(Tgroups) * f.G, 1);
    for (int t = 0; t < f.T; ++t) {
      int64_t cnt = 0;
      std::vector<int64_t> st{0};
      while (!st.empty()) {
        int64_t o = st.back();
        st.pop_back();
        ++cnt;
        if (m.trees[size_t(t)].feature[size_t(o)] >= 0) {
          st.push_back(2 * o + 1);
          st.push_back(2 * o + 2);
        }
      }
      if (cnt > kMaxExplicitNodes) {
        err = "tree " + std::to_string(t) + " has more than 65535 reachable nodes";
        return false;
      }
      tree_nodes[size_t(t)] = cnt;
    }
    node_prefix.assign(tree_nodes.size() + 1, 0);
    for (size_t i = 0; i < tree_nodes.size(); ++i)
      node_prefix[i + 1] = node_prefix[i] + size_t(tree_nodes[i]);
  }
  auto block_bytes = [&](int t0, int n) -> size_t {
    if (complete) return round_up(round_up(size_t(n) * NI * 8, 16) + size_t(n) * NL * 4, 16);
    const size_t head = round_up(16 + 4 * size_t(n), 16);
    return round_up(head + 8 * (node_prefix[size_t(t0 + n)] - node_prefix[size_t(t0)]), 16);
  };

  // --- launch plan -------------------------------------------------------
  std::vector<std::pair<int, int>> blocks;
  LaunchPlan plan;
  const int64_t S = std::max(f.S, 1);  // one slot even when no split reads a feature
  for (const Candidate& c : kCandidates) {
    const size_t tile = round_up(size_t(S) * c.R * 4, 128);
    const size_t used = kSmemHeader + size_t(c.bufs) * tile;
    if (used > kSmemBudget) continue;
    const size_t avail = kSmemBudget - used;
    if (Tgroups == 0) {
      plan = LaunchPlan{c.R, c.bufs, 0, 0, 0, used, "no trees"};
      blocks.clear();
      break;
    }
    if (c.resident) {
      const size_t need = round_up(block_bytes(0, Tgroups * f.G), 128);
      if (need > avail) continue;
      blocks = {{0, Tgroups * f.G}};
      plan = LaunchPlan{c.R, c.bufs, Tgroups * f.G, 1, uint32_t(need), used + need,
                        "forest resident in shared memory"};
      break;
    }
    const size_t max_block = (avail / 2) / 128 * 128;
    if (complete) {
      // equal blocks: the largest multiple of G trees that fits, rebalanced
      int Tb = 0;
      for (int t = f.G; t <= Tgroups * f.G && block_bytes(0, t) <= max_block; t += f.G) Tb = t;
      const int min_tb = (c.bufs > 1) ? std::min(4 * f.G, Tgroups * f.G) : f.G;
      if (Tb < min_tb) continue;
      const int nb = (Tgroups * f.G + Tb - 1) / Tb;
      Tb = int(round_up(size_t((Tgroups * f.G + nb - 1) / nb), size_t(f.G)));
      blocks.clear();
      for (int b = 0; b < nb; ++b) blocks.push_back({b * Tb, Tb});
      const size_t bb = round_up(block_bytes(0, Tb), 128);
      plan = LaunchPlan{c.R, c.bufs, Tb, nb, uint32_t(bb), used + 2 * bb,
                        "forest streamed in tree blocks"};
      break;
    }
    if (!make_blocks(Tgroups, f.G, max_block, block_bytes, blocks)) continue;
    const double avg = double(Tgroups * f.G) / double(blocks.size());
    if (c.bufs > 1 && avg < 4.0 * f.G && blocks.size() > 1) continue;
    size_t mx = 0;
    for (auto& b : blocks) mx = std::max(mx, block_bytes(b.first, b.second));
    mx = round_up(mx, 128);
    plan = LaunchPlan{c.R, c.bufs, 0, int(blocks.size()), uint32_t(mx), used + 2 * mx,
                      "forest streamed in tree blocks"};
    break;
  }
  if (plan.R == 0) {
    err = "the forest's " + std::to_string(f.S) +
          " used features do not fit a row tile in shared memory";
    return false;
  }
  f.plan = plan;
  const int nb = int(blocks.size());
  f.Tpad = nb ? blocks.back().first + blocks.back().second : 0;

  // --- emit ----------------------------------------------------------------
  f.block_off.assign(size_t(nb) + 1, 0);
  for (int b = 0; b < nb; ++b)
    f.block_off[size_t(b) + 1] = f.block_off[size_t(b)] + block_bytes(blocks[size_t(b)].first,
                                                                      blocks[size_t(b)].second);
  f.blob.assign(size_t(f.block_off[size_t(nb)]), 0);
  const float neg_zero = -0.0f;
  uint32_t nz_bits;
  std::memcpy(&nz_bits, &neg_zero, 4);

  if (complete) {
    f.D = D;
    const int Tb = plan.Tb;
    f.leaf_off = uint32_t(round_up(size_t(Tb) * NI * 8, 16));
    f.leaf_heap.assign(size_t(f.Tpad) * NL, -1);
    for (int t = 0; t < f.Tpad; ++t) {
      const int b = t / Tb, i = t % Tb;
      uint8_t* blk = f.blob.data() + f.block_off[size_t(b)];
      auto* recs = reinterpret_cast<uint2_like*>(blk) + size_t(i) * NI;
      auto* leaves = reinterpret_cast<float*>(blk + f.leaf_off) + size_t(i) * NL;
      int32_t* heap = f.leaf_heap.data() + size_t(t) * NL;
      if (t >= f.T) {
        for (int n = 0; n < NI; ++n) recs[n] = uint2_like{0u, 0u};
        for (int n = 0; n < NL; ++n) leaves[n] = neg_zero;
        continue;
      }
      const Tree& tr = m.trees[size_t(t)];
      // (padded index p, original index o or -1, original leaf or -1, level)
      std::function<void(int64_t, int64_t, int64_t, int)> fill = [&](int64_t p, int64_t o,
                                                                     int64_t lf, int L) {
        if (L == D) {
          const int64_t src = lf >= 0 ? lf : o;
          leaves[p - NI] = tr.leaf[size_t(src)];
          heap[p - NI] = int32_t(src);
          return;
        }
        if (lf < 0 && tr.feature[size_t(o)] >= 0) {
          const uint32_t slot = uint32_t(slot_of[size_t(tr.feature[size_t(o)])]);
          recs[p] = encode_split(tr, o, slot << 4, data_bins, f.full_masks);
          fill(2 * p + 1, 2 * o + 1, -1, L + 1);
          fill(2 * p + 2, 2 * o + 2, -1, L + 1);
        } else {
          const int64_t leaf_src = lf >= 0 ? lf : o;
          recs[p] = uint2_like{0u, 0u};
          fill(2 * p + 1, -1, leaf_src, L + 1);
          fill(2 * p + 2, -1, leaf_src, L + 1);
        }
      };
      fill(0, 0, -1, 0);
    }
  } else {
    f.leaf_heap.assign(node_prefix.back(), -1);
    f.block_rec_base.assign(size_t(nb), 0);
    for (int b = 0; b < nb; ++b) {
      const int t0 = blocks[size_t(b)].first, n = blocks[size_t(b)].second;
      uint8_t* blk = f.blob.data() + f.block_off[size_t(b)];
      uint32_t* head = reinterpret_cast<uint32_t*>(blk);
      head[0] = uint32_t(n);
      head[1] = uint32_t(t0);
      const size_t rec_off = round_up(16 + 4 * size_t(n), 16);
      auto* recs = reinterpret_cast<uint2_like*>(blk + rec_off);
      const size_t base = node_prefix[size_t(t0)];
      f.block_rec_base[size_t(b)] = uint32_t(base);
      for (int i = 0; i < n; ++i) {
        const int t = t0 + i;
        const uint32_t start = uint32_t(node_prefix[size_t(t)] - base);
        head[4 + i] = start;
        uint2_like* r = recs + start;
        int32_t* heap = f.leaf_heap.data() + node_prefix[size_t(t)];
        if (t >= f.T) {
          r[0] = uint2_like{kRecLeaf, nz_bits};
          continue;
        }
        const Tree& tr = m.trees[size_t(t)];
        // breadth-first, children of a node stored adjacently
        std::vector<int64_t> order{0};
        uint32_t next = 1;
        for (size_t q = 0; q < order.size(); ++q) {
          const int64_t o = order[q];
          if (tr.feature[size_t(o)] < 0) {
            uint32_t bits;
            std::memcpy(&bits, &tr.leaf[size_t(o)], 4);
            r[q] = uint2_like{kRecLeaf, bits};
            heap[q] = int32_t(o);
            continue;
          }
          const uint32_t slot = uint32_t(slot_of[size_t(tr.feature[size_t(o)])]);
          uint2_like rec = encode_split(tr, o, slot << 4, data_bins, f.full_masks);
          rec.x |= next << 16;
          r[q] = rec;
          order.push_back(2 * o + 1);
          order.push_back(2 * o + 2);
          next += 2;
        }
        f.nodes += int64_t(order.size());
      }
    }
  }
  if (f.full_masks.empty()) f.full_masks.assign(8, 0u);
  if (f.leaf_heap.empty()) f.leaf_heap.assign(1, -1);
  return true;
}

std::string describe_forest(const FlatForest& f) {
  std::string s = "{";
  s += "\"layout\":\"" + std::string(f.layout == Layout::kComplete ? "complete" : "explicit") + "\"";
  s += ",\"trees\":" + std::to_string(f.T);
  s += ",\"padded_trees\":" + std::to_string(f.Tpad);
  s += ",\"group\":" + std::to_string(f.G);
  s += ",\"classes\":" + std::to_string(f.K);
  s += ",\"slots\":" + std::to_string(f.S);
  s += ",\"depth\":" + std::to_string(f.layout == Layout::kComplete ? f.D : f.max_depth);
  s += ",\"rows_per_tile\":" + std::to_string(f.plan.R);
  s += ",\"tile_buffers\":" + std::to_string(f.plan.tile_bufs);
  s += ",\"blocks\":" + std::to_string(f.plan.nblocks);
  s += ",\"block_buffer_bytes\":" + std::to_string(f.plan.buf_bytes);
  s += ",\"smem_bytes\":" + std::to_string(f.plan.smem);
  s += ",\"forest_bytes\":" + std::to_string(f.blob.size());
  s += ",\"full_masks\":" + std::to_string(f.full_masks.size() / 8);
  s += ",\"plan\":\"" + f.plan.note + "\"";
  s += "}";
  return s;
}

}  // namespace mb
