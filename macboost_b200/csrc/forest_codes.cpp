// Binned-code flattening of complete-layout forests.
//
// For every feature a numeric split reads, the forest's distinct thresholds
// on that feature, sorted, t_0 < t_1 < ... < t_{m-1}, define the code of a
// value v as the number of thresholds below it:  code(v) = #{j : t_j < v}.
// Then, for the split on t_J,  v <= t_J  <=>  code(v) <= J, exactly (IEEE
// comparisons of finite thresholds; -0.0 and +0.0 are one threshold).  Each
// row tile is converted once -- one branch-free search per value in an
// Eytzinger-ordered table -- and every node visit afterwards compares two
// small integers:  go_right = code > J.
//
// Missing values get a sentinel per *plane*: the NaN-right plane stores the
// largest code (it exceeds every J: NaN goes right), the NaN-left plane stores
// 0 (0 <= J: NaN goes left); a split reads the plane of its default direction.
// Categorical splits read a third plane holding the value's category code
// (rint(v) in 0..dataBins-1, else dataBins, _pyinfer.py:80-86) and test their
// 256-bit mask.
//
// Code tile: 4-byte words, one per (thread, group of 4/code_bytes slots), so a
// warp's 32 code loads hit 32 distinct banks whatever slots its lanes read.
// Node record (4 bytes):  bits 14..31  byte offset of the code in the tile
// row (slot group * 4R + slot within the word * code_bytes);  bit 13  categorical;
// bits 0..12  J (numeric) or the categorical node's mask index.  Trees are
// complete heaps padded to depth D (as in the f32 layout) with heap node n in
// 4-byte slot n + 1, so every level starts on a 128-byte line and one warp's
// record loads for a level take one wavefront.  Leaves follow at leaf_off.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <limits>

#include "forest.h"

namespace mb {
namespace {

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr uint32_t kCodeCatBit = 0x2000u;
constexpr uint32_t kCodeIndexMask = 0x1FFFu;
constexpr int kCodeOffsetShift = 14;

struct FeatureUse {
  bool used = false, right = false, left = false, cat = false;
  std::vector<float> thr;  // numeric thresholds (with repeats until sorted)
};

// must match CodesBounds (kernels_codes.cu); K outside the dedicated
// instantiations runs the generic kernel (KT = 0)
int max_threads_codes(int K, int G) {
  const bool dedicated = K >= 1 && K <= 8;
  return G >= 12 ? 256 : (G >= 10 || !dedicated || K >= 5 ? 512 : 768);
}

}  // namespace

bool flatten_codes(const Model& m, FlatForest& f, std::string& why, int force_G, int force_R) {
  const int D = std::max(1, m.max_depth);
  if (D > kMaxCompleteDepth) {
    why = "forest deeper than the complete layout";
    return false;
  }
  const int NL = 1 << D, NI = NL - 1;
  const size_t F = size_t(m.num_features);
  std::vector<FeatureUse> use(F);
  size_t n_cat_nodes = 0;
  for (const Tree& t : m.trees) {
    std::vector<int64_t> st{0};
    while (!st.empty()) {
      const int64_t o = st.back();
      st.pop_back();
      const int32_t fe = t.feature[size_t(o)];
      if (fe < 0) continue;
      FeatureUse& u = use[size_t(fe)];
      u.used = true;
      const uint32_t fl = t.flags[size_t(o)];
      if ((fl & kFlagCategorical) && !t.cat_mask.empty()) {
        u.cat = true;
        ++n_cat_nodes;
      } else {
        ((fl & kFlagDefaultLeft) ? u.left : u.right) = true;
        u.thr.push_back(t.threshold[size_t(o)]);
      }
      st.push_back(2 * o + 1);
      st.push_back(2 * o + 2);
    }
  }
  size_t m_max = 0;
  for (FeatureUse& u : use) {
    std::sort(u.thr.begin(), u.thr.end());
    u.thr.erase(std::unique(u.thr.begin(), u.thr.end(),
                            [](float a, float b) { return a == b; }),
                u.thr.end());
    m_max = std::max(m_max, u.thr.size());
  }
  int cw;
  if (m_max <= 254) {
    cw = 1;
  } else if (m_max <= 8190) {
    cw = 2;
  } else {
    why = "a feature has more than 8190 distinct thresholds";
    return false;
  }
  if (n_cat_nodes > kCodeIndexMask + 1) {
    why = "more than 8192 categorical splits";
    return false;
  }
  int d = 1;
  while ((size_t(1) << d) - 1 < m_max) ++d;

  // staged features, search tables, code slots
  FlatForest g;
  g.codes = true;
  g.layout = Layout::kComplete;
  g.T = int(m.trees.size());
  g.K = m.K;
  g.max_depth = m.max_depth;
  g.D = D;
  g.code_bytes = cw;
  g.search_depth = d;
  std::vector<int32_t> slotR(F, -1), slotL(F, -1), slotC(F, -1), table(F, -1);
  int n_tables = 0, n_slots = 0;
  for (size_t fe = 0; fe < F; ++fe) {
    const FeatureUse& u = use[fe];
    if (!u.used) continue;
    g.stage_feature.push_back(int32_t(fe));
    if (!u.thr.empty()) table[fe] = n_tables++;
    if (u.right) slotR[fe] = n_slots++;
    if (u.left) slotL[fe] = n_slots++;
    if (u.cat) slotC[fe] = n_slots++;
    g.bin_plan.insert(g.bin_plan.end(), {table[fe], slotR[fe], slotL[fe], slotC[fe]});
  }
  g.S_stage = int(g.stage_feature.size());
  g.S_total = g.S_stage;
  g.S_code = n_slots;
  const int per_word = 4 / cw;
  const int code_words = std::max(1, (n_slots + per_word - 1) / per_word);
  // Eytzinger tables: in-order fill of a complete binary tree of 2^d - 1 keys
  // (+Inf padding), 1-based; searching i = 2i + (t[i] < v) for d steps ends at
  // i = 2^d + code(v).
  const size_t tsize = size_t(1) << d;
  // (at least one table: the kernel searches table 0 for categorical-only
  // features and discards the result)
  g.search.assign(std::max<size_t>(size_t(n_tables), 1) * tsize,
                  std::numeric_limits<float>::infinity());
  for (size_t fe = 0; fe < F; ++fe) {
    if (table[fe] < 0) continue;
    const std::vector<float>& a = use[fe].thr;
    float* T = g.search.data() + size_t(table[fe]) * tsize;
    size_t idx = 0;
    std::function<void(size_t)> fill = [&](size_t k) {
      if (k >= tsize) return;
      fill(2 * k);
      T[k] = idx < a.size() ? a[idx] : std::numeric_limits<float>::infinity();
      ++idx;
      fill(2 * k + 1);
    };
    fill(1);
    T[0] = 0.0f;
  }

  // --- plan: (G, R, resident / streamed) ---------------------------------
  struct Best {
    LaunchPlan p;
    int G = 0;
    double cost = 1e300;
  } best;
  const int Rs[] = {768, 640, 512, 384, 256, 128};
  auto block_bytes = [&](int n) -> size_t {
    return round_up(round_up(size_t(n) * NL * 4, 128) + size_t(n) * NL * 4, 128);
  };
  for (int G : group_options(m.K)) {
    if (force_G && G != force_G) continue;
    const int ngroups = (g.T + G - 1) / G;
    for (int R : Rs) {
      if (R > max_threads_codes(m.K, G) || (force_R && R != force_R)) continue;
      const size_t raw = round_up(size_t(std::max(g.S_stage, 1)) * R * 4, 128);
      const size_t codes = round_up(size_t(code_words) * R * 4, 128);
      // record offsets must fit 18 bits
      if (size_t(code_words) * R * 4 >= (size_t(1) << 18)) continue;
      const size_t used = kSmemHeader + raw + codes;
      if (used > kSmemBudget) continue;
      const size_t avail = kSmemBudget - used;
      LaunchPlan p;
      p.R = R;
      p.tile_bufs = 1;
      p.planes = true;
      p.tile_bytes = uint32_t(raw);
      if (ngroups == 0) {
        p.smem = used;
        p.note = "no trees";
      } else if (block_bytes(ngroups * G) <= avail) {
        p.Tb = ngroups * G;
        p.nblocks = 1;
        p.buf_bytes = uint32_t(round_up(block_bytes(p.Tb), 128));
        p.smem = used + p.buf_bytes;
        p.note = "binned codes, forest resident in shared memory";
      } else {
        const size_t max_block = (avail / 2) / 128 * 128;
        int Tb = 0;
        for (int t = G; t <= ngroups * G && block_bytes(t) <= max_block; t += G) Tb = t;
        if (Tb == 0) continue;
        // the block count (>= the minimum) that pads the fewest trees
        const int nb_min = (ngroups * G + Tb - 1) / Tb;
        int nb = nb_min, best_pad = 1 << 30;
        for (int c = nb_min; c <= nb_min + nb_min / 2 + 1; ++c) {
          const int tb = int(round_up(size_t((ngroups + c - 1) / c), 1)) * G;
          if (block_bytes(tb) > max_block) continue;
          const int pad = c * tb - g.T;
          if (pad < best_pad) {
            best_pad = pad;
            nb = c;
          }
        }
        Tb = ((ngroups + nb - 1) / nb) * G;
        p.Tb = Tb;
        p.nblocks = nb;
        p.buf_bytes = uint32_t(round_up(block_bytes(Tb), 128));
        p.smem = used + 2 * size_t(p.buf_bytes);
        p.note = "binned codes, forest streamed in tree blocks";
      }
      // Cost model (SM clocks per row), calibrated on B200: the walk costs ~21
      // clk per warp and depth-6 tree (one wavefront per 4-byte record and per
      // code gather, but more integer issue than the fp32 walk); each search
      // step of the per-value conversion costs ~0.1 clk per row while the
      // search tables stay in L1 (<= 32 KB), ~0.4 otherwise.
      const int Tpad = p.nblocks * p.Tb;
      const double warps = double(R) / 32.0;
      const double eff =
          std::min(1.0, std::pow(warps / 16.0, 0.45) * std::pow(double(G) / 8.0, 0.15));
      const double walk = double(Tpad) * 21.0 * double(D) / 6.0 / 32.0 / eff;
      const double table_bytes = double(n_tables) * double(tsize) * 4.0;
      const double bin = double(n_tables) * d * (table_bytes <= 32768.0 ? 0.1 : 0.4) +
                         double(g.S_stage) * 0.1;
      const double load = double(g.S_stage) * 4.0 / 23.0;
      const double stream =
          p.nblocks > 1
              ? (double(p.nblocks) * 1500.0 + double(p.buf_bytes) * p.nblocks / 64.0) / double(R)
              : 0.0;
      const double cost = std::max(walk + bin, load) + 2500.0 / double(R) + stream;
      p.est_clk_per_row = cost;
      if (cost < best.cost * 0.999) {
        best.p = p;
        best.G = G;
        best.cost = cost;
      }
    }
  }
  if (best.p.R == 0) {
    why = "no binned-code plan fits shared memory";
    return false;
  }
  g.plan = best.p;
  g.G = best.G;
  const int R = g.plan.R, Tb = g.plan.Tb, nb = g.plan.nblocks;
  g.Tpad = nb * Tb;
  const uint32_t word_stride = uint32_t(R) * 4u;  // bytes between slot groups
  auto code_off = [&](int slot) -> uint32_t {
    return uint32_t(slot / per_word) * word_stride + uint32_t(slot % per_word) * uint32_t(cw);
  };

  // --- emit --------------------------------------------------------------
  const uint32_t bb = Tb ? uint32_t(block_bytes(Tb)) : 0u;
  g.leaf_off = Tb ? uint32_t(round_up(size_t(Tb) * NL * 4, 128)) : 0u;
  g.block_off.assign(size_t(nb) + 1, 0);
  for (int b = 0; b < nb; ++b) g.block_off[size_t(b) + 1] = g.block_off[size_t(b)] + bb;
  g.blob.assign(size_t(nb) * bb, 0);
  g.leaf_heap.assign(std::max<size_t>(size_t(g.Tpad) * NL, 1), -1);
  const float neg_zero = -0.0f;
  for (int t = 0; t < g.Tpad; ++t) {
    uint8_t* blk = g.blob.data() + size_t(t / Tb) * bb;
    auto* recs = reinterpret_cast<uint32_t*>(blk) + size_t(t % Tb) * NL;
    auto* leaves = reinterpret_cast<float*>(blk + g.leaf_off) + size_t(t % Tb) * NL;
    int32_t* heap = g.leaf_heap.data() + size_t(t) * NL;
    if (t >= g.T) {
      for (int n = 0; n < NL; ++n) recs[n] = 0u;
      for (int n = 0; n < NL; ++n) leaves[n] = neg_zero;
      continue;
    }
    const Tree& tr = m.trees[size_t(t)];
    std::function<void(int64_t, int64_t, int64_t, int)> fill = [&](int64_t p, int64_t o,
                                                                   int64_t lf, int L) {
      if (L == D) {
        const int64_t src = lf >= 0 ? lf : o;
        leaves[p - NI] = tr.leaf[size_t(src)];
        heap[p - NI] = int32_t(src);
        return;
      }
      if (lf < 0 && tr.feature[size_t(o)] >= 0) {
        const size_t fe = size_t(tr.feature[size_t(o)]);
        const uint32_t fl = tr.flags[size_t(o)];
        uint32_t rec;
        if ((fl & kFlagCategorical) && !tr.cat_mask.empty()) {
          const uint32_t idx = uint32_t(g.cat_masks.size() / 8);
          g.cat_masks.insert(g.cat_masks.end(), &tr.cat_mask[size_t(o) * 8],
                             &tr.cat_mask[size_t(o) * 8] + 8);
          rec = (code_off(slotC[fe]) << kCodeOffsetShift) | kCodeCatBit | idx;
        } else {
          const std::vector<float>& a = use[fe].thr;
          const float thr = tr.threshold[size_t(o)];
          const uint32_t J = uint32_t(std::lower_bound(a.begin(), a.end(), thr) - a.begin());
          const int slot = (fl & kFlagDefaultLeft) ? slotL[fe] : slotR[fe];
          rec = (code_off(slot) << kCodeOffsetShift) | J;
        }
        recs[p + 1] = rec;
        fill(2 * p + 1, 2 * o + 1, -1, L + 1);
        fill(2 * p + 2, 2 * o + 2, -1, L + 1);
      } else {
        const int64_t leaf_src = lf >= 0 ? lf : o;
        recs[p + 1] = 0u;  // padding split: both subtrees end in the same leaf
        fill(2 * p + 1, -1, leaf_src, L + 1);
        fill(2 * p + 2, -1, leaf_src, L + 1);
      }
    };
    fill(0, 0, -1, 0);
    g.nodes += int64_t(NL) * 2 - 1;
  }
  // bin_plan slots -> byte offsets within a thread's code words
  for (size_t i = 0; i < g.bin_plan.size(); i += 4)
    for (size_t k = 1; k < 4; ++k)
      if (g.bin_plan[i + k] >= 0) g.bin_plan[i + k] = int32_t(code_off(g.bin_plan[i + k]));
  if (g.cat_masks.empty()) g.cat_masks.assign(8, 0u);
  g.full_masks.assign(8, 0u);
  g.plan.tile_bytes = uint32_t(round_up(size_t(std::max(g.S_stage, 1)) * R * 4, 128));
  g.code_tile_bytes = uint32_t(round_up(size_t(code_words) * R * 4, 128));
  f = std::move(g);
  return true;
}

}  // namespace mb
