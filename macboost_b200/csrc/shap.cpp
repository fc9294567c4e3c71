// TreeSHAP path tables (see shap.h).
#include "shap.h"

#include <cmath>
#include <limits>

namespace mb {

namespace {

// One split on the way from the root to a leaf.
struct Step {
  int64_t node;
  bool left;  // the path continues to the left child
};

struct Unique {
  int32_t feature;
  double z = 1.0;
  float lo = std::numeric_limits<float>::quiet_NaN();
  float hi = std::numeric_limits<float>::infinity();
  bool nan_ok = true;
  bool has_cat = false;
  uint32_t allowed[8] = {~0u, ~0u, ~0u, ~0u, ~0u, ~0u, ~0u, ~0u};
};

uint64_t binomial(int n, int k) {
  uint64_t r = 1;
  for (int i = 1; i <= k; ++i) r = r * uint64_t(n - k + i) / uint64_t(i);
  return r;
}

}  // namespace

bool build_shap(const Model& m, ShapForest& s, std::string& err) {
  const int K = m.K;
  const int64_t F = m.num_features;
  s = ShapForest();
  s.feature_slot.assign(size_t(F), -1);
  std::vector<std::vector<ShapPathRec>> per_class(static_cast<size_t>(K));
  std::vector<std::vector<ShapUniqueRec>> uniq_class(static_cast<size_t>(K));

  // shapBias (SHAP.swift:56-72): baseScores plus each covered tree's
  // cover-weighted mean leaf, visiting nodes in the reference's stack order.
  std::vector<double> bias(static_cast<size_t>(K));
  for (int k = 0; k < K; ++k) bias[size_t(k)] = double(m.base_scores[size_t(k)]);

  for (size_t t = 0; t < m.trees.size(); ++t) {
    const Tree& tr = m.trees[t];
    const int64_t n_nodes = int64_t(tr.feature.size());
    if (tr.cover.empty()) continue;
    if (int64_t(tr.cover.size()) != n_nodes) {
      err = "tree " + std::to_string(t) + " has " + std::to_string(tr.cover.size()) +
            " cover values for " + std::to_string(n_nodes) + " nodes";
      return false;
    }
    const double total = double(tr.cover[0]);
    if (!(total > 0)) continue;  // SHAP.swift:63 and :190
    const int k = int(t % size_t(K));
    const bool masked = !tr.cat_mask.empty();
    {
      double mean = 0.0;
      std::vector<int64_t> stack{0};
      while (!stack.empty()) {
        const int64_t n = stack.back();
        stack.pop_back();
        if (tr.feature[size_t(n)] >= 0) {
          stack.push_back(2 * n + 1);
          stack.push_back(2 * n + 2);
        } else {
          mean += double(tr.leaf[size_t(n)]) * double(tr.cover[size_t(n)]) / total;
        }
      }
      bias[size_t(k)] += mean;
    }
    // leaves left to right; `steps` is the current root-to-node path
    std::vector<Step> steps;
    std::vector<std::pair<int64_t, int>> todo{{0, 0}};  // (node, depth)
    while (!todo.empty()) {
      const auto [n, depth] = todo.back();
      todo.pop_back();
      steps.resize(size_t(depth));
      if (depth > 0) {
        const int64_t parent = (n - 1) / 2;
        steps[size_t(depth) - 1] = Step{parent, n == 2 * parent + 1};
      }
      if (tr.feature[size_t(n)] >= 0) {
        todo.push_back({2 * n + 2, depth + 1});
        todo.push_back({2 * n + 1, depth + 1});
        continue;
      }
      if (depth == 0) continue;  // root is a leaf: the bias only
      std::vector<Unique> us;
      for (const Step& st : steps) {
        const int64_t p = st.node;
        const int64_t child = st.left ? 2 * p + 1 : 2 * p + 2;
        const int32_t f = tr.feature[size_t(p)];
        const double cn = double(tr.cover[size_t(p)]);
        const double frac = cn > 0 ? double(tr.cover[size_t(child)]) / cn : 0.0;
        Unique* u = nullptr;
        for (Unique& x : us)
          if (x.feature == f) u = &x;
        if (!u) {
          us.push_back(Unique());
          u = &us.back();
          u->feature = f;
        }
        u->z *= frac;
        const uint32_t fl = tr.flags[size_t(p)];
        if ((fl & kFlagCategorical) && masked) {
          u->has_cat = true;
          const uint32_t* mw = &tr.cat_mask[size_t(p) * 8];
          for (int w = 0; w < 8; ++w) u->allowed[w] &= st.left ? mw[w] : ~mw[w];
        } else {
          const float th = tr.threshold[size_t(p)];
          // left: v <= th for every such split (a NaN threshold admits no
          // value: hi becomes NaN and stays so); right: !(v <= th), i.e.
          // v > the largest such threshold (a NaN threshold admits all)
          if (st.left) {
            if (!std::isnan(u->hi)) u->hi = std::isnan(th) ? th : std::min(u->hi, th);
          } else if (!std::isnan(th)) {
            u->lo = std::isnan(u->lo) ? th : std::max(u->lo, th);
          }
          u->nan_ok = u->nan_ok && (((fl & kFlagDefaultLeft) != 0) == st.left);
        }
      }
      if (int(us.size()) > kShapMaxUnique) {
        err = "tree " + std::to_string(t) + " has a path through " + std::to_string(us.size()) +
              " distinct features; the contributions kernel handles " +
              std::to_string(kShapMaxUnique);
        return false;
      }
      ShapPathRec pr{};
      pr.first = uint32_t(uniq_class[size_t(k)].size());
      pr.U = uint32_t(us.size());
      pr.leaf = double(tr.leaf[size_t(n)]);
      per_class[size_t(k)].push_back(pr);
      s.max_unique = std::max(s.max_unique, int(us.size()));
      for (const Unique& u : us) {
        if (s.feature_slot[size_t(u.feature)] < 0) {
          s.feature_slot[size_t(u.feature)] = int32_t(s.slot_feature.size());
          s.slot_feature.push_back(u.feature);
        }
        ShapUniqueRec r{};
        r.z = u.z;
        r.lo = u.lo;
        r.hi = u.hi;
        r.slot = uint32_t(s.feature_slot[size_t(u.feature)]);
        r.flags = (u.nan_ok ? kShapNanOk : 0u) | (u.has_cat ? kShapHasCat : 0u);
        if (u.has_cat) {
          r.mask = uint32_t(s.masks.size() / 8);
          s.masks.insert(s.masks.end(), u.allowed, u.allowed + 8);
        }
        uniq_class[size_t(k)].push_back(r);
      }
    }
  }
  // class-major concatenation
  s.class_begin.push_back(0);
  for (int k = 0; k < K; ++k) {
    const uint32_t base = uint32_t(s.uniq.size());
    for (ShapPathRec p : per_class[size_t(k)]) {
      p.first += base;
      s.paths.push_back(p);
    }
    s.uniq.insert(s.uniq.end(), uniq_class[size_t(k)].begin(), uniq_class[size_t(k)].end());
    s.class_begin.push_back(uint32_t(s.paths.size()));
  }
  s.bias.resize(size_t(K));
  for (int k = 0; k < K; ++k) s.bias[size_t(k)] = float(bias[size_t(k)]);
  // staged blocks: consecutive paths of one class, bounded in paths and records
  s.class_block.push_back(0);
  for (int k = 0; k < K; ++k) {
    uint32_t p = s.class_begin[size_t(k)];
    const uint32_t end = s.class_begin[size_t(k) + 1];
    while (p < end) {
      const uint32_t u0 = s.paths[p].first;
      uint32_t q = p;
      while (q < end && q - p < uint32_t(kShapBlockPaths) &&
             s.paths[q].first + s.paths[q].U - u0 <= uint32_t(kShapBlockUniq))
        ++q;
      s.block_path.push_back(p);
      s.block_uniq.push_back(u0);
      p = q;
    }
    s.class_block.push_back(uint32_t(s.block_path.size()));
  }
  s.block_path.push_back(uint32_t(s.paths.size()));
  s.block_uniq.push_back(uint32_t(s.uniq.size()));
  // Shapley weights s! (U-1-s)! / U! = 1 / (U * C(U-1, s)), zero-padded
  s.coef.assign(size_t(kShapMaxUnique + 1) * kShapCoefRow, 0.0);
  for (int U = 1; U <= kShapMaxUnique; ++U)
    for (int j = 0; j < U; ++j)
      s.coef[size_t(U) * kShapCoefRow + kShapMaxUnique + j] =
          1.0 / (double(U) * double(binomial(U - 1, j)));
  return true;
}

}  // namespace mb
