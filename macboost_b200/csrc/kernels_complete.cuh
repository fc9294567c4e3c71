// sm_100a forest kernel for the complete (padded-heap) layout.
//
// Semantics (per row, bit-exact with the reference CPU predictor,
// Sources/MacBoost/Booster.swift:2035-2117 and python/macboost/_pyinfer.py:52-89):
//   acc[c] = baseScores[c];  for t in tree order: acc[t % K] += leaf of t
// where the walk goes left iff
//   categorical node : bit `code` of the node mask, code = rint(v) if v finite
//                      and 0 <= rint(v) < dataBins, else dataBins
//   NaN              : the node's default direction (flags bit0)
//   otherwise        : v <= threshold (fp32 compare, no flush-to-zero)
//
// Execution model.  One persistent CTA per SM, one thread per row of a row
// tile of R rows.  The tile's feature columns come from HBM by cp.async.bulk
// completing on mbarriers.  With the forest resident in shared memory each
// warp stages and scores its own 32-row chunks (one 128-byte copy per staged
// feature, the warp's own mbarrier), so a warp waiting for its rows leaves the
// SM to the others; a forest larger than shared memory streams one block of
// trees at a time through two buffers, with CTA-wide tiles of R rows (one copy
// of R values per staged feature, one or two tile buffers).  Each
// thread walks G trees at once (G independent chains of shared-memory loads)
// and adds their leaves to fp32 accumulators strictly in tree order.
//
// The walk keeps the node as a 32-bit shared address o; with heap node n in
// 8-byte slot n + 1 of a tree whose slots start at A, the child is
// o' = 2*o - A + 8*go_right, and after D levels the leaf value sits at
// (o >> 1) + k.  The x gather reads slot row (record.x) at this thread's
// column: rows of a tile are 4*R bytes apart with R a multiple of 32, so a
// warp's 32 gathers hit 32 distinct banks whatever features the lanes read,
// and each heap level of a tree starts on a 128-byte line, so a warp's record
// loads for one level cost one wavefront (two for the 32-node level of a
// depth-6 tree).  The kernel is bound by those shared-memory wavefronts and
// by instruction issue, not by HBM: see the bench's roofline report.
//
// Tensor cores are not used: tree traversal is a data-dependent walk, not a
// dense contraction.  Every mbarrier wait is bounded (globaltimer); on expiry
// the CTA records kErrWaitTimeout in *err and all its threads return together.
#pragma once

#include <type_traits>

#include "kernels_common.cuh"

namespace mb {
namespace complete {


struct NoTop {};

// The walk of every tree block of every row tile.  With TopRecords (`top`),
// levels 0 and 1 come from the kernel parameter: the root record is warp
// uniform, and both level-1 records are loaded (uniform) and selected, so a
// tree's first two levels cost no shared-memory wavefront; the walk then
// resumes at heap node 3 + 2 r0 + r1 (slot 4 + 2 r0 + r1).  PAY (no planes,
// no categorical splits): numeric records carry their default direction as
// the fmax operand itself (dev::route).
template <int KT, int G, bool PLANES, bool CAT, int DC, bool PAY, class Top>
__device__ __forceinline__ void complete_tiles(const KArgs& a, unsigned char* smem, const Top& top) {
  constexpr bool kTop = !std::is_same<Top, NoTop>::value;
  const int D = DC > 0 ? DC : a.D;  // DC: depth fixed at compile time, 0 = from a.D
  const uint32_t NL = 1u << D;          // slots (and leaves) per tree
  auto score = [&](uint32_t fb, int b, long long row, uint32_t rowbase, dev::Acc<KT>& acc,
                   bool clean) {
    const int t_block = b * a.Tb;
    const uint32_t leaves = fb + a.leaf_off;
    auto walk = [&](auto nonan_tag) {
    constexpr bool NN = decltype(nonan_tag)::value;
    for (int g0 = 0; g0 < a.Tb; g0 += G) {
      uint32_t A[G], o[G];
#pragma unroll
      for (int j = 0; j < G; ++j) {
        A[j] = fb + uint32_t(g0 + j) * NL * 8u;
        o[j] = A[j] + 8u;  // root: heap node 0 in slot 1
      }
      if constexpr (kTop) {
        const int t0 = 3 * (t_block + g0);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const unsigned long long q0 = top.rec[t0 + 3 * j];
          const uint32_t r0 = dev::route<PLANES, CAT, NN, PAY>(make_uint2(unsigned(q0), unsigned(q0 >> 32)),
                                                       rowbase, a.masks, a.data_bins);
          const unsigned long long q1 = top.rec[t0 + 3 * j + 1];
          const unsigned long long q2 = top.rec[t0 + 3 * j + 2];
          const unsigned long long q = r0 ? q2 : q1;
          const uint32_t r1 = dev::route<PLANES, CAT, NN, PAY>(make_uint2(unsigned(q), unsigned(q >> 32)),
                                                       rowbase, a.masks, a.data_bins);
          o[j] = A[j] + 8u * (4u + 2u * r0 + r1);
        }
      }
      for (int L = kTop ? 2 : 0; L < D; ++L) {
        uint2 r[G];
#pragma unroll
        for (int j = 0; j < G; ++j) r[j] = dev::lds_v2(o[j]);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const uint32_t right = dev::route<PLANES, CAT, NN, PAY>(r[j], rowbase, a.masks, a.data_bins);
          o[j] = 2u * o[j] - A[j] + (right << 3);
        }
      }
#pragma unroll
      for (int j = 0; j < G; ++j) {
        // heap node n = (o - A)/8 - 1 is leaf n - (NL - 1) of the tree
        const uint32_t k = leaves + uint32_t(g0 + j) * NL * 4u - (A[j] >> 1) - 4u * NL;
        acc.add(j, t_block + g0 + j, dev::lds_f32((o[j] >> 1) + k));
      }
      if (a.out_leaf != nullptr && row < a.rows) {
        const int t0 = t_block + g0;
        int li[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const uint32_t leaf = (o[j] - A[j]) / 8u - NL;
          li[j] = t0 + j < a.T ? __ldg(a.leaf_heap + size_t(t0 + j) * NL + leaf) : 0;
        }
        dev::store_leaf_run<G>(a.out_leaf + row * a.T + t0, li, a.T - t0);
      }
    }
    };
    if (!PLANES && clean)
      walk(std::true_type{});
    else
      walk(std::false_type{});
  };
  dev::run_rows<KT, !PLANES>(a, smem, score);
}

template <int KT, int G, bool PLANES, bool CAT, int DC = 0, bool PAY = false>
__global__ void __launch_bounds__(dev::Bounds<KT, G>::kMaxThreads, 1)
    forest_complete_kernel(const KArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  complete_tiles<KT, G, PLANES, CAT, DC, PAY>(a, smem, NoTop{});
}

template <int KT, int G, bool PLANES, bool CAT, int DC = 0, bool PAY = false>
__global__ void __launch_bounds__(dev::Bounds<KT, G>::kMaxThreads, 1)
    forest_complete_top_kernel(const KArgs a, const TopRecords top) {
  extern __shared__ __align__(128) unsigned char smem[];
  complete_tiles<KT, G, PLANES, CAT, DC, PAY>(a, smem, top);
}

using KernelFn = void (*)(const KArgs);
using TopKernelFn = void (*)(const KArgs, const TopRecords);

// Fixed-depth builds (kernels_complete_fixed.cu): the kernel for (planes,
// cat, pay, K, G, D), or null where only the run-time-depth build exists.
KernelFn pick_fixed(bool planes, bool cat, bool pay, int K, int G, int D);
TopKernelFn pick_top_fixed(bool planes, bool cat, bool pay, int K, int G, int D);

}  // namespace complete
}  // namespace mb
