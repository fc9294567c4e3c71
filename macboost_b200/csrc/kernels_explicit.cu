// sm_100a forest kernel for the explicit (breadth-first, leaf-record) layout
// used for deep, sparse trees such as leaf-wise models.  Same semantics,
// staging pipeline and bounded waits as the complete-layout kernel
// (kernels_complete.cu); only the walk differs: each record names the
// distance to its first child, children are adjacent, and leaf records loop on
// themselves, so the G trees of a group all take the group's step count (its
// deepest leaf) without per-step branches and end on their leaves.
#include <type_traits>

#include "kernels_common.cuh"

namespace mb {
namespace {

// COMPACT: record bits 18-31 hold 8 x the child distance (a byte offset).
template <int KT, int G, bool CAT, bool COMPACT>
__global__ void __launch_bounds__(dev::Bounds<KT, G>::kMaxThreads, 1)
    forest_explicit_kernel(const KArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  auto score = [&](uint32_t fb, int b, long long row, uint32_t rowbase, dev::Acc<KT>& acc,
                   bool clean) {
    // block header: [0] trees, [1] first tree index, [4 + i] first record of
    // tree i, [4 + trees + g] steps of group g
    const int ntrees = int(dev::lds_u32(fb));
    const int t_block = int(dev::lds_u32(fb + 4u));
    const uint32_t steps_at = fb + 16u + 4u * uint32_t(ntrees);
    const uint32_t recs =
        fb + ((16u + 4u * uint32_t(ntrees + ntrees / G) + 15u) & ~15u);
    for (int g0 = 0; g0 < ntrees; g0 += G) {
      const int steps = int(dev::lds_u32(steps_at + 4u * uint32_t(g0 / G)));
      uint32_t o[G];
#pragma unroll
      for (int j = 0; j < G; ++j) o[j] = recs + 8u * dev::lds_u32(fb + 16u + 4u * uint32_t(g0 + j));
      auto walk = [&](auto nonan_tag) {
        constexpr bool NN = decltype(nonan_tag)::value;
        for (int it = 0; it < steps; ++it) {
          uint2 r[G];
#pragma unroll
          for (int j = 0; j < G; ++j) r[j] = dev::lds_v2(o[j]);
#pragma unroll
          for (int j = 0; j < G; ++j) {
            // records carry the child distance above the slot offset, so the
            // slot is always masked; leaves read the -Inf slot with the
            // default-left bit (go_right = 0; with NN, !(-Inf <= leaf) = 0)
            // and have distance 0: they stay put
            const uint32_t right =
                dev::route<false, CAT, NN>(r[j], rowbase, a.masks, a.data_bins);
            if (COMPACT)
              o[j] += (r[j].x >> kRecChildShift) + (right ? 8u : 0u);
            else
              o[j] += ((r[j].x >> kRecChildShift) + right) * 8u;
          }
        }
      };
      if (clean)
        walk(std::true_type{});
      else
        walk(std::false_type{});
#pragma unroll
      for (int j = 0; j < G; ++j) acc.add(j, t_block + g0 + j, dev::lds_f32(o[j] + 4u));
      if (a.out_leaf != nullptr && row < a.rows) {
        const size_t rec_base = a.block_rec_base[b];
        const int t0 = t_block + g0;
        int li[G];
#pragma unroll
        for (int j = 0; j < G; ++j)
          li[j] = t0 + j < a.T ? __ldg(a.leaf_heap + rec_base + (o[j] - recs) / 8u) : 0;
        dev::store_leaf_run<G>(a.out_leaf + row * a.T + t0, li, a.T - t0);
      }
    }
  };
  dev::run_rows<KT, true>(a, smem, score);
}

using KernelFn = void (*)(const KArgs);

template <int KT, int G>
KernelFn pick3(bool cat, bool compact) {
  if (compact)
    return cat ? forest_explicit_kernel<KT, G, true, true>
               : forest_explicit_kernel<KT, G, false, true>;
  return cat ? forest_explicit_kernel<KT, G, true, false>
             : forest_explicit_kernel<KT, G, false, false>;
}

// (K, G) pairs must match mb::group_options (forest.cpp).  NaN planes need no
// separate instantiation: explicit records always mask the slot offset and
// clear the default-left bit when planes are in use.
KernelFn pick(bool, bool cat, bool compact, int K, int G) {
  switch (K) {
    case 1: return G == 16 ? pick3<1, 16>(cat, compact) : pick3<1, 8>(cat, compact);
    case 2: return pick3<2, 8>(cat, compact);
    case 3: return pick3<3, 6>(cat, compact);
    case 4: return pick3<4, 8>(cat, compact);
    case 5: return pick3<5, 5>(cat, compact);
    case 6: return pick3<6, 6>(cat, compact);
    case 7: return pick3<7, 7>(cat, compact);
    case 8: return pick3<8, 8>(cat, compact);
    case 10: return pick3<10, 10>(cat, compact);
    case 12: return pick3<12, 12>(cat, compact);
    case 16: return pick3<16, 16>(cat, compact);
    default: return pick3<0, 8>(cat, compact);
  }
}

}  // namespace

cudaError_t launch_explicit(bool planes, bool cat, const KArgs& a, size_t smem, int grid,
                            cudaStream_t stream, int* occupancy_out) {
  KernelFn fn = pick(planes, cat, a.compact_children != 0, a.K, a.G);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  if (occupancy_out)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occupancy_out, fn, a.R, smem);
  fn<<<grid, a.R, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb
