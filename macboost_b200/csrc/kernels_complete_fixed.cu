// Fixed-depth builds of the complete-layout forest kernel: single-class
// forests (regression, binary objectives) of depth 4 to 8 in groups of 8
// trees, the common gradient-boosting shapes, and 10-class forests of depth
// 6 in groups of 10 (one tree per class: a 10-class softmax model).  With the
// depth known at compile time the level loop unrolls and the per-tree slot
// arithmetic folds; on B200 the depth-6 build runs cfg2-like forests 4-8%
// faster than the run-time-depth build.  Same semantics and layout
// (kernels_complete.cuh).
#include "kernels_complete.cuh"

namespace mb {
namespace complete {
namespace {

template <int KT, int G, int D>
KernelFn fixed(bool planes, bool cat, bool pay) {
  if (planes)
    return cat ? forest_complete_kernel<KT, G, true, true, D>
               : forest_complete_kernel<KT, G, true, false, D>;
  if (cat) return forest_complete_kernel<KT, G, false, true, D>;
  return pay ? forest_complete_kernel<KT, G, false, false, D, true>
             : forest_complete_kernel<KT, G, false, false, D>;
}

template <int KT, int G, int D>
TopKernelFn fixed_top(bool planes, bool cat, bool pay) {
  if (planes)
    return cat ? forest_complete_top_kernel<KT, G, true, true, D>
               : forest_complete_top_kernel<KT, G, true, false, D>;
  if (cat) return forest_complete_top_kernel<KT, G, false, true, D>;
  return pay ? forest_complete_top_kernel<KT, G, false, false, D, true>
             : forest_complete_top_kernel<KT, G, false, false, D>;
}

}  // namespace

KernelFn pick_fixed(bool planes, bool cat, bool pay, int K, int G, int D) {
  if (K == 10 && G == 10 && D == 6) return fixed<10, 10, 6>(planes, cat, pay);
  if (K != 1 || G != 8) return nullptr;
  switch (D) {
    case 4: return fixed<1, 8, 4>(planes, cat, pay);
    case 5: return fixed<1, 8, 5>(planes, cat, pay);
    case 6: return fixed<1, 8, 6>(planes, cat, pay);
    case 7: return fixed<1, 8, 7>(planes, cat, pay);
    case 8: return fixed<1, 8, 8>(planes, cat, pay);
    default: return nullptr;
  }
}

TopKernelFn pick_top_fixed(bool planes, bool cat, bool pay, int K, int G, int D) {
  if (K == 10 && G == 10 && D == 6) return fixed_top<10, 10, 6>(planes, cat, pay);
  if (K != 1 || G != 8) return nullptr;
  switch (D) {
    case 4: return fixed_top<1, 8, 4>(planes, cat, pay);
    case 5: return fixed_top<1, 8, 5>(planes, cat, pay);
    case 6: return fixed_top<1, 8, 6>(planes, cat, pay);
    case 7: return fixed_top<1, 8, 7>(planes, cat, pay);
    case 8: return fixed_top<1, 8, 8>(planes, cat, pay);
    default: return nullptr;
  }
}

}  // namespace complete
}  // namespace mb
