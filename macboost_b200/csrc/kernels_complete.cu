// Run-time-depth builds of the complete-layout forest kernel and its
// launchers (the kernel itself: kernels_complete.cuh).
#include "kernels_complete.cuh"

namespace mb {
namespace complete {
namespace {

template <int KT, int G>
KernelFn pick3(bool planes, bool cat, bool pay) {
  if (planes)
    return cat ? forest_complete_kernel<KT, G, true, true>
               : forest_complete_kernel<KT, G, true, false>;
  if (cat) return forest_complete_kernel<KT, G, false, true>;
  return pay ? forest_complete_kernel<KT, G, false, false, 0, true>
             : forest_complete_kernel<KT, G, false, false>;
}

// (K, G) pairs must match mb::group_options (forest.cpp); a fixed-depth
// build where one exists.
KernelFn pick(bool planes, bool cat, bool pay, int K, int G, int D) {
  if (KernelFn f = pick_fixed(planes, cat, pay, K, G, D)) return f;
  switch (K) {
    case 1: return G == 16 ? pick3<1, 16>(planes, cat, pay) : pick3<1, 8>(planes, cat, pay);
    case 2: return pick3<2, 8>(planes, cat, pay);
    case 3: return pick3<3, 6>(planes, cat, pay);
    case 4: return pick3<4, 8>(planes, cat, pay);
    case 5: return pick3<5, 5>(planes, cat, pay);
    case 6: return pick3<6, 6>(planes, cat, pay);
    case 7: return pick3<7, 7>(planes, cat, pay);
    case 8: return pick3<8, 8>(planes, cat, pay);
    case 10: return pick3<10, 10>(planes, cat, pay);
    case 12: return pick3<12, 12>(planes, cat, pay);
    case 16: return pick3<16, 16>(planes, cat, pay);
    default: return pick3<0, 8>(planes, cat, pay);
  }
}

template <int KT, int G>
TopKernelFn pick3_top(bool planes, bool cat, bool pay) {
  if (planes)
    return cat ? forest_complete_top_kernel<KT, G, true, true>
               : forest_complete_top_kernel<KT, G, true, false>;
  if (cat) return forest_complete_top_kernel<KT, G, false, true>;
  return pay ? forest_complete_top_kernel<KT, G, false, false, 0, true>
             : forest_complete_top_kernel<KT, G, false, false>;
}

// The same (K, G) pairs as pick; a fixed-depth build where one exists.
TopKernelFn pick_top(bool planes, bool cat, bool pay, int K, int G, int D) {
  if (TopKernelFn f = pick_top_fixed(planes, cat, pay, K, G, D)) return f;
  switch (K) {
    case 1: return G == 16 ? pick3_top<1, 16>(planes, cat, pay) : pick3_top<1, 8>(planes, cat, pay);
    case 2: return pick3_top<2, 8>(planes, cat, pay);
    case 3: return pick3_top<3, 6>(planes, cat, pay);
    case 4: return pick3_top<4, 8>(planes, cat, pay);
    case 5: return pick3_top<5, 5>(planes, cat, pay);
    case 6: return pick3_top<6, 6>(planes, cat, pay);
    case 7: return pick3_top<7, 7>(planes, cat, pay);
    case 8: return pick3_top<8, 8>(planes, cat, pay);
    case 10: return pick3_top<10, 10>(planes, cat, pay);
    case 12: return pick3_top<12, 12>(planes, cat, pay);
    case 16: return pick3_top<16, 16>(planes, cat, pay);
    default: return pick3_top<0, 8>(planes, cat, pay);
  }
}

}  // namespace
}  // namespace complete

using complete::KernelFn;
using complete::TopKernelFn;

cudaError_t launch_complete_top(bool planes, bool cat, bool pay, const KArgs& a,
                                const TopRecords& top, size_t smem, int grid,
                                cudaStream_t stream, int* occupancy_out) {
  TopKernelFn fn = complete::pick_top(planes, cat, pay, a.K, a.G, a.D);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  if (occupancy_out)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occupancy_out, fn, a.R, smem);
  fn<<<grid, a.R, smem, stream>>>(a, top);
  return cudaGetLastError();
}

cudaError_t launch_complete(bool planes, bool cat, bool pay, const KArgs& a, size_t smem,
                            int grid, cudaStream_t stream, int* occupancy_out) {
  KernelFn fn = complete::pick(planes, cat, pay, a.K, a.G, a.D);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  if (occupancy_out)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occupancy_out, fn, a.R, smem);
  fn<<<grid, a.R, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb
