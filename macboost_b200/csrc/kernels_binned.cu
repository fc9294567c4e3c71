// sm_100a kernels for binned data: binning raw values into the trainer's
// tiled bin layout, and walking trees in split form over binned rows.
//
// Replaces the Metal kernels bin_data (Sources/MacBoost/Shaders.swift:41-76),
// predict_tree_binned and assign_leaves (Shaders.swift:1741-1781) with their
// goes_left rule on a bin (Shaders.swift:466-476).  Layout (bin_index,
// Shaders.swift:37-39): features in tiles of 8; for n rows, bin (f, i) sits at
// (f / 8) * n * 8 + i * 8 + f % 8, so the 8 bins of one row and tile are one
// 8-byte word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"
#include "kernels_common.cuh"

namespace mb {
namespace {

// The reference's search for a value's bin (Shaders.swift:41-76) is a binary
// search over the feature's n = dataBins - 1 upper edges:
//   lo = 0, hi = n; while (lo < hi) { mid = (lo + hi) / 2;
//                                     if (v > e[mid]) lo = mid + 1; else hi = mid; }
// Its probes form a fixed binary tree of mids that depends on n only.  That
// tree is laid out breadth-first (node p's children at 2p + 1 and 2p + 2,
// padded to a complete tree of depth D) with the edge each node compares, so
// a search is D steps of p = 2p + 1 + (v > E[p]) over a table in shared
// memory: level k of the search reads 2^k consecutive entries (one
// shared-memory wavefront for k <= 5), where the sorted array's probes are
// spread over the whole row of edges.  Padding nodes compare against +Inf, so
// every non-NaN value goes left through them (v > +Inf is false) and ends at
// the leftmost leaf below the reference search's terminal, where `res` holds
// that terminal's bin.  The probes and comparisons are the reference's, in its
// order, so unsorted or repeated edges bin exactly as there.
struct BinSearch {
  unsigned char edge[255];  // edge index compared at node p < 2^D - 1; 0xFF: padding
  unsigned char res[256];   // bin at leaf position p - (2^D - 1)
  int D;                    // search steps
};

// Node p of the mid tree over [lo, hi] at depth d; `D` its maximum depth.
void build_mid_tree(BinSearch& t, unsigned lo, unsigned hi, unsigned p, int d, int D) {
  if (lo >= hi) {
    for (; d < D; ++d) {  // padding below a terminal: always left
      t.edge[p] = 0xFF;
      p = 2 * p + 1;
    }
    t.res[p - ((1u << D) - 1)] = static_cast<unsigned char>(lo);
    return;
  }
  const unsigned mid = (lo + hi) >> 1;
  t.edge[p] = static_cast<unsigned char>(mid);
  build_mid_tree(t, lo, mid, 2 * p + 1, d + 1, D);
  build_mid_tree(t, mid + 1, hi, 2 * p + 2, d + 1, D);
}

int mid_tree_depth(unsigned lo, unsigned hi) {
  if (lo >= hi) return 0;
  const unsigned mid = (lo + hi) >> 1;
  return 1 + std::max(mid_tree_depth(lo, mid), mid_tree_depth(mid + 1, hi));
}

// Persistent blocks of 256 threads over one tile of 8 features (blockIdx.y):
// the tile's search tables are staged in shared memory once per block, then
// each thread bins its rows' 8 values -- the 8 searches interleaved, D steps
// each -- and packs them into one 8-byte store (a warp writes 256 contiguous
// bytes).
template <int DT>  // search steps fixed at compile time (8: 256 bins), or 0: tree.D
__global__ void __launch_bounds__(256, 3) bin_data_kernel(const float* __restrict__ x, long long rows,
                                                       long long cols, long long ld, int layout,
                                                       const float* __restrict__ edges,
                                                       int num_bins,
                                                       const unsigned char* __restrict__ cat,
                                                       unsigned char* __restrict__ bins,
                                                       const BinSearch tree) {
  __shared__ float E[8][256];
  __shared__ unsigned char res[256];
  const long long g = blockIdx.y;
  const unsigned data_bins = unsigned(num_bins) - 1u;
  const unsigned n = data_bins - 1u;  // edges per feature
  const int D = tree.D;
  const unsigned inner = (1u << D) - 1u;
  for (unsigned q = threadIdx.x; q < 8u * 256u; q += blockDim.x) {
    const unsigned k = q >> 8, p = q & 255u;
    const long long f = g * 8 + k;
    float e = __int_as_float(0x7f800000);  // +Inf: padding, and features past cols
    if (p < inner && f < cols && tree.edge[p] != 0xFF) e = __ldg(edges + size_t(f) * n + tree.edge[p]);
    E[k][p] = e;
  }
  for (unsigned q = threadIdx.x; q < 256u; q += blockDim.x) res[q] = tree.res[q];
  unsigned catbits = 0;  // bit k: feature g * 8 + k is categorical
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if (g * 8 + k < cols && __ldg(cat + g * 8 + k) == 1) catbits |= 1u << k;
  __syncthreads();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
       i += (long long)gridDim.x * blockDim.x) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const long long f = g * 8 + k;
      v[k] = f < cols ? (layout == 0 ? __ldg(x + f * ld + i) : __ldg(x + i * cols + f)) : 0.0f;
    }
    // p: node of each feature's search, as a byte offset into its table row
    unsigned p[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) p[k] = 0;
    auto step = [&]() {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float e = *reinterpret_cast<const float*>(reinterpret_cast<const char*>(E[k]) + p[k]);
        p[k] = 2u * p[k] + (v[k] > e ? 8u : 4u);
      }
    };
    if (DT > 0) {
#pragma unroll
      for (int s2 = 0; s2 < DT; ++s2) step();
    } else {
      for (int s2 = 0; s2 < D; ++s2) step();
    }
    unsigned long long packed = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      unsigned b;
      if (isnan(v[k])) {
        b = data_bins;  // the reserved missing bin
      } else if ((catbits >> k) & 1u) {
        // clamp(int(rint(v)), 0, dataBins - 1); the int conversion saturates
        const float r = rintf(v[k]);
        b = r < 0.0f ? 0u : (r > float(data_bins - 1) ? data_bins - 1 : unsigned(int(r)));
      } else {
        b = res[(p[k] >> 2) - inner];
      }
      if (g * 8 + k >= cols) b = 0;  // bytes past the last feature stay zero
      packed |= (unsigned long long)(b & 0xFFu) << (8 * k);
    }
    *reinterpret_cast<unsigned long long*>(bins + (g * rows + i) * 8) = packed;
  }
}

// Final heap index of row i in tree t, walking at most max_depth splits.
// A split naming a feature outside the matrix or a child outside the tree
// sets kErrBadTree and ends the walk there.
__device__ __forceinline__ unsigned walk_binned(const BinnedArgs& a, int t, long long i) {
  const long long b0 = __ldg(a.tree_off + t);
  const long long nodes = __ldg(a.tree_off + t + 1) - b0;
  unsigned node = 0;
  for (int d = 0; d < a.max_depth; ++d) {
    const int f = __ldg(a.feature + b0 + node);
    if (f < 0) break;
    if (f >= a.cols || 2ll * node + 2 >= nodes) {
      atomicOr(a.err, kErrBadTree);
      break;
    }
    const unsigned b = a.bins[(size_t(f >> 3) * size_t(a.n) + size_t(i)) * 8 + (f & 7)];
    const unsigned fl = __ldg(a.flags + b0 + node);
    bool left;
    if (fl & 2u)
      left = (__ldg(a.catmask + (b0 + node) * 8 + (b >> 5)) >> (b & 31)) & 1u;
    else if (b == unsigned((a.num_bins - 1) & 0xFF))
      left = (fl & 1u) != 0;
    else
      left = b <= (__ldg(a.sbin + b0 + node) & 0xFFu);
    node = 2 * node + 1 + (left ? 0 : 1);
  }
  return node;
}

// The same walk reading bins from a staged row tile: tile tb holds, per
// 8-feature tile g, the R rows' 8-byte words at tb + (g * R + r) * 8.
__device__ __forceinline__ unsigned walk_staged(const BinnedArgs& a, int t, uint32_t tb, int r,
                                                int R) {
  const long long b0 = __ldg(a.tree_off + t);
  const unsigned nodes = unsigned(__ldg(a.tree_off + t + 1) - b0);
  const int* feat = a.feature + b0;
  const unsigned* flags = a.flags + b0;
  const unsigned* sbin = a.sbin + b0;
  const uint32_t row = tb + uint32_t(r) * 8u;
  const uint32_t gstride = uint32_t(R) * 8u;
  const unsigned last = unsigned((a.num_bins - 1) & 0xFF);
  unsigned node = 0;
  for (int d = 0; d < a.max_depth; ++d) {
    const int f = __ldg(feat + node);
    if (f < 0) break;
    if (f >= a.cols || 2u * node + 2u >= nodes) {
      atomicOr(a.err, kErrBadTree);
      break;
    }
    unsigned b;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(b) : "r"(row + uint32_t(f >> 3) * gstride + uint32_t(f & 7)));
    const unsigned fl = __ldg(flags + node);
    bool left;
    if (fl & 2u)
      left = (__ldg(a.catmask + (size_t(b0) + node) * 8 + (b >> 5)) >> (b & 31)) & 1u;
    else if (b == last)
      left = (fl & 1u) != 0;
    else
      left = b <= (__ldg(sbin + node) & 0xFFu);
    node = 2u * node + (left ? 1u : 2u);
  }
  return node;
}

// Staged node records (one 8-byte record per node, every tree of the call,
// copied to shared memory once per CTA): x = split bin (bits 0-7) | default
// left (bit 8) | categorical (bit 9) | leaf (bit 10) | bad split (bit 11) |
// byte offset of the feature's bin in a staged row (bits 15-31: tile g at
// g * R * 8, bin f % 8 within the row's word); y = the node's global index
// (its categorical mask).  A bad split names a feature outside the matrix or
// a child outside its tree, checked once here instead of at every level.
constexpr uint32_t kRecBinDL = 1u << 8, kRecBinCat = 1u << 9, kRecBinLeaf = 1u << 10,
                   kRecBinBad = 1u << 11;
constexpr int kRecBinOffShift = 15;

__device__ __forceinline__ void stage_records(const BinnedArgs& a, uint32_t recs, int R) {
  const long long g0 = __ldg(a.tree_off);
  for (int t = 0; t < a.T; ++t) {
    const long long b0 = __ldg(a.tree_off + t);
    const long long nodes = __ldg(a.tree_off + t + 1) - b0;
    for (long long n = threadIdx.x; n < nodes; n += blockDim.x) {
      const long long q = b0 + n;
      const int f = __ldg(a.feature + q);
      uint32_t x;
      if (f < 0) {
        x = kRecBinLeaf;
      } else if (f >= a.cols || 2ll * n + 2 >= nodes) {
        x = kRecBinBad;
      } else {
        const unsigned fl = __ldg(a.flags + q);
        const uint32_t off = uint32_t(f >> 3) * uint32_t(R) * 8u + uint32_t(f & 7);
        x = (__ldg(a.sbin + q) & 0xFFu) | ((fl & 1u) ? kRecBinDL : 0u) |
            ((fl & 2u) ? kRecBinCat : 0u) | (off << kRecBinOffShift);
      }
      asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(recs + uint32_t(q - g0) * 8u),
                   "r"(x), "r"(uint32_t(q)) : "memory");
    }
  }
}

// The walk over staged records of one tree (records of its root at `tree`):
// the same rule as walk_staged.
__device__ __forceinline__ unsigned walk_records(const BinnedArgs& a, uint32_t tree,
                                                 uint32_t row, unsigned last) {
  unsigned node = 0;
  for (int d = 0; d < a.max_depth; ++d) {
    const uint2 r = dev::lds_v2(tree + node * 8u);
    if (r.x & (kRecBinLeaf | kRecBinBad)) {
      if (r.x & kRecBinBad) atomicOr(a.err, kErrBadTree);
      break;
    }
    unsigned b;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(b) : "r"(row + (r.x >> kRecBinOffShift)));
    bool left;
    if (r.x & kRecBinCat)
      left = (__ldg(a.catmask + size_t(r.y) * 8 + (b >> 5)) >> (b & 31)) & 1u;
    else
      left = (b == last) ? (r.x & kRecBinDL) != 0 : b <= (r.x & 0xFFu);
    node = 2u * node + (left ? 1u : 2u);
  }
  return node;
}

// Persistent CTAs over row tiles of R = blockDim rows; each tile's bins (one
// R x 8-byte run per feature tile, 16-byte aligned) arrive by cp.async.bulk,
// double-buffered on two mbarriers with bounded waits, so the bin matrix is
// streamed from HBM once and every level of the walk reads shared memory.
template <int KT, bool FOREST>
__global__ void __launch_bounds__(256) binned_staged_kernel(const BinnedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int R = blockDim.x, tid = threadIdx.x;
  const int groups = int((a.cols + 7) / 8);
  const uint32_t tile_bytes = uint32_t(groups) * uint32_t(R) * 8u;
  const uint32_t sbase = dev::smem_u32(smem);
  const uint32_t bar0 = sbase, buf0 = sbase + 128u;
  const long long ntiles = (a.n + R - 1) / R;
  auto issue = [&](long long tile, uint32_t buf) {
    const long long r0 = tile * R;
    const long long nr = a.n - r0 < R ? a.n - r0 : R;
    const uint32_t bytes = uint32_t(((nr + 1) & ~1ll) * 8);  // whole 16-byte units
    const uint32_t bar = bar0 + 8u * buf;
    dev::mbar_arrive_expect_tx(bar, bytes * uint32_t(groups));
    for (int g = 0; g < groups; ++g)
      dev::bulk_g2s(buf0 + buf * tile_bytes + uint32_t(g) * uint32_t(R) * 8u,
                    a.bins + (size_t(g) * size_t(a.n) + size_t(r0)) * 8, bytes, bar);
  };
  // node records after the two tile buffers, when every tree of the call fits
  const uint32_t recs = buf0 + 2u * tile_bytes;
  const long long total_nodes = __ldg(a.tree_off + a.T) - __ldg(a.tree_off);
  bool staged = total_nodes >= 0 && total_nodes * 8 <= (long long)a.rec_cap;
  if (staged) {  // uniform over the CTA: the offsets must not decrease
    bool mono = true;
    for (int t = tid; t < a.T; t += R)
      mono = mono && __ldg(a.tree_off + t + 1) >= __ldg(a.tree_off + t);
    staged = __syncthreads_and(mono);
  }
  const unsigned last = unsigned((a.num_bins - 1) & 0xFF);
  if (tid == 0) {
    dev::mbar_init(bar0, 1);
    dev::mbar_init(bar0 + 8, 1);
    dev::fence_mbar_init();
  }
  if (staged && blockIdx.x < ntiles) stage_records(a, recs, R);
  __syncthreads();
  if (tid == 0 && blockIdx.x < ntiles) issue(blockIdx.x, 0);
  uint32_t parity = 0;
  int k = 0;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++k) {
    const uint32_t buf = uint32_t(k & 1);
    const bool ok = dev::mbar_wait(bar0 + 8u * buf, (parity >> buf) & 1u, a.err);
    parity ^= 1u << buf;
    // all threads are done with the tile in the other buffer: prefetch into it
    if (__syncthreads_or(!ok)) return;
    if (tid == 0 && tile + gridDim.x < ntiles) issue(tile + gridDim.x, buf ^ 1u);
    const long long i = tile * R + tid;
    if (i < a.n) {
      const uint32_t tb = buf0 + buf * tile_bytes;
      const uint32_t row = tb + uint32_t(tid) * 8u;
      const long long g0 = __ldg(a.tree_off);
      auto walk = [&](int t) -> unsigned {
        if (!staged) return walk_staged(a, t, tb, tid, R);
        const long long b0 = __ldg(a.tree_off + t);
        if (__ldg(a.tree_off + t + 1) <= b0) {  // a tree without nodes
          atomicOr(a.err, kErrBadTree);
          return 0u;
        }
        return walk_records(a, recs + uint32_t(b0 - g0) * 8u, row, last);
      };
      if (!FOREST) {
        for (int t = 0; t < a.T; ++t) {
          const unsigned node = walk(t);
          if (a.preds)
            a.preds[size_t(t % a.K) * size_t(a.n) + i] += __ldg(a.leaf + __ldg(a.tree_off + t) + node);
          if (a.leaf_idx) a.leaf_idx[size_t(t) * size_t(a.n) + i] = int(node);
        }
      } else {
        dev::Acc<KT> acc;
        acc.init(a.base, a.K);
        for (int t = 0; t < a.T; ++t) {
          const unsigned node = walk(t);
          if (a.ka.kind == kKindLeaf)
            a.ka.out_leaf[size_t(i) * a.T + t] = int(node);
          else
            acc.add(t, t, __ldg(a.leaf + __ldg(a.tree_off + t) + node));
        }
        if (a.ka.kind != kKindLeaf) dev::epilogue<KT>(a.ka, acc, i);
      }
    }
  }
}

template <int KT>
__global__ void __launch_bounds__(256) binned_kernel(const BinnedArgs a) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    if (!a.forest_mode) {
      // predict_tree_binned / assign_leaves, one tree after the other
      for (int t = 0; t < a.T; ++t) {
        const unsigned node = walk_binned(a, t, i);
        if (a.preds) a.preds[size_t(t % a.K) * size_t(a.n) + i] += __ldg(a.leaf + __ldg(a.tree_off + t) + node);
        if (a.leaf_idx) a.leaf_idx[size_t(t) * size_t(a.n) + i] = int(node);
      }
      continue;
    }
    dev::Acc<KT> acc;
    acc.init(a.base, a.K);
    for (int t = 0; t < a.T; ++t) {
      const unsigned node = walk_binned(a, t, i);
      if (a.ka.kind == kKindLeaf)
        a.ka.out_leaf[size_t(i) * a.T + t] = int(node);
      else
        acc.add(t, t, __ldg(a.leaf + __ldg(a.tree_off + t) + node));
    }
    if (a.ka.kind != kKindLeaf) dev::epilogue<KT>(a.ka, acc, i);
  }
}

}  // namespace

cudaError_t launch_bin_data(const float* x, long long rows, long long cols, long long ld,
                            int layout, const float* edges, int num_bins,
                            const unsigned char* categorical, unsigned char* bins,
                            cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  if (num_bins < 3 || num_bins > 256) return cudaErrorInvalidValue;
  // the search tree of the reference's binary search over num_bins - 2 edges
  BinSearch tree{};
  const unsigned n = unsigned(num_bins) - 2u;
  tree.D = mid_tree_depth(0, n);
  build_mid_tree(tree, 0, n, 0, 0, tree.D);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (cols + 7) / 8;
  const long long blocks = (rows + 255) / 256;
  // about 8 blocks per SM over all feature tiles; each block loops over rows
  long long want = std::max<long long>(1, 8ll * sms / tiles);
  const dim3 grid(unsigned(std::min(blocks, want)), unsigned(tiles));
  if (tree.D == 8)
    bin_data_kernel<8><<<grid, 256, 0, stream>>>(x, rows, cols, ld, layout, edges, num_bins,
                                                 categorical, bins, tree);
  else
    bin_data_kernel<0><<<grid, 256, 0, stream>>>(x, rows, cols, ld, layout, edges, num_bins,
                                                 categorical, bins, tree);
  return cudaGetLastError();
}

cudaError_t launch_binned(const BinnedArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // staged tiles: every run (g * n + r0) * 8 bytes from a 16-byte aligned base
  // starts 16-byte aligned when n and R are even; two buffers of R x 8 bytes
  // per feature tile must fit in shared memory
  const long long groups = (a.cols + 7) / 8;
  const int R = 256;
  const size_t tiles = 128 + 2 * size_t(groups) * R * 8;
  if ((a.n % 2) == 0 && (reinterpret_cast<uintptr_t>(a.bins) % 16) == 0 && groups > 0 &&
      tiles <= 200 * 1024) {
    // node records (8 bytes each) beside the tiles: room for all of the call's
    // nodes when the caller counted them (up to 96 KB), else 8 KB, enough for
    // one tree of up to 1,024 nodes; the kernel stages them when they fit (it
    // reads the node count itself)
    BinnedArgs b = a;
    const size_t avail = std::min<size_t>(96 * 1024, 200 * 1024 - tiles);
    const size_t rec_bytes = a.node_hint > 0 ? size_t(a.node_hint) * 8 : 8 * 1024;
    b.rec_cap = rec_bytes <= avail ? uint32_t((rec_bytes + 15) / 16 * 16) : 0u;
    const size_t smem = tiles + b.rec_cap;
    const long long ntiles = (a.n + R - 1) / R;
    void (*k)(const BinnedArgs) = !a.forest_mode ? binned_staged_kernel<1, false>
                                  : a.K == 1     ? binned_staged_kernel<1, true>
                                                 : binned_staged_kernel<0, true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, R, smem);
    if (e != cudaSuccess) return e;
    long long want = (long long)(per_sm < 1 ? 1 : per_sm) * sms;
    const int cap = plan_grid_cap_from_env();  // MACBOOST_PLAN "grid" (tests)
    if (cap > 0 && want > cap) want = cap;
    const int grid = int(ntiles < want ? ntiles : want);
    k<<<grid, R, smem, stream>>>(b);
    return cudaGetLastError();
  }
  const long long want = (a.n + 255) / 256;
  const int grid = int(want < 16ll * sms ? want : 16ll * sms);
  if (a.forest_mode && a.K == 1)
    binned_kernel<1><<<grid, 256, 0, stream>>>(a);
  else
    binned_kernel<0><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb
