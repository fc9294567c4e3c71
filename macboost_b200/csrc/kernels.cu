// sm_100a forest-inference kernels.
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
// Execution model: one persistent CTA per SM; one thread per row of a row
// tile.  A tile's feature columns are brought from HBM into shared memory with
// cp.async.bulk (one bulk copy per staged feature: a contiguous run of R fp32
// values of the feature-major input), completing on an mbarrier; with two
// tile buffers the next tile streams in while the current one is scored.  The
// forest (or, when it is larger than shared memory, one block of trees at a
// time, double-buffered) is staged the same way.  Each thread walks G trees
// at once -- G independent dependency chains of shared-memory loads -- and
// adds their leaves to its fp32 accumulators strictly in tree order.  The tile
// keeps one feature per 4*R-byte row of shared memory with R a multiple of 32,
// so the per-level gather x[feature][row] of a warp touches 32 distinct banks
// whatever features its lanes read.  Node records of one level of a tree are
// contiguous, so the record loads of a warp also stay within few wavefronts.
//
// Tensor cores are not used: tree traversal is a data-dependent walk, not a
// dense contraction.  Every mbarrier wait is bounded (globaltimer); on expiry
// the CTA records kErrWaitTimeout in *err and all its threads return together.
#include <cuda_runtime.h>

#include <cstdint>

#include "forest.h"
#include "kernels.h"

namespace mb {
namespace {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of an mbarrier.  Returns false on timeout
// (after recording the error).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
}

struct Smem {
  uint32_t bars;          // shared address of 4 mbarriers: tile0, tile1, forest0, forest1
  float* tiles;           // tile_bufs * tile_floats
  unsigned tile_floats;
  unsigned char* fbuf;    // 1 or 2 forest buffers of buf_bytes
};

__device__ __forceinline__ Smem carve(unsigned char* smem, const KArgs& a) {
  Smem s;
  s.bars = smem_u32(smem);
  s.tiles = reinterpret_cast<float*>(smem + kSmemHeader);
  const unsigned tile_slots = a.S > 0 ? unsigned(a.S) : 1u;  // as sized by the host plan
  const unsigned tile_bytes = (tile_slots * unsigned(a.R) * 4u + 127u) & ~127u;
  s.tile_floats = tile_bytes / 4u;
  s.fbuf = smem + kSmemHeader + size_t(a.tile_bufs) * tile_bytes;
  return s;
}

// Warp 0: stage the feature columns of row tile `tile` with bulk copies.
__device__ __forceinline__ void issue_tile(const KArgs& a, long long tile, float* dst,
                                           uint32_t bar, int lane) {
  const long long r0 = tile * a.R;
  long long nv = a.rows - r0;
  if (nv > a.R) nv = a.R;
  const uint32_t nbytes = uint32_t(((nv + 3) & ~3ll) * 4);
  if (lane == 0) mbar_arrive_expect_tx(bar, nbytes * uint32_t(a.S));
  __syncwarp();
  for (int s = lane; s < a.S; s += 32) {
    const long long f = a.slot_feature ? a.slot_feature[s] : s;
    bulk_g2s(smem_u32(dst + size_t(s) * a.R), a.x + f * a.ld + r0, nbytes, bar);
  }
}

// All threads: stage a row tile with ordinary coalesced loads (used when the
// input's address or stride does not allow 16-byte bulk copies).
__device__ __forceinline__ void load_tile_sync(const KArgs& a, long long tile, float* dst) {
  const long long row = tile * a.R + threadIdx.x;
  const bool ok = row < a.rows;
  for (int s = 0; s < a.S; ++s) {
    const long long f = a.slot_feature ? a.slot_feature[s] : s;
    dst[size_t(s) * a.R + threadIdx.x] = ok ? __ldg(a.x + f * a.ld + row) : 0.0f;
  }
}

// Warp 0: stage forest block b.
__device__ __forceinline__ void issue_block(const KArgs& a, int b, unsigned char* dst,
                                            uint32_t bar, int lane) {
  const unsigned long long off = a.block_off[b];
  const uint32_t bytes = uint32_t(a.block_off[b + 1] - off);
  if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
  __syncwarp();
  constexpr uint32_t kChunk = 16384;
  for (uint32_t o = uint32_t(lane) * kChunk; o < bytes; o += 32u * kChunk) {
    const uint32_t n = (bytes - o < kChunk) ? (bytes - o) : kChunk;
    bulk_g2s(smem_u32(dst + o), a.blob + off + o, n, bar);
  }
}

// Routing decision for one node: 1 = right child, 0 = left child.
template <bool CAT>
__device__ __forceinline__ uint32_t go_right(uint2 r, float v, const unsigned* masks,
                                             int data_bins) {
  if (CAT && (r.x & kRecCategorical)) {
    int code = data_bins;                    // non-finite / unseen -> missing bin
    if (isfinite(v)) {
      const float q = rintf(v);              // round half to even
      if (q >= 0.0f && q < float(data_bins)) code = int(q);
    }
    uint32_t left;
    if (r.x & kRecFullMask)
      left = (__ldg(masks + size_t(r.y) * 8 + (code >> 5)) >> (code & 31)) & 1u;
    else
      left = code < 32 ? (r.y >> code) & 1u : (r.x & kRecDefaultLeft);
    return left ^ 1u;
  }
  const float t = __uint_as_float(r.y);
  // default-left: NaN fails v > t and goes left; default-right: NaN fails
  // v <= t and goes right; every other value goes left iff v <= t.
  return (r.x & kRecDefaultLeft) ? uint32_t(v > t) : uint32_t(!(v <= t));
}

// Per-thread accumulators: KT compile-time classes, or (KT == 0) up to 128.
template <int KT>
struct Acc {
  float v[KT];
  __device__ __forceinline__ void init(const float* base, int) {
#pragma unroll
    for (int c = 0; c < KT; ++c) v[c] = __ldg(base + c);
  }
  __device__ __forceinline__ void add(int j, int, float l) { v[j % KT] += l; }
  __device__ __forceinline__ float get(int c) const { return v[c]; }
  __device__ __forceinline__ int k(int) const { return KT; }
};
template <>
struct Acc<0> {
  float v[128];
  int K;
  __device__ __forceinline__ void init(const float* base, int K_) {
    K = K_;
    for (int c = 0; c < K; ++c) v[c] = __ldg(base + c);
  }
  __device__ __forceinline__ void add(int, int t, float l) { v[t % K] += l; }
  __device__ __forceinline__ float get(int c) const { return v[c]; }
  __device__ __forceinline__ int k(int) const { return K; }
};

template <int KT>
__device__ __forceinline__ void epilogue(const KArgs& a, const Acc<KT>& acc, long long row) {
  if (a.out == nullptr) return;
  const int K = acc.k(a.K);
  float* o = a.out;
  if (a.kind == kKindProba) {
    if (K == 1) {
      // MacBoostClassifier.predict_proba, binary (__init__.py:444-445), float64
      const double p = 1.0 / (1.0 + exp(-double(acc.get(0))));
      o[2 * row] = float(1.0 - p);
      o[2 * row + 1] = float(p);
    } else {
      // softmax in float64 (__init__.py:440-442)
      double m = double(acc.get(0));
      for (int c = 1; c < K; ++c) m = fmax(m, double(acc.get(c)));
      double s = 0.0;
      for (int c = 0; c < K; ++c) s += exp(double(acc.get(c)) - m);
      for (int c = 0; c < K; ++c) o[row * K + c] = float(exp(double(acc.get(c)) - m) / s);
    }
    return;
  }
  if (a.kind == kKindPredict && a.log_link) {
    // poisson / tweedie mean, exp of the fp32 margin (Booster.swift:1995-1997)
    for (int c = 0; c < K; ++c) o[row * K + c] = float(exp(double(acc.get(c))));
    return;
  }
  for (int c = 0; c < K; ++c) o[row * K + c] = acc.get(c);
}

// Shared per-tile pipeline: waits, prefetches and the bounded-wait abort
// protocol; `score(block_ptr, block_index, first_tree, xrow, acc)` scores one
// forest block for this thread's row.
template <int KT, class ScoreBlock>
__device__ __forceinline__ void run_tiles(const KArgs& a, unsigned char* smem, ScoreBlock score) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const Smem sm = carve(smem, a);
  const uint32_t bar_tile0 = sm.bars, bar_f0 = sm.bars + 16;
  const bool streaming = a.nblocks > 1;
  const bool bulk = a.bulk && a.S > 0;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(sm.bars + 8u * i, 1);
    fence_mbar_init();
  }
  __syncthreads();

  long long tile = blockIdx.x;
  if (tile >= a.ntiles) return;  // uniform over the CTA

  if (warp == 0) {
    if (a.nblocks > 0) issue_block(a, 0, sm.fbuf, bar_f0, lane);
    if (bulk) issue_tile(a, tile, sm.tiles, bar_tile0, lane);
  }
  unsigned fseq = 0;  // forest blocks consumed by this CTA

  for (int k = 0; tile < a.ntiles; tile += gridDim.x, ++k) {
    const int tb = (a.tile_bufs == 2) ? (k & 1) : 0;
    float* tl = sm.tiles + size_t(tb) * sm.tile_floats;
    const long long next = tile + gridDim.x;
    if (bulk && a.tile_bufs == 2 && warp == 0 && next < a.ntiles) {
      // buffer tb^1 held tile k-1, released by the barrier ending that iteration
      if (lane == 0) fence_proxy_async();
      __syncwarp();
      issue_tile(a, next, sm.tiles + size_t(tb ^ 1) * sm.tile_floats, bar_tile0 + 8u * (tb ^ 1),
                 lane);
    }
    if (bulk) {
      const uint32_t parity = (a.tile_bufs == 2) ? uint32_t((k >> 1) & 1) : uint32_t(k & 1);
      const bool ok = mbar_wait(bar_tile0 + 8u * tb, parity, a.err);
      if (__syncthreads_or(!ok)) return;
    } else if (a.S > 0) {
      load_tile_sync(a, tile, tl);
      __syncthreads();
    }

    const long long row = tile * a.R + tid;
    const float* xrow = tl + tid;  // slot s of this row at xrow[s * R]
    Acc<KT> acc;
    acc.init(a.base, a.K);
    for (int b = 0; b < a.nblocks; ++b) {
      const unsigned char* fb;
      if (streaming) {
        // release the buffer of block fseq-1, then prefetch block fseq+1 into it
        __syncthreads();
        if (warp == 0) {
          int nb = b + 1;
          if (nb == a.nblocks) nb = (next < a.ntiles) ? 0 : -1;
          if (nb >= 0) {
            if (lane == 0) fence_proxy_async();
            __syncwarp();
            issue_block(a, nb, sm.fbuf + size_t((fseq + 1) & 1) * a.buf_bytes,
                        bar_f0 + 8u * ((fseq + 1) & 1), lane);
          }
        }
        const bool ok = mbar_wait(bar_f0 + 8u * (fseq & 1), (fseq >> 1) & 1, a.err);
        if (__syncthreads_or(!ok)) return;
        fb = sm.fbuf + size_t(fseq & 1) * a.buf_bytes;
        ++fseq;
      } else {
        if (k == 0) {
          const bool ok = mbar_wait(bar_f0, 0, a.err);
          if (__syncthreads_or(!ok)) return;
        }
        fb = sm.fbuf;
      }
      score(fb, b, row, xrow, acc);
    }
    if (row < a.rows) epilogue<KT>(a, acc, row);
    __syncthreads();  // every thread is done with tile buffer tb
    if (bulk && a.tile_bufs == 1 && warp == 0 && next < a.ntiles) {
      if (lane == 0) fence_proxy_async();
      __syncwarp();
      issue_tile(a, next, sm.tiles, bar_tile0, lane);
    }
  }
}

// ---------------------------------------------------------------------------
// Complete layout: every tree is a complete heap of depth D.
// ---------------------------------------------------------------------------
template <int KT, bool CAT>
__global__ void __launch_bounds__(512, 1) forest_complete_kernel(const KArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int G = KT == 0 ? 8 : (KT >= 8 ? KT : KT * (8 / KT));
  const int D = a.D;
  const int NI = (1 << D) - 1;
  const int NL = 1 << D;
  const int R = a.R;
  auto score = [&](const unsigned char* fb, int b, long long row, const float* xrow,
                   Acc<KT>& acc) {
    const uint2* recs = reinterpret_cast<const uint2*>(fb);
    const float* leaves = reinterpret_cast<const float*>(fb + a.leaf_off);
    const int t_block = b * a.Tb;
    for (int g0 = 0; g0 < a.Tb; g0 += G) {
      const uint2* rt = recs + size_t(g0) * NI;
      uint32_t n[G];
#pragma unroll
      for (int j = 0; j < G; ++j) n[j] = 0;
      for (int L = 0; L < D; ++L) {
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const uint2 r = rt[j * NI + n[j]];
          const float v = xrow[(r.x >> 4) * R];
          n[j] = 2 * n[j] + 1 + go_right<CAT>(r, v, a.masks, a.data_bins);
        }
      }
      const float* lv = leaves + size_t(g0) * NL;
#pragma unroll
      for (int j = 0; j < G; ++j) acc.add(j, t_block + g0 + j, lv[j * NL + int(n[j]) - NI]);
      if (a.out_leaf != nullptr && row < a.rows) {
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const int t = t_block + g0 + j;
          if (t < a.T)
            a.out_leaf[row * a.T + t] = __ldg(a.leaf_heap + size_t(t) * NL + int(n[j]) - NI);
        }
      }
    }
  };
  run_tiles<KT>(a, smem, score);
}

// ---------------------------------------------------------------------------
// Explicit layout: breadth-first nodes, children adjacent, leaf records.
// ---------------------------------------------------------------------------
template <int KT, bool CAT>
__global__ void __launch_bounds__(512, 1) forest_explicit_kernel(const KArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int G = KT == 0 ? 8 : (KT >= 8 ? KT : KT * (8 / KT));
  const int R = a.R;
  auto score = [&](const unsigned char* fb, int b, long long row, const float* xrow,
                   Acc<KT>& acc) {
    // block header: [0] trees in the block, [1] index of its first tree,
    // [4 + i] first record of tree i
    const unsigned* head = reinterpret_cast<const unsigned*>(fb);
    const int ntrees = int(head[0]);
    const int t_block = int(head[1]);
    const uint2* recs =
        reinterpret_cast<const uint2*>(fb + ((16u + 4u * unsigned(ntrees) + 15u) & ~15u));
    for (int g0 = 0; g0 < ntrees; g0 += G) {
      uint32_t start[G], n[G];
      uint2 r[G];
#pragma unroll
      for (int j = 0; j < G; ++j) {
        start[j] = head[4 + g0 + j];
        n[j] = start[j];
        r[j] = recs[n[j]];
      }
      while (true) {
        bool any = false;
#pragma unroll
        for (int j = 0; j < G; ++j) {
          if (!(r[j].x & kRecLeaf)) {
            const float v = xrow[((r[j].x >> 4) & 0xFFFu) * R];
            n[j] = start[j] + (r[j].x >> 16) + go_right<CAT>(r[j], v, a.masks, a.data_bins);
            r[j] = recs[n[j]];
            any = true;
          }
        }
        if (!any) break;
      }
#pragma unroll
      for (int j = 0; j < G; ++j) acc.add(j, t_block + g0 + j, __uint_as_float(r[j].y));
      if (a.out_leaf != nullptr && row < a.rows) {
        const size_t rec_base = a.block_rec_base[b];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const int t = t_block + g0 + j;
          if (t < a.T) a.out_leaf[row * a.T + t] = __ldg(a.leaf_heap + rec_base + n[j]);
        }
      }
    }
  };
  run_tiles<KT>(a, smem, score);
}

}  // namespace
}  // namespace mb

namespace mb {
namespace {

// Row-major [rows][F] -> feature-major [F][ld], 32x32 tiles through shared
// memory (padded against bank conflicts).
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ in,
                                                        long long rows, int F,
                                                        float* __restrict__ out, long long ld) {
  __shared__ float t[32][33];
  const long long r0 = static_cast<long long>(blockIdx.x) * 32;
  const int f0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long r = r0 + i;
    const int f = f0 + threadIdx.x;
    if (r < rows && f < F) t[i][threadIdx.x] = in[r * F + f];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int f = f0 + i;
    const long long r = r0 + threadIdx.x;
    if (r < rows && f < F) out[f * ld + r] = t[threadIdx.x][i];
  }
}

using KernelFn = void (*)(const KArgs);

template <int KT>
KernelFn pick_k(int layout, bool cat) {
  if (layout == 0)
    return cat ? forest_complete_kernel<KT, true> : forest_complete_kernel<KT, false>;
  return cat ? forest_explicit_kernel<KT, true> : forest_explicit_kernel<KT, false>;
}

KernelFn pick(int layout, int cat, int K) {
  const bool c = cat != 0;
  switch (K) {
    case 1: return pick_k<1>(layout, c);
    case 2: return pick_k<2>(layout, c);
    case 3: return pick_k<3>(layout, c);
    case 4: return pick_k<4>(layout, c);
    case 5: return pick_k<5>(layout, c);
    case 6: return pick_k<6>(layout, c);
    case 7: return pick_k<7>(layout, c);
    case 8: return pick_k<8>(layout, c);
    case 9: return pick_k<9>(layout, c);
    case 10: return pick_k<10>(layout, c);
    case 11: return pick_k<11>(layout, c);
    case 12: return pick_k<12>(layout, c);
    case 13: return pick_k<13>(layout, c);
    case 14: return pick_k<14>(layout, c);
    case 15: return pick_k<15>(layout, c);
    case 16: return pick_k<16>(layout, c);
    default: return pick_k<0>(layout, c);
  }
}

}  // namespace

cudaError_t launch_forest(int layout, int cat, const KArgs& a, size_t smem, int grid,
                          cudaStream_t stream) {
  KernelFn fn = pick(layout, cat, a.K);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  fn<<<grid, a.R, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t forest_occupancy(int layout, int cat, int K, int R, size_t smem, int* ctas) {
  KernelFn fn = pick(layout, cat, K);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, fn, R, smem);
}

cudaError_t launch_transpose(const float* in, long long rows, int F, float* out, long long ld,
                             cudaStream_t stream) {
  if (rows <= 0 || F <= 0) return cudaSuccess;
  dim3 grid(unsigned((rows + 31) / 32), unsigned((F + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(in, rows, F, out, ld);
  return cudaGetLastError();
}

}  // namespace mb
