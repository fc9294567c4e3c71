// Device helpers shared by the forest kernels (see kernels_complete.cu for
// the execution model).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "forest.h"
#include "kernels.h"

namespace mb {
namespace dev {

// Threads per CTA the kernels are compiled for (mb::max_threads_for_group):
// groups of 10 or more trees, and more than two classes' accumulators, need
// the larger per-thread register budget of fewer threads.
template <int KT, int G>
struct Bounds {
  static constexpr int kMaxThreads =
      G >= 12 ? 256
              : (G >= 10 ? 384
                         : (KT == 0 || KT >= 5 ? 512 : ((KT == 1 || KT == 2) ? 768 : 640)));
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Shared-memory accesses by 32-bit shared-window address.  `volatile` keeps
// them in program order with respect to the mbarrier waits and barriers.
__device__ __forceinline__ uint2 lds_v2(uint32_t a) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
  return r;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds_v4f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_v4f(uint32_t a, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void sts_f32(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
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

// Bounded wait for phase `parity`; false (and *err |= timeout) after
// `limit_ns` of %globaltimer.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* err,
                                          unsigned long long limit_ns = kDefaultWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
}

// Warp 0: stage the staged slots of row tile `tile` with bulk copies, one per
// slot: R consecutive values of one feature (16-byte aligned, multiple of 16).
// With the stall hook the barrier expects the bytes but no copy is issued.
__device__ __forceinline__ void issue_tile(const KArgs& a, long long tile, uint32_t dst,
                                           uint32_t bar, int lane) {
  const long long r0 = tile * a.R;
  long long nv = a.rows - r0;
  if (nv > a.R) nv = a.R;
  const uint32_t nbytes = uint32_t(((nv + 3) & ~3ll) * 4);
  if (lane == 0) mbar_arrive_expect_tx(bar, nbytes * uint32_t(a.S_stage));
  __syncwarp();
  if (a.stall_tiles) return;
  for (int s = lane; s < a.S_stage; s += 32) {
    const long long f = a.stage_feature ? __ldg(a.stage_feature + s) : s;
    bulk_g2s(dst + uint32_t(s) * uint32_t(a.R) * 4u, a.x + f * a.ld + r0, nbytes, bar);
  }
}

// All threads: stage a row tile with ordinary coalesced loads (when the input
// address or stride does not allow bulk copies).
__device__ __forceinline__ void load_tile_sync(const KArgs& a, long long tile, uint32_t dst) {
  const long long row = tile * a.R + threadIdx.x;
  const bool ok = row < a.rows;
  for (int s = 0; s < a.S_stage; ++s) {
    const long long f = a.stage_feature ? __ldg(a.stage_feature + s) : s;
    sts_f32(dst + (uint32_t(s) * uint32_t(a.R) + threadIdx.x) * 4u,
            ok ? __ldg(a.x + f * a.ld + row) : 0.0f);
  }
}

// Each thread, its own row: fill the -Inf slots (NaN -> -Inf).
__device__ __forceinline__ void fill_left_planes(const KArgs& a, uint32_t rowbase) {
  for (int i = 0; i < a.n_conv; ++i) {
    const uint32_t src = uint32_t(__ldg(a.conv_src + i)) * uint32_t(a.R) * 4u;
    const uint32_t dst = uint32_t(__ldg(a.conv_dst + i)) * uint32_t(a.R) * 4u;
    const float v = lds_f32(rowbase + src);
    sts_f32(rowbase + dst, isnan(v) ? -__int_as_float(0x7f800000) : v);
  }
}

// The same for a warp's 32-row slice (slot s of the slice at slice + s * R
// * 4): eight lanes copy one slot's 128 bytes with 16-byte accesses, four
// slots per pass.  Lanes write other lanes' rows, so the warp syncs after.
__device__ __forceinline__ void fill_left_planes_warp(const KArgs& a, uint32_t slice, int lane) {
  const float ninf = -__int_as_float(0x7f800000);
  const uint32_t part = uint32_t(lane & 7) * 16u;
  for (int i = lane >> 3; i < a.n_conv; i += 4) {
    const uint32_t src = uint32_t(__ldg(a.conv_src + i)) * uint32_t(a.R) * 4u;
    const uint32_t dst = uint32_t(__ldg(a.conv_dst + i)) * uint32_t(a.R) * 4u;
    float4 v = lds_v4f(slice + src + part);
    v.x = isnan(v.x) ? ninf : v.x;
    v.y = isnan(v.y) ? ninf : v.y;
    v.z = isnan(v.z) ? ninf : v.z;
    v.w = isnan(v.w) ? ninf : v.w;
    sts_v4f(slice + dst + part, v);
  }
  __syncwarp();
}

// Category code of a staged value: rint(v) (half to even) when 0 <= rint(v) <
// dataBins, else dataBins, the missing bin (NaN and infinities fail both
// comparisons); Booster.swift:2052-2058, _pyinfer.py:80-86.
__device__ __forceinline__ uint32_t category_code(float v, int data_bins) {
  const float q = rintf(v);
  return (q >= 0.0f && q < float(data_bins)) ? uint32_t(q) : uint32_t(data_bins);
}

// Each thread, its own row: write the category codes of the code slots (as
// integer bits), from the value slots.
__device__ __forceinline__ void fill_codes(const KArgs& a, uint32_t rowbase) {
  for (int i = 0; i < a.n_codes; ++i) {
    const uint32_t src = uint32_t(__ldg(a.code_src + i)) * uint32_t(a.R) * 4u;
    const uint32_t dst = uint32_t(__ldg(a.code_dst + i)) * uint32_t(a.R) * 4u;
    sts_f32(rowbase + dst, __uint_as_float(category_code(lds_f32(rowbase + src), a.data_bins)));
  }
}

// The same for a warp's 32-row slice, eight lanes per slot with 16-byte
// accesses; the warp syncs after (lanes write other lanes' rows).
__device__ __forceinline__ void fill_codes_warp(const KArgs& a, uint32_t slice, int lane) {
  const uint32_t part = uint32_t(lane & 7) * 16u;
  for (int i = lane >> 3; i < a.n_codes; i += 4) {
    const uint32_t src = uint32_t(__ldg(a.code_src + i)) * uint32_t(a.R) * 4u;
    const uint32_t dst = uint32_t(__ldg(a.code_dst + i)) * uint32_t(a.R) * 4u;
    float4 v = lds_v4f(slice + src + part);
    v.x = __uint_as_float(category_code(v.x, a.data_bins));
    v.y = __uint_as_float(category_code(v.y, a.data_bins));
    v.z = __uint_as_float(category_code(v.z, a.data_bins));
    v.w = __uint_as_float(category_code(v.w, a.data_bins));
    sts_v4f(slice + dst + part, v);
  }
  __syncwarp();
}

// Warp 0: stage forest block b (16 KB bulk copies spread over the lanes).
__device__ __forceinline__ void issue_block(const KArgs& a, int b, uint32_t dst, uint32_t bar,
                                            int lane) {
  const unsigned long long off = a.block_off[b];
  const uint32_t bytes = uint32_t(a.block_off[b + 1] - off);
  if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
  __syncwarp();
  constexpr uint32_t kChunk = 16384;
  for (uint32_t o = uint32_t(lane) * kChunk; o < bytes; o += 32u * kChunk) {
    const uint32_t n = (bytes - o < kChunk) ? (bytes - o) : kChunk;
    bulk_g2s(dst + o, a.blob + off + o, n, bar);
  }
}

// Routing decision: 1 = right child.  PLANES: numeric records address the
// slot of their default direction and compare unordered; otherwise bit0 of
// the record selects the ordered compare for default-left, unless NONAN (a
// tile without NaN) makes both compares equal.  CAT: categorical records
// (bit1) test the node's mask at the value's code.  PAY (no planes, no
// categorical splits): the record word itself is the fmax operand below
// (kRecPayloadLeft/Right), one instruction less per node than the shift.
template <bool PLANES, bool CAT, bool NONAN = false, bool PAY = false>
__device__ __forceinline__ uint32_t route(uint2 r, uint32_t rowbase, const unsigned* masks,
                                          int data_bins) {
  const uint32_t addr = rowbase + ((PLANES && !CAT) ? r.x : (r.x & kRecSlotMask));
  const float v = lds_f32(addr);
  if constexpr (CAT) {
    // Both decisions, then a select: the 32 rows of a warp sit at categorical
    // and numeric nodes alike below the root, and a branch would run both
    // sides anyway.  Numeric: as below (the record's low bits are the
    // default-left bit and zeros only for numeric records; the categorical
    // result replaces the other).  Categorical: categorical records address a
    // slot of category codes (fill_codes wrote them when the tile landed), and
    // the node's mask bit at the code decides.
    const float t = __uint_as_float(r.y);
    uint32_t right_num;
    if (PLANES || NONAN) {
      right_num = uint32_t(!(v <= t));
    } else {
      const float c = __uint_as_float(__funnelshift_l(0u, 0x7FC00000u, r.x));
      right_num = uint32_t(!(fmaxf(v, c) <= t));
    }
    const uint32_t code = __float_as_uint(v);
    uint32_t left;
    if (r.x & kRecFullMask)  // a mask that bits 32..dataBins do not share: in memory
      left = (__ldg(masks + size_t(r.y) * 8 + (code >> 5)) >> (code & 31u)) & 1u;
    else
      left = code < 32u ? (r.y >> (code & 31u)) & 1u : (r.x & kRecDefaultLeft);
    return (r.x & kRecCategorical) ? (left ^ 1u) : right_num;
  }
  const float t = __uint_as_float(r.y);
  // NONAN: the row tile holds no NaN, so the default direction cannot matter
  // and v > t == !(v <= t) (thresholds and leaf values are never NaN)
  if (PLANES || NONAN) return uint32_t(!(v <= t));
  // NaN to the default side with one unordered compare: max(v, -Inf) turns
  // NaN into -Inf (left of every threshold) and leaves any other value as it
  // is; max(v, NaN) leaves every value, NaN included, as it is, and the
  // unordered compare sends NaN right (fmax returns the non-NaN operand).
  // c is 0x7FC00000 (NaN) shifted left by the default-left bit: 0xFF800000
  // (-Inf).  A numeric record's low five bits are that bit (bit 0) and zeros
  // (slot offsets are multiples of 128 bytes), and the funnel shift takes its
  // count modulo 32, so the record word itself is the shift count.
  static_assert(kRecDefaultLeft == 1u && (kRecSlotMask & 31u) == 0u, "record layout");
  // PAY: r.x is a NaN (default right: fmax keeps v) or a float at or below
  // -2^127 that no default-left threshold lies under (fmax turns NaN into a
  // value left of the threshold; a value below it is left either way).
  static_assert(!PAY || (!PLANES && !CAT), "payload records: no planes, no categorical splits");
  if constexpr (PAY) return uint32_t(!(fmaxf(v, __uint_as_float(r.x)) <= t));
  const float c = __uint_as_float(__funnelshift_l(0u, 0x7FC00000u, r.x));
  return uint32_t(!(fmaxf(v, c) <= t));
}

// Leaf-index output (kKindLeaf, row-major rows x T int32): this thread's row
// gets the n <= G consecutive indices of a tree group at p with the widest
// stores its alignment allows -- 16-byte stores when the run is a whole group
// of a multiple of 4 trees on a 16-byte boundary (T and the group start
// multiples of 4), so that a warp's store covers whole 32-byte sectors over
// two instructions instead of writing 4 bytes of 32 sectors in each of G.
template <int G>
__device__ __forceinline__ void store_leaf_run(int* p, const int (&v)[G], int n) {
  const uintptr_t ad = reinterpret_cast<uintptr_t>(p);
  if (G % 4 == 0 && n == G && (ad & 15u) == 0) {
#pragma unroll
    for (int j = 0; j < G; j += 4)
      asm volatile("st.global.v4.s32 [%0], {%1, %2, %3, %4};" ::"l"(p + j), "r"(v[j]),
                   "r"(v[(j + 1) % G]), "r"(v[(j + 2) % G]), "r"(v[(j + 3) % G])
                   : "memory");
  } else if (G % 2 == 0 && n == G && (ad & 7u) == 0) {
#pragma unroll
    for (int j = 0; j < G; j += 2)
      asm volatile("st.global.v2.s32 [%0], {%1, %2};" ::"l"(p + j), "r"(v[j]), "r"(v[(j + 1) % G])
                   : "memory");
  } else {
#pragma unroll
    for (int j = 0; j < G; ++j)
      if (j < n) p[j] = v[j];
  }
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
  __device__ __forceinline__ int k() const { return KT; }
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
  __device__ __forceinline__ int k() const { return K; }
};

template <int KT>
__device__ __forceinline__ void epilogue(const KArgs& a, const Acc<KT>& acc, long long row) {
  if (a.out == nullptr) return;
  const int K = acc.k();
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
  if (a.kind == kKindCli) {
    // Sources/MacBoostCLI/main.swift:344-364, in float32: predict (exp for
    // log-link objectives), then a softmax over classes (max-shifted, class-
    // order sum, divide) when K > 1, or 1 / (1 + exp(-x)) for the binary
    // objective.  exp is evaluated as the float32 rounding of the float64 exp.
    float v[KT == 0 ? 128 : KT];
    for (int c = 0; c < K; ++c) {
      v[c] = acc.get(c);
      if (a.log_link) v[c] = float(exp(double(v[c])));
    }
    if (K > 1) {
      float mx = -__int_as_float(0x7f800000);
      for (int c = 0; c < K; ++c) mx = v[c] > mx ? v[c] : mx;
      float sum = 0.0f;
      for (int c = 0; c < K; ++c) {
        v[c] = float(exp(double(v[c] - mx)));
        sum += v[c];
      }
      for (int c = 0; c < K; ++c) o[row * K + c] = v[c] / sum;
    } else if (a.binary) {
      o[row] = 1.0f / (1.0f + float(exp(double(-v[0]))));
    } else {
      o[row] = v[0];
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

// Barrier and phase of the j-th row-tile copy a CTA (or warp) issues: copies
// alternate between two buffers, each with its own barrier, or reuse one.
__device__ __forceinline__ uint32_t copy_bar(uint32_t bar0, int bufs, int j) {
  return bufs == 2 ? bar0 + 8u * uint32_t(j & 1) : bar0;
}
__device__ __forceinline__ uint32_t copy_parity(int bufs, int j) {
  return bufs == 2 ? uint32_t((j >> 1) & 1) : uint32_t(j & 1);
}

// The abort path's last step: before a CTA (or warp) that gave up returns,
// one thread waits, bounded, for every bulk copy it issued and did not
// consume -- the one that timed out included -- so that no copy can still be
// writing this CTA's shared memory once it has exited.  Forest block copy i
// completes phase (i >> 1) & 1 of barrier bar_f0 + 8 (i & 1); row-tile copies
// as copy_bar / copy_parity.  The status word already holds the timeout.
static __device__ __noinline__ void drain_copies(const KArgs& a, uint32_t bar_f0, unsigned f_cons,
                                             unsigned f_issued, uint32_t bar_t0, int bufs,
                                             int t_cons, int t_issued) {
  for (unsigned i = f_cons; i < f_issued; ++i)
    mbar_wait(bar_f0 + 8u * (i & 1u), (i >> 1) & 1u, a.err, a.wait_ns);
  for (int j = t_cons; j < t_issued; ++j)
    mbar_wait(copy_bar(bar_t0, bufs, j), copy_parity(bufs, j), a.err, a.wait_ns);
}

// The tile order of a CTA-wide persistent loop.  Tile 0 of CTA b is b and
// tile 1 is b + gridDim.x; with the launch's counter pair (KArgs::sched) the
// later ones are claimed in row order, one tile ahead -- thread 0 claims tile
// k + 2 during iteration k into shared slot k & 1, which the CTA reads after
// a barrier that ends iteration k -- so CTAs on faster SMs take more tiles;
// without counters the order is fixed (tile + k * gridDim.x).  Thread 0 of
// every CTA counts the CTA out of `done` as it leaves (after its claims,
// __threadfence), and the last CTA out sets both counters back to zero.
struct TileOrder {
  const KArgs& a;
  uint32_t slots;  // two 8-byte shared-memory slots
  __device__ __forceinline__ void claim_ahead(int k) const {
    if (a.sched != nullptr && threadIdx.x == 0) {
      const unsigned long long v =
          2ull * gridDim.x + atomicAdd(a.sched, 1ull);
      asm volatile("st.shared.u64 [%0], %1;" ::"r"(slots + 8u * uint32_t(k & 1)), "l"(v)
                   : "memory");
    }
  }
  // Tile after `next`, read after the barrier that ends iteration k.
  __device__ __forceinline__ long long after(int k, long long next) const {
    if (a.sched == nullptr) return next + gridDim.x;
    unsigned long long v;
    asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(slots + 8u * uint32_t(k & 1)) : "memory");
    return (long long)v;
  }
  __device__ __forceinline__ void leave() const {
    if (a.sched != nullptr && threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(a.sched + 1, 1ull) + 1 == (unsigned long long)gridDim.x) {
        atomicExch(a.sched, 0ull);
        atomicExch(a.sched + 1, 0ull);
      }
    }
  }
};

// The per-CTA pipeline shared by both layouts: a persistent loop over row
// tiles (double- or single-buffered bulk staging), forest blocks (resident,
// or streamed through two buffers), the -Inf plane fill, and the bounded-wait
// abort protocol.  `score(fb, b, row, rowbase, acc)` walks every tree of the
// forest block at shared address fb for this thread's row.
template <int KT, bool CHECK_NAN = false, class ScoreBlock>
__device__ __forceinline__ void run_tiles(const KArgs& a, unsigned char* smem, ScoreBlock score) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t base = smem_u32(smem);
  const uint32_t bar_tile0 = base, bar_f0 = base + 16;
  const uint32_t tiles = base + uint32_t(kSmemHeader);
  const uint32_t fbuf = tiles + uint32_t(a.tile_bufs) * a.tile_bytes;
  const bool streaming = a.nblocks > 1;
  const bool bulk = a.bulk && a.S_stage > 0;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(base + 8u * i, 1);
    fence_mbar_init();
  }
  if (a.neg_inf_slot != 0xFFFFFFFFu) {
    // constant -Inf slot read by explicit-layout leaf records; no copy writes it
    for (int b = 0; b < a.tile_bufs; ++b)
      sts_f32(tiles + uint32_t(b) * a.tile_bytes + a.neg_inf_slot + uint32_t(tid) * 4u,
              -__int_as_float(0x7f800000));
  }
  __syncthreads();

  const TileOrder order{a, base + 64u};
  long long tile = blockIdx.x;
  if (tile >= a.ntiles) {  // uniform over the CTA
    order.leave();
    return;
  }
  long long next = tile + gridDim.x;

  if (warp == 0) {
    if (a.nblocks > 0) issue_block(a, 0, fbuf, bar_f0, lane);
    if (bulk) issue_tile(a, tile, tiles, bar_tile0, lane);
  }
  // Forest blocks consumed by this CTA (resident forest: 1 once it has
  // landed).  Copies in flight, for the abort path, follow from the loop
  // state: tile copy k is this CTA's k-th tile; tile k + 1 is in flight during
  // iteration k when it is double-buffered; block fseq of the forest is in
  // flight until consumed, and block fseq + 1 once prefetched.
  unsigned fseq = 0;
  const unsigned f_any = a.nblocks > 0 ? 1u : 0u;

  for (int k = 0; tile < a.ntiles; ++k) {
    const int tb = (a.tile_bufs == 2) ? (k & 1) : 0;
    const uint32_t tl = tiles + uint32_t(tb) * a.tile_bytes;
    order.claim_ahead(k);
    const bool ahead = bulk && a.tile_bufs == 2 && next < a.ntiles;
    if (ahead && warp == 0) {
      // buffer tb^1 held tile k-1, released by the barrier ending that iteration
      if (lane == 0) fence_proxy_async();
      __syncwarp();
      issue_tile(a, next, tiles + uint32_t(tb ^ 1) * a.tile_bytes, bar_tile0 + 8u * (tb ^ 1),
                 lane);
    }
    const int t_issued = k + (ahead ? 2 : 1);
    if (bulk) {
      const bool ok = mbar_wait(copy_bar(bar_tile0, a.tile_bufs, k),
                                copy_parity(a.tile_bufs, k), a.err, a.wait_ns);
      if (__syncthreads_or(!ok)) {
        if (tid == 0)
          drain_copies(a, bar_f0, fseq, streaming ? fseq + 1 : f_any, bar_tile0, a.tile_bufs, k,
                       t_issued);
        order.leave();
        return;
      }
    } else if (a.S_stage > 0) {
      load_tile_sync(a, tile, tl);
      __syncthreads();
    }

    const long long row = tile * a.R + tid;
    const uint32_t rowbase = tl + uint32_t(tid) * 4u;
    fill_left_planes(a, rowbase);  // own row only: no barrier needed
    // CHECK_NAN: the CTA scans the staged tile (16-byte loads) once; a tile
    // without NaN lets the walk drop the default-direction test.  Rows past
    // the end of the input hold stale values, which can only clear `clean`.
    bool clean = false;
    if (CHECK_NAN) {
      const uint32_t n4 = uint32_t(a.S_stage) * uint32_t(a.R) / 4u;
      bool nan = false;
      for (uint32_t i = uint32_t(tid); i < n4; i += blockDim.x) {
        const float4 q = lds_v4f(tl + 16u * i);
        nan = nan || isnan(q.x) || isnan(q.y) || isnan(q.z) || isnan(q.w);
      }
      clean = !__syncthreads_or(nan);
    }
    // own row only, after the scan above has read every row: the codes may
    // replace values in place
    fill_codes(a, rowbase);
    Acc<KT> acc;
    acc.init(a.base, a.K);
    for (int b = 0; b < a.nblocks; ++b) {
      uint32_t fb;
      if (streaming) {
        // release the buffer of block fseq-1, then prefetch block fseq+1 into it
        __syncthreads();
        int nb = b + 1;
        if (nb == a.nblocks) nb = (next < a.ntiles) ? 0 : -1;
        if (nb >= 0 && warp == 0) {
          if (lane == 0) fence_proxy_async();
          __syncwarp();
          issue_block(a, nb, fbuf + ((fseq + 1) & 1) * a.buf_bytes,
                      bar_f0 + 8u * ((fseq + 1) & 1), lane);
        }
        const bool ok = mbar_wait(bar_f0 + 8u * (fseq & 1), (fseq >> 1) & 1, a.err, a.wait_ns);
        if (__syncthreads_or(!ok)) {
          if (tid == 0)
            drain_copies(a, bar_f0, fseq, fseq + (nb >= 0 ? 2u : 1u), bar_tile0, a.tile_bufs,
                         k + 1, t_issued);
          order.leave();
          return;
        }
        fb = fbuf + (fseq & 1) * a.buf_bytes;
        ++fseq;
      } else {
        if (k == 0) {
          const bool ok = mbar_wait(bar_f0, 0, a.err, a.wait_ns);
          if (__syncthreads_or(!ok)) {
            if (tid == 0) drain_copies(a, bar_f0, 0, 1, bar_tile0, a.tile_bufs, k + 1, t_issued);
            order.leave();
            return;
          }
          fseq = 1;
        }
        fb = fbuf;
      }
      score(fb, b, row, rowbase, acc, clean);
    }
    if (row < a.rows) epilogue<KT>(a, acc, row);
    __syncthreads();  // every thread is done with tile buffer tb
    if (bulk && a.tile_bufs == 1 && next < a.ntiles && warp == 0) {
      if (lane == 0) fence_proxy_async();
      __syncwarp();
      issue_tile(a, next, tiles, bar_tile0, lane);
    }
    tile = next;
    next = order.after(k, next);  // claimed this iteration, before the barrier above
  }
  order.leave();
}

// The per-warp pipeline, for a forest resident in shared memory (one block):
// each warp stages and scores its own chunks of 32 rows, independently of the
// other warps of the CTA.  Chunk c covers rows [32c, 32c + 32); warp w of CTA
// b starts with chunk w * gridDim.x + b and claims its next chunks from the
// launch's counters in row order (claim below), so the chunks in flight at
// any time form one contiguous run of rows and the work evens out across SMs
// and warps however fast each runs.  A
// chunk lands, one bulk copy of 128 bytes per staged slot, in the warp's 32
// columns of the row-tile layout (slot s, row j of the warp at
// tile + 4 * (s * R + 32 w + j)), on the warp's own mbarrier.  With two tile
// buffers the next chunk is in flight while the current one is scored; with
// one, the next copy is issued when the warp is done, and the other warps keep
// the SM busy meanwhile.  No CTA-wide barrier follows the forest wait, and a
// chunk's NaN test is a warp vote.  A warp that gives up waiting drains its own
// copies (drain_copies) and returns; the other warps go on with theirs.
template <int KT, bool CHECK_NAN = false, class ScoreBlock>
__device__ __forceinline__ void run_warps(const KArgs& a, unsigned char* smem, ScoreBlock score) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int W = int(blockDim.x >> 5);
  const uint32_t base = smem_u32(smem);
  const uint32_t bar_f0 = base + 16;
  const uint32_t bar_w = base + 128u + 16u * uint32_t(warp);  // buffers 0 and 1
  const uint32_t tiles = base + uint32_t(kSmemHeader);
  const uint32_t fbuf = tiles + uint32_t(a.tile_bufs) * a.tile_bytes;
  const bool bulk = a.bulk && a.S_stage > 0;
  const long long nchunks = (a.rows + 31) / 32;
  const long long stride = (long long)gridDim.x * W;
  long long c = (long long)warp * gridDim.x + blockIdx.x;

  if (tid == 0) {
    mbar_init(bar_f0, 1);
    fence_mbar_init();
  }
  if (lane == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_w + 8u, 1);
    fence_mbar_init();
  }
  if (a.neg_inf_slot != 0xFFFFFFFFu) {
    for (int b = 0; b < a.tile_bufs; ++b)
      sts_f32(tiles + uint32_t(b) * a.tile_bytes + a.neg_inf_slot + uint32_t(tid) * 4u,
              -__int_as_float(0x7f800000));
  }
  __syncthreads();
  // Chunks after a warp's first: claimed from the launch's counter pair when
  // there is one (warps that finish early take more chunks, so every SM and
  // every warp ends within about one chunk of the others, whatever the SMs'
  // speeds), else the fixed order c + k * stride.  Claims return stride +
  // next++; a warp stops at its first claim past the last chunk.  Every warp
  // counts itself out in `done` as it leaves (the claims it made come first,
  // __threadfence), and the last one out of the grid sets both counters back
  // to zero for the next launch on its stream.
  auto claim = [&](long long cur) -> long long {
    if (a.sched == nullptr) return cur + stride;
    unsigned long long v = 0;
    if (lane == 0) v = atomicAdd(a.sched, 1ull);
    return stride + (long long)__shfl_sync(0xffffffffu, v, 0);
  };
  auto leave = [&]() {
    if (a.sched != nullptr && lane == 0) {
      __threadfence();
      const unsigned long long n = atomicAdd(a.sched + 1, 1ull);
      if (n + 1 == (unsigned long long)gridDim.x * (unsigned long long)W) {
        atomicExch(a.sched, 0ull);
        atomicExch(a.sched + 1, 0ull);
      }
    }
  };
  // Warp 0 holds the CTA's lowest chunk (b): when it has none, no warp of the
  // CTA has one and nothing was issued; when it has one, it stages the forest,
  // which every warp that gets past here can then wait for.
  if (c >= nchunks) {
    leave();
    return;
  }
  if (warp == 0) issue_block(a, 0, fbuf, bar_f0, lane);

  auto issue = [&](long long cc, int buf) {
    const long long r0 = cc * 32;
    long long nv = a.rows - r0;
    if (nv > 32) nv = 32;
    const uint32_t nbytes = uint32_t(((nv + 3) & ~3ll) * 4);
    const uint32_t bar = bar_w + 8u * uint32_t(buf);
    if (lane == 0) mbar_arrive_expect_tx(bar, nbytes * uint32_t(a.S_stage));
    __syncwarp();
    if (a.stall_tiles) return;  // test hook: the bytes never come
    const uint32_t dst = tiles + uint32_t(buf) * a.tile_bytes + uint32_t(warp) * 128u;
    for (int s = lane; s < a.S_stage; s += 32) {
      const long long f = a.stage_feature ? __ldg(a.stage_feature + s) : s;
      bulk_g2s(dst + uint32_t(s) * uint32_t(a.R) * 4u, a.x + f * a.ld + r0, nbytes, bar);
    }
  };
  // Before a copy overwrites a buffer this warp has read or written.
  auto release = [&]() {
    __syncwarp();
    fence_proxy_async();
    __syncwarp();
  };

  // Chunk copy k is this warp's k-th chunk; during iteration k, copy k + 1 is
  // in flight when it was issued ahead (two buffers).
  if (bulk) issue(c, 0);
  bool forest_ready = false;
  long long cn = 0;
  for (int k = 0; c < nchunks; c = cn, ++k) {
    const int buf = (a.tile_bufs == 2) ? (k & 1) : 0;
    cn = claim(c);  // its latency overlaps this chunk's walk
    const bool ahead = bulk && a.tile_bufs == 2 && cn < nchunks;
    if (ahead) {
      release();  // buffer buf^1 held chunk k-1
      issue(cn, buf ^ 1);
    }
    const int k_issued = k + (ahead ? 2 : 1);
    const uint32_t rowbase = tiles + uint32_t(buf) * a.tile_bytes + uint32_t(tid) * 4u;
    const long long row = c * 32 + lane;
    if (bulk) {
      const bool ok = mbar_wait(copy_bar(bar_w, a.tile_bufs, k), copy_parity(a.tile_bufs, k),
                                a.err, a.wait_ns);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) drain_copies(a, bar_f0, forest_ready ? 1u : 0u, 1u, bar_w, a.tile_bufs, k, k_issued);
        __syncwarp();
        leave();
        return;
      }
    } else {
      for (int s = 0; s < a.S_stage; ++s) {
        const long long f = a.stage_feature ? __ldg(a.stage_feature + s) : s;
        sts_f32(rowbase + uint32_t(s) * uint32_t(a.R) * 4u,
                row < a.rows ? __ldg(a.x + f * a.ld + row) : 0.0f);
      }
      __syncwarp();
    }
    if (!forest_ready) {
      const bool ok = mbar_wait(bar_f0, 0, a.err, a.wait_ns);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0) drain_copies(a, bar_f0, 0u, 1u, bar_w, a.tile_bufs, k + 1, k_issued);
        __syncwarp();
        leave();
        return;
      }
      forest_ready = true;
    }
    fill_left_planes_warp(a, tiles + uint32_t(buf) * a.tile_bytes + uint32_t(warp) * 128u, lane);
    fill_codes_warp(a, tiles + uint32_t(buf) * a.tile_bytes + uint32_t(warp) * 128u, lane);
    // CHECK_NAN: the warp scans its 32 rows of every staged slot (16-byte
    // loads, 8 lanes per slot); rows past the end of the input hold stale
    // values, which can only clear `clean`.
    bool clean = false;
    if (CHECK_NAN) {
      const uint32_t slice = tiles + uint32_t(buf) * a.tile_bytes + uint32_t(warp) * 128u;
      bool nan = false;
      for (int i = lane; i < a.S_stage * 8; i += 32) {
        const float4 q = lds_v4f(slice + uint32_t(i >> 3) * uint32_t(a.R) * 4u +
                                 uint32_t(i & 7) * 16u);
        nan = nan || isnan(q.x) || isnan(q.y) || isnan(q.z) || isnan(q.w);
      }
      clean = !__any_sync(0xffffffffu, nan);
    }
    Acc<KT> acc;
    acc.init(a.base, a.K);
    score(fbuf, 0, row, rowbase, acc, clean);
    if (row < a.rows) epilogue<KT>(a, acc, row);
    if (bulk && a.tile_bufs == 1 && cn < nchunks) {
      release();
      issue(cn, 0);
    }
  }
  leave();
}

// The pipeline for the forest block layout: per-warp chunks when the forest
// is resident, else CTA-wide tiles with streamed tree blocks.
template <int KT, bool CHECK_NAN = false, class ScoreBlock>
__device__ __forceinline__ void run_rows(const KArgs& a, unsigned char* smem, ScoreBlock score) {
  if (a.nblocks == 1)
    run_warps<KT, CHECK_NAN>(a, smem, score);
  else
    run_tiles<KT, CHECK_NAN>(a, smem, score);
}

}  // namespace dev

// Per-layout launchers (kernels_complete.cu, kernels_explicit.cu, kernels_codes.cu).
cudaError_t launch_codes(int code_bytes, bool cat, const KArgs& a, size_t smem, int grid,
                         cudaStream_t stream, int* occupancy_out);
cudaError_t launch_complete_top(bool planes, bool cat, bool pay, const KArgs& a,
                                const TopRecords& top, size_t smem, int grid,
                                cudaStream_t stream, int* occupancy_out);
cudaError_t launch_complete(bool planes, bool cat, bool pay, const KArgs& a, size_t smem,
                            int grid, cudaStream_t stream, int* occupancy_out);
cudaError_t launch_explicit(bool planes, bool cat, const KArgs& a, size_t smem, int grid,
                            cudaStream_t stream, int* occupancy_out);

}  // namespace mb
