// sm_100a forest kernel for the binned-code layout (complete trees).
//
// Same semantics as the f32 kernels (bit-exact margins, tree-order fp32
// accumulation; see kernels_complete.cu).  Per row tile:
//   1. the staged feature columns land in a raw fp32 tile by cp.async.bulk;
//   2. every thread converts its own row: for each staged value one
//      branch-free search in the feature's Eytzinger-ordered threshold table
//      (i = 2i + (t[i] < v), d steps) gives code(v) = #thresholds below v,
//      written to the NaN-right plane (NaN -> largest code), the NaN-left plane
//      (NaN -> 0) and/or the categorical plane (category code), as the
//      feature's splits require;
//   3. once all rows are converted the raw tile is free and the next tile's
//      bulk copies are issued, overlapping the walk;
//   4. each thread walks G trees at once over 4-byte records: one shared load
//      for the record, one for the code, go_right = code > J (or the
//      categorical mask bit), child o' = 2o - A + 4*go_right; the leaf value
//      sits at o + k after D levels.
// A warp's record loads for one tree level fall in one 128-byte line and its
// code loads in 32 distinct banks, so each costs one shared-memory wavefront.
// Every mbarrier wait is bounded (kernels_common.cuh).
#include "kernels_common.cuh"

namespace mb {
namespace {

constexpr uint32_t kCodeCatBit = 0x2000u;
constexpr uint32_t kCodeIndexMask = 0x1FFFu;
constexpr int kCodeOffsetShift = 14;

template <int KT, int G>
struct CodesBounds {
  static constexpr int kMaxThreads = G >= 12 ? 256 : (G >= 10 || KT == 0 || KT >= 5 ? 512 : 768);
};

template <int CW>
__device__ __forceinline__ uint32_t lds_code(uint32_t a) {
  uint32_t v;
  if (CW == 1)
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
  else
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int CW>
__device__ __forceinline__ void sts_code(uint32_t a, uint32_t v) {
  if (CW == 1)
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(a), "r"(v) : "memory");
  else
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

// Category code of a value: rint(v) when finite and in [0, dataBins), else
// dataBins, the missing bin (_pyinfer.py:80-86, Booster.swift:2052-2058).
__device__ __forceinline__ uint32_t category_code(float v, int data_bins) {
  uint32_t code = uint32_t(data_bins);
  if (isfinite(v)) {
    const float q = rintf(v);
    if (q >= 0.0f && q < float(data_bins)) code = uint32_t(q);
  }
  return code;
}

template <int CW>
__device__ __forceinline__ void store_codes(const int4& bp, float v, uint32_t code,
                                            uint32_t code_row, int data_bins) {
  constexpr uint32_t kNanRight = CW == 1 ? 0xFFu : 0xFFFFu;
  if (bp.y >= 0) sts_code<CW>(code_row + uint32_t(bp.y), isnan(v) ? kNanRight : code);
  if (bp.z >= 0) sts_code<CW>(code_row + uint32_t(bp.z), code);  // NaN searched to 0
  if (bp.w >= 0) sts_code<CW>(code_row + uint32_t(bp.w), category_code(v, data_bins));
}

// This thread's row: raw fp32 values of the staged slots -> codes.  Four
// searches run interleaved for latency hiding.
template <int CW>
__device__ __forceinline__ void bin_row(const KArgs& a, uint32_t raw_row, uint32_t code_row) {
  const int d = a.search_depth;
  const uint32_t top = 1u << d;
  const int4* plan = reinterpret_cast<const int4*>(a.bin_plan);
  const uint32_t slot_bytes = uint32_t(a.R) * 4u;
  int s = 0;
  for (; s + 4 <= a.S_stage; s += 4) {
    int4 bp[4];
    float v[4];
    uint32_t i[4];
    const float* t[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      bp[q] = __ldg(plan + s + q);
      v[q] = dev::lds_f32(raw_row + uint32_t(s + q) * slot_bytes);
      i[q] = 1u;
      t[q] = a.search + size_t(bp[q].x < 0 ? 0 : bp[q].x) * top;
    }
    for (int k = 0; k < d; ++k) {
#pragma unroll
      for (int q = 0; q < 4; ++q) i[q] = 2u * i[q] + uint32_t(__ldg(t[q] + i[q]) < v[q]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) store_codes<CW>(bp[q], v[q], i[q] - top, code_row, a.data_bins);
  }
  for (; s < a.S_stage; ++s) {
    const int4 bp = __ldg(plan + s);
    const float v = dev::lds_f32(raw_row + uint32_t(s) * slot_bytes);
    uint32_t i = 1u;
    if (bp.x >= 0) {
      const float* t = a.search + size_t(bp.x) * top;
      for (int k = 0; k < d; ++k) i = 2u * i + uint32_t(__ldg(t + i) < v);
    } else {
      i = top;
    }
    store_codes<CW>(bp, v, i - top, code_row, a.data_bins);
  }
}

template <int CW, bool CAT>
__device__ __forceinline__ uint32_t code_route(uint32_t r, uint32_t code_row,
                                               const unsigned* masks) {
  const uint32_t code = lds_code<CW>(code_row + (r >> kCodeOffsetShift));
  if (CAT && (r & kCodeCatBit)) {
    const uint32_t w = __ldg(masks + size_t(r & kCodeIndexMask) * 8 + (code >> 5));
    return ((w >> (code & 31u)) & 1u) ^ 1u;
  }
  return uint32_t(code > (r & kCodeIndexMask));
}

template <int KT, int G, int CW, bool CAT>
__global__ void __launch_bounds__(CodesBounds<KT, G>::kMaxThreads, 1)
    forest_codes_kernel(const KArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t base = dev::smem_u32(smem);
  const uint32_t bar_tile = base, bar_f0 = base + 16;
  const uint32_t raw = base + uint32_t(kSmemHeader);
  const uint32_t codes = raw + a.tile_bytes;
  const uint32_t fbuf = codes + a.code_tile_bytes;
  const bool streaming = a.nblocks > 1;
  const bool bulk = a.bulk && a.S_stage > 0;
  const int D = a.D;
  const uint32_t NL = 1u << D;
  const uint32_t NI = NL - 1;
  const uint32_t raw_row = raw + uint32_t(tid) * 4u;
  const uint32_t code_row = codes + uint32_t(tid) * 4u;

  if (tid == 0) {
    for (int i = 0; i < 4; ++i) dev::mbar_init(base + 8u * i, 1);
    dev::fence_mbar_init();
  }
  __syncthreads();
  const dev::TileOrder order{a, base + 64u};
  long long tile = blockIdx.x;
  if (tile >= a.ntiles) {  // uniform over the CTA
    order.leave();
    return;
  }
  long long next = tile + gridDim.x;
  if (warp == 0) {
    if (a.nblocks > 0) dev::issue_block(a, 0, fbuf, bar_f0, lane);
    if (bulk) dev::issue_tile(a, tile, raw, bar_tile, lane);
  }
  // Forest blocks consumed (resident forest: 1 once it has landed).  Copies
  // in flight, for the abort path, follow from the loop state: raw tile copy k
  // is this CTA's k-th tile (one buffer; tile k + 1 is issued once tile k is
  // binned), block fseq is in flight until consumed, block fseq + 1 once
  // prefetched.
  unsigned fseq = 0;
  const unsigned f_any = a.nblocks > 0 ? 1u : 0u;
  for (int k = 0; tile < a.ntiles; ++k) {
    order.claim_ahead(k);  // read after the barrier that follows the binning
    if (bulk) {
      const bool ok = dev::mbar_wait(bar_tile, uint32_t(k & 1), a.err, a.wait_ns);
      if (__syncthreads_or(!ok)) {
        if (tid == 0)
          dev::drain_copies(a, bar_f0, fseq, streaming ? fseq + 1 : f_any, bar_tile, 1, k, k + 1);
        order.leave();
        return;
      }
    } else if (a.S_stage > 0) {
      dev::load_tile_sync(a, tile, raw);
      __syncthreads();
    }
    bin_row<CW>(a, raw_row, code_row);
    __syncthreads();  // the raw tile is consumed: stage the next one during the walk
    if (bulk && next < a.ntiles && warp == 0) {
      if (lane == 0) dev::fence_proxy_async();
      __syncwarp();
      dev::issue_tile(a, next, raw, bar_tile, lane);
    }
    const int t_issued = k + ((bulk && next < a.ntiles) ? 2 : 1);
    const long long row = tile * a.R + tid;
    dev::Acc<KT> acc;
    acc.init(a.base, a.K);
    for (int b = 0; b < a.nblocks; ++b) {
      uint32_t fb;
      if (streaming) {
        __syncthreads();  // release the buffer of block fseq-1 ...
        int nb = b + 1;   // ... and prefetch block fseq+1 into it
        if (nb == a.nblocks) nb = (next < a.ntiles) ? 0 : -1;
        if (nb >= 0 && warp == 0) {
          if (lane == 0) dev::fence_proxy_async();
          __syncwarp();
          dev::issue_block(a, nb, fbuf + ((fseq + 1) & 1) * a.buf_bytes,
                           bar_f0 + 8u * ((fseq + 1) & 1), lane);
        }
        const bool ok =
            dev::mbar_wait(bar_f0 + 8u * (fseq & 1), (fseq >> 1) & 1, a.err, a.wait_ns);
        if (__syncthreads_or(!ok)) {
          if (tid == 0)
            dev::drain_copies(a, bar_f0, fseq, fseq + (nb >= 0 ? 2u : 1u), bar_tile, 1, k + 1,
                              t_issued);
          order.leave();
          return;
        }
        fb = fbuf + (fseq & 1) * a.buf_bytes;
        ++fseq;
      } else {
        if (k == 0) {
          const bool ok = dev::mbar_wait(bar_f0, 0, a.err, a.wait_ns);
          if (__syncthreads_or(!ok)) {
            if (tid == 0) dev::drain_copies(a, bar_f0, 0, 1, bar_tile, 1, k + 1, t_issued);
            order.leave();
            return;
          }
          fseq = 1;
        }
        fb = fbuf;
      }
      const int t_block = b * a.Tb;
      const uint32_t leaves = fb + a.leaf_off;
      for (int g0 = 0; g0 < a.Tb; g0 += G) {
        uint32_t A[G], o[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          A[j] = fb + uint32_t(g0 + j) * NL * 4u;
          o[j] = A[j] + 4u;  // heap node 0 in slot 1
        }
        for (int L = 0; L < D; ++L) {
          uint32_t r[G];
#pragma unroll
          for (int j = 0; j < G; ++j) r[j] = dev::lds_u32(o[j]);
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const uint32_t right = code_route<CW, CAT>(r[j], code_row, a.masks);
            o[j] = 2u * o[j] - A[j] + (right << 2);
          }
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
          // o = A + 4(n + 1) for heap node n; its leaf is n - NI
          const uint32_t kk = leaves + uint32_t(g0 + j) * NL * 4u - A[j] - 4u - 4u * NI;
          acc.add(j, t_block + g0 + j, dev::lds_f32(o[j] + kk));
        }
        if (a.out_leaf != nullptr && row < a.rows) {
          const int t0 = t_block + g0;
          int li[G];
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const uint32_t leaf = (o[j] - A[j]) / 4u - 1u - NI;
            li[j] = t0 + j < a.T ? __ldg(a.leaf_heap + size_t(t0 + j) * NL + leaf) : 0;
          }
          dev::store_leaf_run<G>(a.out_leaf + row * a.T + t0, li, a.T - t0);
        }
      }
    }
    if (row < a.rows) dev::epilogue<KT>(a, acc, row);
    tile = next;
    next = order.after(k, next);
  }
  order.leave();
}

using KernelFn = void (*)(const KArgs);

template <int KT, int G>
KernelFn pick2(int cw, bool cat) {
  if (cw == 1) return cat ? forest_codes_kernel<KT, G, 1, true> : forest_codes_kernel<KT, G, 1, false>;
  return cat ? forest_codes_kernel<KT, G, 2, true> : forest_codes_kernel<KT, G, 2, false>;
}

// (K, G) pairs must match mb::group_options (forest.cpp).
KernelFn pick(int cw, bool cat, int K, int G) {
  switch (K) {
    case 1: return G == 16 ? pick2<1, 16>(cw, cat) : pick2<1, 8>(cw, cat);
    case 2: return pick2<2, 8>(cw, cat);
    case 3: return pick2<3, 6>(cw, cat);
    case 4: return pick2<4, 8>(cw, cat);
    case 5: return pick2<5, 5>(cw, cat);
    case 6: return pick2<6, 6>(cw, cat);
    case 7: return pick2<7, 7>(cw, cat);
    case 8: return pick2<8, 8>(cw, cat);
    case 10: return pick2<10, 10>(cw, cat);
    case 12: return pick2<12, 12>(cw, cat);
    case 16: return pick2<16, 16>(cw, cat);
    default: return pick2<0, 8>(cw, cat);
  }
}

}  // namespace

cudaError_t launch_codes(int code_bytes, bool cat, const KArgs& a, size_t smem, int grid,
                         cudaStream_t stream, int* occupancy_out) {
  KernelFn fn = pick(code_bytes, cat, a.K, a.G);
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  if (occupancy_out)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occupancy_out, fn, a.R, smem);
  fn<<<grid, a.R, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb
