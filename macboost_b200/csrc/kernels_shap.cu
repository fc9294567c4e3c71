// sm_100a TreeSHAP contributions kernel (path-dependent TreeSHAP, float64).
//
// Replaces the gpu_treeshap Metal kernel (Sources/MacBoost/Shaders.swift:
// 1635-1734) and the recursive CPU TreeSHAP (SHAP.swift:170-326).
//
// A leaf's share of the Shapley values depends only on its root-to-leaf path.
// After merging repeated features, a path has U distinct features, each with
// a cover fraction z_i (row-independent) and an indicator o_i in {0, 1}
// (whether the row satisfies all of that feature's splits on the path).  With
// On = {i : o_i = 1}, m = |On|, c_U(s) = s!(U-1-s)!/U! and e_d(Z) the
// elementary symmetric polynomials of the z's in a set Z, the leaf (value v)
// adds to feature j
//   j in On :  v (1 - z_j) P_off sum_s c_U(s) e_{m-1-s}(On \ {j})
//   j not On: -v P_off sum_s c_U(s) e_{m-s}(On)            (the same for all j not On)
// where P_off is the product of the z's outside On.  This is the permutation
// weighting that TreeSHAP's EXTEND / UNWIND recurrences compute, evaluated
// from the polynomial prod_{i in On} (1 + z_i t): O(U^2) fused multiply-adds,
// no divisions, branch-free over the row-dependent On set.
//
// Mapping: one thread per row; a CTA holds a tile of R rows and walks the
// class's paths block by block.  Each block of path records (at most
// kShapBlockPaths paths and kShapBlockUniq feature records, contiguous in
// global memory) is staged into shared memory by one bulk copy pair, double
// buffered on two mbarriers, so every warp reads the records it needs from
// shared memory.  All threads walk the same paths in the same order, so a
// row's contributions are summed in a fixed order and runs repeat bit for
// bit.  Row values are read from the feature-major input (L1-resident for
// the tile); the per-row float64 accumulators live in shared memory
// (accumulator of slot s, row r at s * R + r: a warp touches 32 consecutive
// doubles), or, for models with too many features, in a global scratch
// region per CTA.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "kernels_common.cuh"
#include "shap.h"

namespace mb {
namespace {

constexpr uint32_t kStagePathBytes = uint32_t(kShapBlockPaths) * sizeof(ShapPathRec);
constexpr uint32_t kStageBytes = kStagePathBytes + uint32_t(kShapBlockUniq) * sizeof(ShapUniqueRec);
constexpr uint32_t kHeaderBytes = 128;  // two mbarriers, padded
static_assert(kStagePathBytes % 16 == 0 && kStageBytes % 16 == 0, "bulk copies move 16-byte units");

template <int MAXU>
struct ShapLayout {
  static constexpr int kRow = 2 * MAXU + 1;   // weights c_U(s), s in [-MAXU, MAXU]
  static constexpr int kCoef = (MAXU + 1) * kRow;
  static constexpr uint32_t kCoefBytes = uint32_t(kCoef) * 8u;
  // bulk-copy destinations must be 16-byte aligned: round up to 128
  static constexpr uint32_t kStage0 = (kHeaderBytes + kCoefBytes + 127u) & ~127u;
  static constexpr uint32_t kPhi = kStage0 + 2u * kStageBytes;
};

__device__ __forceinline__ int shap_cat_code(float v, int data_bins) {
  // categorical code: Booster.swift:2052-2058 / _pyinfer.py:80-86
  if (!isfinite(v)) return data_bins;
  const float r = rintf(v);
  return (r >= 0.0f && r < float(data_bins)) ? int(r) : data_bins;
}

// One thread: stage block b (path records, then its feature records).
__device__ __forceinline__ void issue_paths(const ShapArgs& a, unsigned b, uint32_t dst,
                                            uint32_t bar) {
  const unsigned p0 = __ldg(a.block_path + b), p1 = __ldg(a.block_path + b + 1);
  const unsigned u0 = __ldg(a.block_uniq + b), u1 = __ldg(a.block_uniq + b + 1);
  const uint32_t pb = (p1 - p0) * uint32_t(sizeof(ShapPathRec));
  const uint32_t ub = (u1 - u0) * uint32_t(sizeof(ShapUniqueRec));
  dev::mbar_arrive_expect_tx(bar, pb + ub);
  dev::bulk_g2s(dst, static_cast<const ShapPathRec*>(a.paths) + p0, pb, bar);
  dev::bulk_g2s(dst + kStagePathBytes, static_cast<const ShapUniqueRec*>(a.uniq) + u0, ub, bar);
}

// Row-side inputs of one path evaluation.
struct PathCtx {
  const ShapArgs* a;
  const double* coef_row;  // c_U(s) for this U, indexable by s in [-U, U]
  double* phi;             // this row's accumulators: slot s at phi[s * R]
  long long row;
  int R;
};

// One row, one path of exactly U distinct features: straight-line code, so
// the U deflation chains interleave.
template <int U>
__device__ __forceinline__ void path_fixed(const PathCtx& c, const ShapUniqueRec* uq, double v) {
  const ShapArgs& a = *c.a;
  float xs[U];
  double zr[U];
  unsigned slots[U];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    slots[j] = uq[j].slot;
    zr[j] = uq[j].z;
    xs[j] = __ldg(a.x + (a.slot_map ? __ldg(a.slot_map + slots[j]) : int(slots[j])) * a.ld + c.row);
  }
  double E[U + 1];
  E[0] = 1.0;
#pragma unroll
  for (int i = 1; i <= U; ++i) E[i] = 0.0;
  double poff = 1.0;
  unsigned on = 0;
  int m = 0;
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const float xv = xs[j];
    const unsigned fl = uq[j].flags;
    bool pass = isnan(xv) ? (fl & kShapNanOk) != 0 : (!(xv <= uq[j].lo) && xv <= uq[j].hi);
    if (fl & kShapHasCat) {
      const int cc = shap_cat_code(xv, a.data_bins);
      pass = pass && ((__ldg(a.masks + size_t(uq[j].mask) * 8 + (cc >> 5)) >> (cc & 31)) & 1u);
    }
    const double zo = pass ? zr[j] : 0.0;
    poff *= pass ? 1.0 : zr[j];
    on |= unsigned(pass) << j;
    m += int(pass);
#pragma unroll
    for (int s = j + 1; s >= 1; --s) E[s] = fma(zo, E[s - 1], E[s]);
  }
  double w[U + 1];  // w[i] = c_U(m - i)
#pragma unroll
  for (int i = 0; i <= U; ++i) w[i] = c.coef_row[m - i];
  double goff = 0.0;
#pragma unroll
  for (int i = 0; i <= U; ++i) goff = fma(E[i], w[i], goff);
  double ep[U], g[U];
#pragma unroll
  for (int j = 0; j < U; ++j) {
    ep[j] = 1.0;
    g[j] = w[1 < U + 1 ? 1 : 0];
  }
#pragma unroll
  for (int i = 1; i < U; ++i)
#pragma unroll
    for (int j = 0; j < U; ++j) {
      ep[j] = fma(-zr[j], ep[j], E[i]);
      g[j] = fma(ep[j], w[i + 1], g[j]);
    }
  const double off_c = -v * goff * poff;
  const double on_scale = v * poff;
#pragma unroll
  for (int j = 0; j < U; ++j) {
    const double cj = ((on >> j) & 1u) ? on_scale * (1.0 - zr[j]) * g[j] : off_c;
    c.phi[size_t(slots[j]) * c.R] += cj;
  }
}

// MAXT, MINB: launch bounds.  The dense build (128 threads, 4 CTAs per SM)
// caps registers at 128 so that four 128-row CTAs fit an SM when the
// accumulators live in global memory.
template <int MAXU, bool SMEM, int MAXT = 256, int MINB = 1>
__global__ void __launch_bounds__(MAXT, MINB) shap_kernel(const ShapArgs a) {
  using L = ShapLayout<MAXU>;
  extern __shared__ __align__(128) unsigned char smem[];
  const int R = a.R;
  const int tid = threadIdx.x;
  const int S = a.S;
  const uint32_t sbase = dev::smem_u32(smem);
  const uint32_t bar0 = sbase;  // buffer i's mbarrier at bar0 + 8 i
  double* coef = reinterpret_cast<double*>(smem + kHeaderBytes);
  double* phi = SMEM ? reinterpret_cast<double*>(smem + L::kPhi)
                     : a.scratch + size_t(blockIdx.x) * size_t(S) * R;
  for (int i = tid; i < L::kCoef; i += blockDim.x) {
    const int U = i / L::kRow, s = i - U * L::kRow - MAXU;
    coef[i] = a.coef[U * kShapCoefRow + kShapMaxUnique + s];
  }
  if (tid == 0) {
    dev::mbar_init(bar0, 1);
    dev::mbar_init(bar0 + 8, 1);
    dev::fence_mbar_init();
  }
  __syncthreads();
  uint32_t uses = 0;  // bit i: parity of buffer i's next completion
  const int W = a.F + 1;

  for (long long tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
    const long long r0 = tile * R;
    const int nr = int(a.rows - r0 < R ? a.rows - r0 : R);
    const long long row = r0 + tid;
    for (int k = 0; k < a.K; ++k) {
      for (int s = 0; s < S; ++s) phi[size_t(s) * R + tid] = 0.0;
      const unsigned b0 = __ldg(a.class_block + k), b1 = __ldg(a.class_block + k + 1);
      if (tid == 0 && b0 < b1) issue_paths(a, b0, sbase + L::kStage0, bar0);
      for (unsigned b = b0; b < b1; ++b) {
        const uint32_t buf = (b - b0) & 1u;
        const bool ok = dev::mbar_wait(bar0 + 8u * buf, (uses >> buf) & 1u, a.err);
        uses ^= 1u << buf;
        // every thread is done with block b - 1, whose buffer block b + 1 reuses
        if (__syncthreads_or(!ok)) return;
        if (tid == 0 && b + 1 < b1)
          issue_paths(a, b + 1, sbase + L::kStage0 + (buf ^ 1u) * kStageBytes, bar0 + 8u * (buf ^ 1u));
        if (tid >= nr) continue;
        const unsigned char* stage = smem + L::kStage0 + buf * kStageBytes;
        const ShapPathRec* sp = reinterpret_cast<const ShapPathRec*>(stage);
        const ShapUniqueRec* su = reinterpret_cast<const ShapUniqueRec*>(stage + kStagePathBytes);
        const unsigned p0 = __ldg(a.block_path + b), np = __ldg(a.block_path + b + 1) - p0;
        const unsigned u0 = __ldg(a.block_uniq + b);
        for (unsigned lp = 0; lp < np; ++lp) {
          const ShapUniqueRec* uq = su + (sp[lp].first - u0);
          const int U = int(sp[lp].U);
          const double v = sp[lp].leaf;
          if (MAXU == 12) {
            const PathCtx pc{&a, coef + U * L::kRow + MAXU, phi + tid, row, R};
            switch (U) {
              case 1: path_fixed<1>(pc, uq, v); break;
              case 2: path_fixed<2>(pc, uq, v); break;
              case 3: path_fixed<3>(pc, uq, v); break;
              case 4: path_fixed<4>(pc, uq, v); break;
              case 5: path_fixed<5>(pc, uq, v); break;
              case 6: path_fixed<6>(pc, uq, v); break;
              case 7: path_fixed<7>(pc, uq, v); break;
              case 8: path_fixed<8>(pc, uq, v); break;
              case 9: path_fixed<9>(pc, uq, v); break;
              case 10: path_fixed<10>(pc, uq, v); break;
              case 11: path_fixed<11>(pc, uq, v); break;
              default: path_fixed<12>(pc, uq, v); break;
            }
            continue;
          }
          // longer paths: the same arithmetic over a run-time U
          // the path's records and row values into registers (independent loads)
          float xs[MAXU];
          double zr[MAXU];
          unsigned slots[MAXU];
#pragma unroll
          for (int j = 0; j < MAXU; ++j) {
            if (j < U) {
              slots[j] = uq[j].slot;
              zr[j] = uq[j].z;
              xs[j] = __ldg(a.x + (a.slot_map ? __ldg(a.slot_map + slots[j]) : int(slots[j])) * a.ld +
                            row);
            }
          }
          double E[MAXU + 1];
          E[0] = 1.0;
#pragma unroll
          for (int i = 1; i <= MAXU; ++i) E[i] = 0.0;
          double poff = 1.0;
          unsigned on = 0;
          int m = 0;
#pragma unroll
          for (int j = 0; j < MAXU; ++j) {
            if (j >= U) break;
            const float xv = xs[j];
            const unsigned fl = uq[j].flags;
            bool pass = isnan(xv) ? (fl & kShapNanOk) != 0 : (!(xv <= uq[j].lo) && xv <= uq[j].hi);
            if (fl & kShapHasCat) {
              const int c = shap_cat_code(xv, a.data_bins);
              pass = pass && ((__ldg(a.masks + size_t(uq[j].mask) * 8 + (c >> 5)) >> (c & 31)) & 1u);
            }
            // E(t) <- E(t) * (1 + z t) when the row passes (at most j + 1
            // factors so far), else P_off <- P_off * z
            const double zo = pass ? zr[j] : 0.0;
            poff *= pass ? 1.0 : zr[j];
            on |= unsigned(pass) << j;
            m += int(pass);
#pragma unroll
            for (int s = j + 1; s >= 1; --s) E[s] = fma(zo, E[s - 1], E[s]);
          }
          // weights w[i] = c_U(m - i), i = 0..U (zero outside 0 <= m - i < U)
          const double* cU = coef + U * L::kRow + MAXU + m;
          double w[MAXU + 1];
#pragma unroll
          for (int i = 0; i <= MAXU; ++i)
            if (i <= U) w[i] = cU[-i];
          double goff = 0.0;
#pragma unroll
          for (int i = 0; i <= MAXU; ++i) {
            if (i > U) break;
            goff = fma(E[i], w[i], goff);
          }
          const double off_c = -v * goff * poff;
          const double on_scale = v * poff;
#pragma unroll
          for (int j = 0; j < MAXU; ++j) {
            if (j >= U) break;
            double c = off_c;
            if ((on >> j) & 1u) {
              // E(t) / (1 + z_j t), term by term, dotted with c_U(m - 1 - i)
              const double z = zr[j];
              double ep = 1.0;
              double g = w[1];
#pragma unroll
              for (int i = 1; i < MAXU; ++i) {
                if (i >= U) break;
                ep = fma(-z, ep, E[i]);
                g = fma(ep, w[i + 1], g);
              }
              c = on_scale * (1.0 - z) * g;
            }
            phi[size_t(slots[j]) * R + tid] += c;
          }
        }
      }
      __syncthreads();
      // rows x K x (F + 1): class k's block of this tile, written row by row
      float* ob = a.out + (r0 * a.K + k) * W;
      for (int i = tid; i < nr * W; i += blockDim.x) {
        const int r = i / W, f = i - r * W;
        float val;
        if (f == a.F) {
          val = a.bias[k];
        } else {
          const int s = a.feature_slot[f];
          val = s >= 0 ? float(phi[size_t(s) * R + r]) : 0.0f;
        }
        ob[size_t(r) * a.K * W + f] = val;
      }
      __syncthreads();
    }
  }
}

using ShapKernel = void (*)(const ShapArgs);

ShapKernel pick(int maxu, bool smem_variant, bool dense) {
  if (dense && maxu <= 12 && !smem_variant) return shap_kernel<12, false, 128, 4>;
  if (maxu <= 12) return smem_variant ? shap_kernel<12, true> : shap_kernel<12, false>;
  return smem_variant ? shap_kernel<kShapMaxUnique, true> : shap_kernel<kShapMaxUnique, false>;
}

}  // namespace

size_t shap_smem_bytes(int maxu, bool smem_variant, int S, int R) {
  const size_t fixed = maxu <= 12 ? ShapLayout<12>::kPhi : ShapLayout<kShapMaxUnique>::kPhi;
  return fixed + (smem_variant ? size_t(S) * R * 8 : 0);
}

cudaError_t shap_occupancy(int maxu, bool smem_variant, int R, size_t smem, int* ctas,
                           bool dense) {
  ShapKernel k = pick(maxu, smem_variant, dense);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, k, R, smem);
}

cudaError_t launch_shap(const ShapArgs& a, int maxu, bool smem_variant, size_t smem, int grid,
                        cudaStream_t stream, bool dense) {
  if (a.rows <= 0) return cudaSuccess;
  ShapKernel k = pick(maxu, smem_variant, dense);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  k<<<grid, a.R, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mb
