/*
 * mbbinned.c -- CPU restatement of MacBoost's binned-data kernels.
 *
 * TEST INFRASTRUCTURE ONLY: the parity oracle for the GPU binning and
 * binned-walk kernels, loaded by tests/ (through oracle/oracle.py) and
 * nothing else.  The product library never links, loads or calls it.
 *
 * What it restates (paths relative to the MacBoost source tree):
 *   Sources/MacBoost/Shaders.swift:37-39    bin_index: tiled bin layout, 8 features
 *                                           per tile, bins[(f/8)*n*8 + i*8 + f%8]
 *   Sources/MacBoost/Shaders.swift:41-76    bin_data: NaN -> missing bin numBins-1;
 *                                           categorical -> clamp(rint(v), 0, numBins-2);
 *                                           numeric -> binary search of the feature's
 *                                           numBins-2 upper edges
 *   Sources/MacBoost/Shaders.swift:466-476  NodeSplit, goes_left on a bin
 *   Sources/MacBoost/Shaders.swift:1741-1758 assign_leaves
 *   Sources/MacBoost/Shaders.swift:1763-1781 predict_tree_binned
 * The categorical conversion of a value outside the int range saturates
 * (the Metal conversion is undefined there).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#define MB_FLAG_DEFAULT_LEFT 1u
#define MB_FLAG_CATEGORICAL 2u

static inline uint64_t bin_index(int64_t f, int64_t i, int64_t n) {
    return (uint64_t)(f >> 3) * (uint64_t)n * 8u + (uint64_t)i * 8u + (uint64_t)(f & 7);
}

/* x feature-major x[f*ld + i] (layout 0) or row-major x[i*cols + f] (1);
 * bins: ceil(cols/8)*8*rows bytes, padding features written as 0. */
int mbref_bin_data(const float *x, int64_t rows, int64_t cols, int64_t ld, int32_t layout,
                   const float *edges, int32_t num_bins, const uint8_t *categorical,
                   uint8_t *bins) {
    if (num_bins < 4 || num_bins > 256 || rows < 0 || cols < 0) return -1;
    const int64_t groups = (cols + 7) / 8;
    const uint32_t data_bins = (uint32_t)num_bins - 1;
    for (int64_t g = 0; g < groups; ++g)
        for (int64_t i = 0; i < rows; ++i)
            for (int k = 0; k < 8; ++k) {
                const int64_t f = g * 8 + k;
                uint8_t b = 0;
                if (f < cols) {
                    const float v = layout == 0 ? x[f * ld + i] : x[i * cols + f];
                    if (isnan(v)) {
                        b = (uint8_t)data_bins;
                    } else if (categorical[f] == 1) {
                        /* clamp(int(rint(v)), 0, dataBins - 1), the int conversion saturating */
                        const float r = rintf(v);
                        b = r < 0.0f ? 0 : r > (float)(data_bins - 1) ? (uint8_t)(data_bins - 1) : (uint8_t)(int)r;
                    } else {
                        const float *e = edges + (size_t)f * (data_bins - 1);
                        uint32_t lo = 0, hi = data_bins - 1;
                        while (lo < hi) {
                            const uint32_t mid = (lo + hi) >> 1;
                            if (v > e[mid]) lo = mid + 1; else hi = mid;
                        }
                        b = (uint8_t)lo;
                    }
                }
                bins[bin_index(f, i, rows)] = b;
            }
    return 0;
}

/* Walk trees t in [0, T) (nodes tree_off[t]..tree_off[t+1]) over a tiled bin
 * matrix of n rows.  preds (class-major, K x n, in/out): preds[(t%K)*n + i]
 * += leaf for each tree in order (predict_tree_binned per tree).  leaf_idx
 * (tree-major, T x n, out): the final heap index (assign_leaves).  Either
 * output may be NULL. */
int mbref_predict_binned(const uint8_t *bins, int64_t n, int32_t num_bins, int32_t T,
                         const int64_t *tree_off, const int32_t *feature, const uint32_t *sbin,
                         const uint32_t *flags, const uint32_t *catmask, const float *leaf,
                         int32_t max_depth, int32_t K, float *preds, int32_t *leaf_idx) {
    if (K < 1 || n < 0 || T < 0) return -1;
    for (int32_t t = 0; t < T; ++t) {
        const int64_t b0 = tree_off[t];
        for (int64_t i = 0; i < n; ++i) {
            uint32_t node = 0;
            for (int32_t d = 0; d < max_depth; ++d) {
                const int32_t f = feature[b0 + node];
                if (f < 0) break;
                const uint8_t b = bins[bin_index(f, i, n)];
                const uint32_t fl = flags[b0 + node];
                int left;
                if (fl & MB_FLAG_CATEGORICAL)
                    left = (catmask[(b0 + node) * 8 + b / 32] >> (b % 32)) & 1u;
                else if (b == (uint8_t)(num_bins - 1))
                    left = (fl & MB_FLAG_DEFAULT_LEFT) != 0;
                else
                    left = b <= (uint8_t)sbin[b0 + node];
                node = 2 * node + 1 + (left ? 0 : 1);
            }
            if (preds) preds[(int64_t)(t % K) * n + i] += leaf[b0 + node];
            if (leaf_idx) leaf_idx[(int64_t)t * n + i] = (int32_t)node;
        }
    }
    return 0;
}
