/*
 * mbref.c -- CPU restatement of MacBoost's reference predictor.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline.  It is loaded by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline / --impl reference legs of bench.py, and by nothing else.  The
 * product path (macboost_b200/libmacboostc.so) never links, loads or calls it,
 * and there is no CPU fallback built on it.
 *
 * What it restates (paths relative to the MacBoost source tree):
 *   Sources/MacBoost/Booster.swift:2035-2074  predictCPU (K == 1)
 *   Sources/MacBoost/Booster.swift:2076-2117  predictCPUMulticlass (K > 1)
 *   python/macboost/_pyinfer.py:52-89         PyModel.predict_raw / _goes_left_at
 *
 * Per row: out[c] = baseScores[c]; for every tree t in file order, walk the
 * implicit heap from node 0 while feature[n] >= 0:
 *   - categorical node (flags bit1, tree has a catMask): code = rint(v) when v
 *     is finite and 0 <= rint(v) < dataBins, else dataBins (the missing bin);
 *     left = bit `code` of the node's 256-bit mask (word n*8 + code/32);
 *   - NaN value: left = flags bit0 (learned default direction);
 *   - otherwise left = (v <= threshold) in fp32;
 *   n = 2n + 1 + (left ? 0 : 1);
 * then out[t % K] += leaf[n] in fp32, strictly in tree order.
 *
 * Where the two reference predictors disagree on inputs the other one cannot
 * express, this restatement follows PyModel, the reference predictor that runs
 * on Linux:
 *   - K == 1 starts from baseScores[0] (PyModel, and the Metal kernel at
 *     Shaders.swift:1553-1555); Booster.swift:2038 uses baseScore, which the
 *     reference's own save() always writes equal to baseScores[0].
 *   - a node flagged categorical in a tree whose catMask is empty routes as a
 *     numeric node (_pyinfer.py:79); Booster.swift would index an empty array.
 *   - a finite value whose rint is outside the Int range maps to the missing
 *     bin (_pyinfer.py:80-86); Booster.swift:2055 would trap on Int(r).
 * The leaf index reported for (row, tree) is the final heap index n, as in
 * Booster.swift:2065-2067 and _pyinfer.py:68-71.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MB_FLAG_DEFAULT_LEFT 1u /* Booster.swift:148 */
#define MB_FLAG_CATEGORICAL 2u  /* Booster.swift:149 */

typedef struct {
    const int64_t *tree_off; /* T+1 offsets into the node arrays */
    int32_t T;
    const int32_t *feature;
    const float *threshold;
    const float *leaf;
    const uint8_t *flags;
    const uint32_t *catmask; /* 8 words per node, valid where has_mask[t] */
    const uint8_t *has_mask; /* per tree: 1 if its catMask was non-empty */
    int32_t data_bins;       /* numBins - 1 */
    int32_t K;
    const float *base; /* K entries */
} mbref_model;

typedef struct {
    const mbref_model *m;
    const float *x;
    int64_t rows, cols, ld; /* ld: feature-major stride (>= rows) */
    int32_t layout;         /* 0 feature-major x[f*ld+i], 1 row-major x[i*cols+f] */
    float *out;             /* rows*K or NULL */
    int32_t *out_leaf;      /* rows*T or NULL */
    int64_t r0, r1;
} mbref_job;

/* Categorical code of a value: _pyinfer.py:80-86, Booster.swift:2052-2058. */
static inline int32_t mbref_cat_code(float v, int32_t data_bins) {
    if (!isfinite(v)) return data_bins;
    float r = rintf(v); /* round half to even under the default FP mode */
    if (r >= 0.0f && r < (float)data_bins) return (int32_t)r;
    return data_bins;
}

static void mbref_rows(const mbref_job *j) {
    const mbref_model *m = j->m;
    const int32_t K = m->K;
    for (int64_t i = j->r0; i < j->r1; ++i) {
        float acc[128];
        for (int32_t c = 0; c < K; ++c) acc[c] = m->base[c];
        for (int32_t t = 0; t < m->T; ++t) {
            const int64_t b = m->tree_off[t];
            int64_t n = 0;
            while (m->feature[b + n] >= 0) {
                const int64_t f = m->feature[b + n];
                const float v = j->layout == 0 ? j->x[f * j->ld + i] : j->x[i * j->cols + f];
                const uint32_t fl = m->flags[b + n];
                int left;
                if ((fl & MB_FLAG_CATEGORICAL) && m->has_mask[t]) {
                    const int32_t cat = mbref_cat_code(v, m->data_bins);
                    const uint32_t w = m->catmask[(b + n) * 8 + (cat >> 5)];
                    left = (int)((w >> (cat & 31)) & 1u);
                } else if (isnan(v)) {
                    left = (fl & MB_FLAG_DEFAULT_LEFT) != 0;
                } else {
                    left = v <= m->threshold[b + n];
                }
                n = 2 * n + 1 + (left ? 0 : 1);
            }
            /* fp32 accumulation in tree order (x86-64 SSE: no excess precision;
             * built with -ffp-contract=off and without -ffast-math) */
            if (j->out) acc[t % K] += m->leaf[b + n];
            if (j->out_leaf) j->out_leaf[i * m->T + t] = (int32_t)n;
        }
        if (j->out)
            for (int32_t c = 0; c < K; ++c) j->out[i * K + c] = acc[c];
    }
}

static void *mbref_thread(void *arg) {
    mbref_rows((const mbref_job *)arg);
    return NULL;
}

/*
 * Predict raw margins (rows*K, row-major) and/or leaf heap indices (rows*T).
 * Rows are split into contiguous chunks over `nthreads` POSIX threads, as
 * predictCPU splits them over DispatchQueue.concurrentPerform; the result does
 * not depend on the split.  Returns 0, or -1 for invalid arguments.
 */
int mbref_predict(const int64_t *tree_off, int32_t T, const int32_t *feature,
                  const float *threshold, const float *leaf, const uint8_t *flags,
                  const uint32_t *catmask, const uint8_t *has_mask, int32_t data_bins,
                  int32_t K, const float *base, const float *x, int64_t rows, int64_t cols,
                  int64_t ld, int32_t layout, float *out, int32_t *out_leaf, int32_t nthreads) {
    if (K < 1 || K > 128 || rows < 0 || cols < 0 || T < 0) return -1;
    if (layout == 0 && ld < rows) return -1;
    mbref_model m = {tree_off, T, feature, threshold, leaf, flags,
                     catmask, has_mask, data_bins, K, base};
    if (nthreads < 1) nthreads = 1;
    if (rows < (int64_t)nthreads * 64) nthreads = 1;
    mbref_job *jobs = (mbref_job *)calloc((size_t)nthreads, sizeof(mbref_job));
    pthread_t *tid = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !tid) {
        free(jobs);
        free(tid);
        return -1;
    }
    for (int32_t k = 0; k < nthreads; ++k) {
        jobs[k].m = &m;
        jobs[k].x = x;
        jobs[k].rows = rows;
        jobs[k].cols = cols;
        jobs[k].ld = ld;
        jobs[k].layout = layout;
        jobs[k].out = out;
        jobs[k].out_leaf = out_leaf;
        jobs[k].r0 = rows * k / nthreads;
        jobs[k].r1 = rows * (k + 1) / nthreads;
    }
    int32_t started = 0;
    for (int32_t k = 1; k < nthreads; ++k) {
        if (pthread_create(&tid[k], NULL, mbref_thread, &jobs[k]) != 0) break;
        started = k;
    }
    /* rows of threads that failed to start are done on the calling thread */
    mbref_rows(&jobs[0]);
    for (int32_t k = started + 1; k < nthreads; ++k) mbref_rows(&jobs[k]);
    for (int32_t k = 1; k <= started; ++k) pthread_join(tid[k], NULL);
    free(jobs);
    free(tid);
    return 0;
}
