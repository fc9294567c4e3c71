/*
 * mbshap.c -- CPU restatement of MacBoost's TreeSHAP contributions.
 *
 * TEST INFRASTRUCTURE ONLY: the parity oracle for the GPU contributions
 * kernel, loaded by tests/ (through oracle/oracle.py) and nothing else.  The
 * product library never links, loads or calls it.
 *
 * What it restates (paths relative to the MacBoost source tree):
 *   Sources/MacBoost/SHAP.swift:170-208  predictContributionsCPU
 *   Sources/MacBoost/SHAP.swift:210-257  goesLeftRaw, shapRecurse
 *   Sources/MacBoost/SHAP.swift:259-325  extendPath, unwindPath, unwoundPathSum
 *   Sources/MacBoost/SHAP.swift:56-72    shapBias
 * i.e. the recursive path-dependent TreeSHAP of Lundberg et al. in float64,
 * with each node's training cover as the background distribution:
 *   out[i][k][f]  = float(sum over the trees t with t % K == k whose root cover
 *                   is > 0 of the Shapley value of feature f for row i)
 *   out[i][k][F]  = float(baseScores[k] + sum over those trees of the
 *                   cover-weighted mean leaf value)
 * Output layout rows x K x (F + 1), float32 (LightGBM's pred_contrib layout).
 *
 * One departure, where the reference is undefined: unwinding an element
 * whose one and zero fractions are both 0 (see unwind_path) sets the
 * remaining weights to 0 instead of dividing by zero.
 *
 * Routing follows the predictor restated in mbref.c (a categorical flag in a
 * tree without a catMask routes numerically; a rint outside the Int range
 * maps to the missing bin), which is where SHAP.swift's goesLeftRaw would
 * index an empty array or trap.  A tree whose cover array is empty takes no
 * part (SHAP.swift:190, :63); the caller rejects cover arrays of any other
 * length than the tree's node count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MB_FLAG_DEFAULT_LEFT 1u
#define MB_FLAG_CATEGORICAL 2u
#define MB_MAX_PATH 64 /* elements on one root-to-leaf path, plus the root dummy */

typedef struct {
    const int64_t *tree_off;
    int32_t T;
    const int32_t *feature;
    const float *threshold;
    const float *leaf;
    const uint8_t *flags;
    const uint32_t *catmask;
    const uint8_t *has_mask;
    const float *cover;
    const uint8_t *has_cover;
    int32_t data_bins;
    int32_t K;
    const double *bias; /* K expected values */
} shap_model;

typedef struct {
    int32_t feat;
    double zero, one, pw;
} path_el;

static inline int32_t cat_code(float v, int32_t data_bins) {
    if (!isfinite(v)) return data_bins;
    float r = rintf(v);
    if (r >= 0.0f && r < (float)data_bins) return (int32_t)r;
    return data_bins;
}

/* goesLeftRaw, SHAP.swift:210-221 */
static int goes_left(const shap_model *m, int32_t t, int64_t g, float v) {
    const uint32_t fl = m->flags[g];
    if ((fl & MB_FLAG_CATEGORICAL) && m->has_mask[t]) {
        const int32_t c = cat_code(v, m->data_bins);
        return (int)((m->catmask[g * 8 + (c >> 5)] >> (c & 31)) & 1u);
    }
    if (isnan(v)) return (fl & MB_FLAG_DEFAULT_LEFT) != 0;
    return v <= m->threshold[g];
}

/* extendPath, SHAP.swift:259-272: append (zero, one, feat) and update the
 * permutation weights of the path of length *len in place. */
static void extend_path(path_el *p, int *len, double zero, double one, int32_t feat) {
    const int l = *len;
    p[l].feat = feat;
    p[l].zero = zero;
    p[l].one = one;
    p[l].pw = l == 0 ? 1.0 : 0.0;
    for (int i = l - 1; i >= 0; --i) {
        p[i + 1].pw += one * p[i].pw * (double)(i + 1) / (double)(l + 1);
        p[i].pw = zero * p[i].pw * (double)(l - i) / (double)(l + 1);
    }
    *len = l + 1;
}

/* unwindPath, SHAP.swift:274-298: remove element `idx` from the path. */
static void unwind_path(path_el *p, int *len, int idx) {
    const int l = *len - 1;
    const double one = p[idx].one, zero = p[idx].zero;
    double next = p[l].pw;
    if (one != 0) {
        for (int i = l - 1; i >= 0; --i) {
            const double tmp = p[i].pw;
            p[i].pw = next * (double)(l + 1) / ((double)(i + 1) * one);
            next = tmp - p[i].pw * zero * (double)(l - i) / (double)(l + 1);
        }
    } else if (zero != 0) {
        for (int i = l - 1; i >= 0; --i) p[i].pw = p[i].pw * (double)(l + 1) / (zero * (double)(l - i));
    } else {
        /* one == zero == 0 (the cold side of a node with zero cover, met again
         * by a later split on the same feature): the path's weight polynomial
         * has the factor 0 + 0 t and is identically zero, so every weight
         * below is zero.  SHAP.swift:285-287 divides by zero here (NaN); zero
         * weights give the values of the Shapley definition. */
        for (int i = l - 1; i >= 0; --i) p[i].pw = 0.0;
    }
    for (int i = idx; i < l; ++i) {
        p[i].feat = p[i + 1].feat;
        p[i].zero = p[i + 1].zero;
        p[i].one = p[i + 1].one;
    }
    *len = l;
}

/* unwoundPathSum, SHAP.swift:300-324 */
static double unwound_sum(const path_el *p, int len, int idx) {
    const int l = len - 1;
    const double one = p[idx].one, zero = p[idx].zero;
    double next = p[l].pw, total = 0.0;
    if (one != 0) {
        for (int i = l - 1; i >= 0; --i) {
            const double tmp = next / ((double)(i + 1) * one);
            total += tmp;
            next = p[i].pw - tmp * zero * (double)(l - i);
        }
    } else if (zero != 0) {
        for (int i = l - 1; i >= 0; --i) total += p[i].pw / (zero * (double)(l - i));
    }
    return total * (double)(l + 1);
}

typedef struct {
    const shap_model *m;
    const float *x;
    int64_t rows, cols, ld;
    int32_t layout;
    int64_t i; /* row */
    double *phi;
} shap_ctx;

static inline float xval(const shap_ctx *c, int64_t f) {
    return c->layout == 0 ? c->x[f * c->ld + c->i] : c->x[c->i * c->cols + f];
}

/* shapRecurse, SHAP.swift:223-257.  `parent` (length plen) is the caller's
 * path; this frame works on its own copy. */
static void recurse(const shap_ctx *c, int32_t t, int64_t node, const path_el *parent, int plen,
                    double pzero, double pone, int32_t pfeat) {
    const shap_model *m = c->m;
    const int64_t b = m->tree_off[t];
    path_el p[MB_MAX_PATH];
    memcpy(p, parent, (size_t)plen * sizeof(path_el));
    int len = plen;
    extend_path(p, &len, pzero, pone, pfeat);
    if (m->feature[b + node] < 0) {
        const double v = (double)m->leaf[b + node];
        for (int i = 1; i < len; ++i) {
            const double w = unwound_sum(p, len, i);
            c->phi[p[i].feat] += w * (p[i].one - p[i].zero) * v;
        }
        return;
    }
    const int32_t f = m->feature[b + node];
    const int left = goes_left(m, t, b + node, xval(c, f));
    const int64_t hot = left ? 2 * node + 1 : 2 * node + 2;
    const int64_t cold = left ? 2 * node + 2 : 2 * node + 1;
    const double cn = (double)m->cover[b + node];
    const double hot_frac = cn > 0 ? (double)m->cover[b + hot] / cn : 0.0;
    const double cold_frac = cn > 0 ? (double)m->cover[b + cold] / cn : 0.0;
    double in_zero = 1.0, in_one = 1.0;
    for (int k = 0; k < len; ++k)
        if (p[k].feat == f) {
            in_zero = p[k].zero;
            in_one = p[k].one;
            unwind_path(p, &len, k);
            break;
        }
    recurse(c, t, hot, p, len, in_zero * hot_frac, in_one, f);
    recurse(c, t, cold, p, len, in_zero * cold_frac, 0.0, f);
}

typedef struct {
    const shap_model *m;
    const float *x;
    int64_t rows, cols, ld;
    int32_t layout;
    float *out;
    int64_t r0, r1;
} shap_job;

static void *shap_rows(void *arg) {
    const shap_job *j = (const shap_job *)arg;
    const shap_model *m = j->m;
    const int64_t W = j->cols + 1;
    double *phi = (double *)malloc((size_t)W * sizeof(double));
    if (!phi) return NULL;
    shap_ctx c = {m, j->x, j->rows, j->cols, j->ld, j->layout, 0, phi};
    for (int64_t i = j->r0; i < j->r1; ++i) {
        c.i = i;
        for (int32_t k = 0; k < m->K; ++k) {
            for (int64_t f = 0; f < W; ++f) phi[f] = 0.0;
            for (int32_t t = k; t < m->T; t += m->K) {
                if (!m->has_cover[t] || !(m->cover[m->tree_off[t]] > 0)) continue;
                recurse(&c, t, 0, NULL, 0, 1.0, 1.0, -1);
            }
            float *o = j->out + (i * m->K + k) * W;
            for (int64_t f = 0; f < j->cols; ++f) o[f] = (float)phi[f];
            o[j->cols] = (float)m->bias[k];
        }
    }
    free(phi);
    return NULL;
}

/* shapBias, SHAP.swift:56-72: per class, baseScores[k] plus each tree's
 * cover-weighted mean leaf value, visiting nodes in the reference's stack order. */
static int shap_bias(const shap_model *m, const float *base, double *bias) {
    for (int32_t k = 0; k < m->K; ++k) bias[k] = (double)base[k];
    int64_t cap = 1024;
    int64_t *stack = (int64_t *)malloc((size_t)cap * sizeof(int64_t));
    if (!stack) return -1;
    for (int32_t t = 0; t < m->T; ++t) {
        if (!m->has_cover[t]) continue;
        const int64_t b = m->tree_off[t];
        const double total = (double)m->cover[b];
        if (!(total > 0)) continue;
        double mean = 0.0;
        int64_t sp = 0;
        stack[sp++] = 0;
        while (sp > 0) {
            const int64_t n = stack[--sp];
            if (m->feature[b + n] >= 0) {
                if (sp + 2 > cap) {
                    cap *= 2;
                    int64_t *s2 = (int64_t *)realloc(stack, (size_t)cap * sizeof(int64_t));
                    if (!s2) {
                        free(stack);
                        return -1;
                    }
                    stack = s2;
                }
                stack[sp++] = 2 * n + 1;
                stack[sp++] = 2 * n + 2;
            } else {
                mean += (double)m->leaf[b + n] * (double)m->cover[b + n] / total;
            }
        }
        bias[t % m->K] += mean;
    }
    free(stack);
    return 0;
}

/*
 * Contributions for `rows` rows (layout 0: x[f*ld+i]; 1: x[i*cols+f]) into
 * out[rows * K * (cols + 1)].  `cover` holds a value per node for the trees
 * with has_cover[t] == 1 (other trees' entries are ignored).  Returns 0, or
 * -1 for invalid arguments or a path deeper than MB_MAX_PATH - 1.
 */
int mbref_shap(const int64_t *tree_off, int32_t T, const int32_t *feature, const float *threshold,
               const float *leaf, const uint8_t *flags, const uint32_t *catmask,
               const uint8_t *has_mask, const float *cover, const uint8_t *has_cover,
               int32_t data_bins, int32_t K, const float *base, const float *x, int64_t rows,
               int64_t cols, int64_t ld, int32_t layout, float *out, int32_t nthreads) {
    if (K < 1 || rows < 0 || cols < 0 || T < 0 || (layout == 0 && ld < rows)) return -1;
    for (int32_t t = 0; t < T; ++t) {
        /* depth bound: heap index of every node below 2^(MB_MAX_PATH - 2) */
        const int64_t n = tree_off[t + 1] - tree_off[t];
        if (n >= ((int64_t)1 << (MB_MAX_PATH - 2))) return -1;
    }
    double *bias = (double *)malloc((size_t)K * sizeof(double));
    if (!bias) return -1;
    shap_model m = {tree_off, T, feature, threshold, leaf, flags, catmask,
                    has_mask, cover, has_cover, data_bins, K, bias};
    if (shap_bias(&m, base, bias) != 0) {
        free(bias);
        return -1;
    }
    if (nthreads < 1) nthreads = 1;
    if (rows < (int64_t)nthreads * 16) nthreads = 1;
    shap_job *jobs = (shap_job *)calloc((size_t)nthreads, sizeof(shap_job));
    pthread_t *tid = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !tid) {
        free(jobs);
        free(tid);
        free(bias);
        return -1;
    }
    for (int32_t k = 0; k < nthreads; ++k) {
        shap_job jb = {&m, x, rows, cols, ld, layout, out, rows * k / nthreads,
                       rows * (k + 1) / nthreads};
        jobs[k] = jb;
    }
    int32_t started = 0;
    for (int32_t k = 1; k < nthreads; ++k) {
        if (pthread_create(&tid[k], NULL, shap_rows, &jobs[k]) != 0) break;
        started = k;
    }
    shap_rows(&jobs[0]);
    for (int32_t k = started + 1; k < nthreads; ++k) shap_rows(&jobs[k]);
    for (int32_t k = 1; k <= started; ++k) pthread_join(tid[k], NULL);
    free(jobs);
    free(tid);
    free(bias);
    return 0;
}
