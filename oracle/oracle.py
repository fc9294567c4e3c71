"""Parity oracle for MacBoost batch inference (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this module; the product (``macboost_b200``) never does.

* The model JSON is read with Python's ``json`` module into numpy arrays, the
  way the reference's ``PyModel.__init__`` reads it
  (python/macboost/_pyinfer.py:22-46): floats go through float64 and are then
  rounded to float32.  This keeps the oracle independent of the product's C++
  parser.
* Margins and leaf indices come from ``mbref.c``, a C restatement of
  ``predictCPU`` (Sources/MacBoost/Booster.swift:2035-2117) with PyModel's
  choices where the two differ (see the header of mbref.c).
* Transforms restate the reference formulas: ``predict`` applies fp32 ``exp``
  for the log-link objectives (Booster.swift:1993-1999, _pyinfer.py:91-95);
  ``predict_proba`` evaluates sigmoid / softmax in float64
  (python/macboost/__init__.py:439-445).
"""

from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmbref.so"

LOG_LINK_OBJECTIVES = (5, 6)   # poisson, tweedie (Booster.swift:15)


def build(force: bool = False) -> Path:
    """Compile mbref.c and mbshap.c into oracle/libmbref.so with gcc (no
    fast-math, no contraction of multiply-adds)."""
    srcs = [HERE / "mbref.c", HERE / "mbshap.c", HERE / "mbbinned.c"]
    if force or not LIB_PATH.exists() or any(LIB_PATH.stat().st_mtime < s.stat().st_mtime
                                             for s in srcs):
        import subprocess
        tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
        subprocess.run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
                        "-fno-fast-math", "-pthread", "-o", str(tmp), *map(str, srcs), "-lm"],
                       check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        lib.mbref_predict.restype = ctypes.c_int32
        lib.mbref_predict.argtypes = [P, ctypes.c_int32, P, P, P, P, P, P, ctypes.c_int32,
                                      ctypes.c_int32, P, P, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int32, P, P, ctypes.c_int32]
        lib.mbref_bin_data.restype = ctypes.c_int32
        lib.mbref_bin_data.argtypes = [P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int32, P, ctypes.c_int32, P, P]
        lib.mbref_predict_binned.restype = ctypes.c_int32
        lib.mbref_predict_binned.argtypes = [P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                             P, P, P, P, P, P, ctypes.c_int32, ctypes.c_int32,
                                             P, P]
        lib.mbref_shap.restype = ctypes.c_int32
        lib.mbref_shap.argtypes = [P, ctypes.c_int32, P, P, P, P, P, P, P, P, ctypes.c_int32,
                                   ctypes.c_int32, P, P, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_int64, ctypes.c_int32, P, ctypes.c_int32]
        _lib = lib
    return _lib


@dataclass
class OracleModel:
    objective: int
    num_bins: int
    num_features: int
    num_classes: int
    base_scores: np.ndarray      # float32[K]
    tree_off: np.ndarray         # int64[T+1]
    feature: np.ndarray          # int32[N]
    threshold: np.ndarray        # float32[N]
    leaf: np.ndarray             # float32[N]
    flags: np.ndarray            # uint8[N]
    catmask: np.ndarray          # uint32[N*8]
    has_mask: np.ndarray         # uint8[T]
    cover: np.ndarray | None = None      # float32[N] (0 where a tree has none)
    has_cover: np.ndarray | None = None  # uint8[T]

    @property
    def num_trees(self) -> int:
        return len(self.tree_off) - 1


def load_model(path) -> OracleModel:
    """Read a MacBoost model.json the way PyModel does (_pyinfer.py:22-46)."""
    with open(path) as fh:
        m = json.load(fh)
    return model_from_dict(m)


def model_from_dict(m: dict) -> OracleModel:
    if m.get("version") != 1:
        raise ValueError("unsupported model file version")
    K = int(m.get("numClasses") or 1)
    base = np.asarray(m.get("baseScores") or [m["baseScore"]], dtype=np.float32)
    feats, thrs, leaves, flags, masks, has = [], [], [], [], [], []
    covers, has_cov = [], []
    off = [0]
    for t in m["trees"]:
        f = np.asarray(t["feature"], dtype=np.int64).astype(np.int32)
        n = len(f)
        feats.append(f)
        cv = np.asarray(t.get("cover") or [], dtype=np.float32)
        if cv.size not in (0, n):
            raise ValueError(f"a tree has {cv.size} cover values for {n} nodes")
        covers.append(cv if cv.size else np.zeros(n, np.float32))
        has_cov.append(1 if cv.size else 0)
        thrs.append(np.asarray(t["threshold"], dtype=np.float32))
        leaves.append(np.asarray(t["leaf"], dtype=np.float32))
        flags.append(np.asarray(t["flags"], dtype=np.uint8))
        cm = np.asarray(t.get("catMask") or [], dtype=np.uint64).astype(np.uint32)
        if cm.size:
            masks.append(cm)
            has.append(1)
        else:
            masks.append(np.zeros(n * 8, dtype=np.uint32))
            has.append(0)
        off.append(off[-1] + n)

    def cat(parts, dt):
        return np.concatenate(parts).astype(dt) if parts else np.zeros(0, dt)

    return OracleModel(
        objective=int(m["objective"]), num_bins=int(m["numBins"]),
        num_features=int(m["numFeatures"]), num_classes=K, base_scores=base,
        tree_off=np.asarray(off, dtype=np.int64), feature=cat(feats, np.int32),
        threshold=cat(thrs, np.float32), leaf=cat(leaves, np.float32),
        flags=cat(flags, np.uint8), catmask=cat(masks, np.uint32),
        has_mask=np.asarray(has, dtype=np.uint8), cover=cat(covers, np.float32),
        has_cover=np.asarray(has_cov, dtype=np.uint8))


def _ptr(a):
    return a.ctypes.data if a is not None and a.size else None


def predict_raw(model: OracleModel, X, layout: str = "row", want_leaf: bool = False,
                nthreads: int | None = None):
    """Raw fp32 margins (rows, K) [and int32 leaf heap indices (rows, T)].

    layout="row": X is (rows, F) row-major; layout="feature": X is (F, rows)
    feature-major, the reference C ABI's layout (CAPI.swift:5-6)."""
    lib = _load()
    X = np.ascontiguousarray(X, dtype=np.float32)
    if layout == "row":
        rows, cols = X.shape
        lay, ld = 1, cols
    else:
        cols, rows = X.shape
        lay, ld = 0, rows
    if cols != model.num_features:
        raise ValueError(f"model expects {model.num_features} features, got {cols}")
    K, T = model.num_classes, model.num_trees
    out = np.empty((rows, K), dtype=np.float32)
    leaf = np.empty((rows, T), dtype=np.int32) if want_leaf else None
    nt = nthreads or os.cpu_count() or 1
    rc = lib.mbref_predict(
        _ptr(model.tree_off), T, _ptr(model.feature), _ptr(model.threshold),
        _ptr(model.leaf), _ptr(model.flags), _ptr(model.catmask), _ptr(model.has_mask),
        model.num_bins - 1, K, _ptr(model.base_scores), _ptr(X), rows, cols, ld, lay,
        out.ctypes.data if rows else None, _ptr(leaf), nt)
    if rc != 0:
        raise RuntimeError("mbref_predict rejected its arguments")
    return (out, leaf) if want_leaf else out


def predict_contrib(model: OracleModel, X, layout: str = "row", nthreads: int | None = None):
    """TreeSHAP contributions, float32 (rows, K * (F + 1)): per class the F
    feature contributions then the expected value (mbshap.c restating
    Sources/MacBoost/SHAP.swift:170-326 and :56-72)."""
    lib = _load()
    X = np.ascontiguousarray(X, dtype=np.float32)
    if layout == "row":
        rows, cols = X.shape
        lay, ld = 1, cols
    else:
        cols, rows = X.shape
        lay, ld = 0, rows
    if cols != model.num_features:
        raise ValueError(f"model expects {model.num_features} features, got {cols}")
    K, T = model.num_classes, model.num_trees
    out = np.empty((rows, K * (cols + 1)), dtype=np.float32)
    rc = lib.mbref_shap(
        _ptr(model.tree_off), T, _ptr(model.feature), _ptr(model.threshold), _ptr(model.leaf),
        _ptr(model.flags), _ptr(model.catmask), _ptr(model.has_mask), _ptr(model.cover),
        _ptr(model.has_cover), model.num_bins - 1, K, _ptr(model.base_scores), _ptr(X), rows,
        cols, ld, lay, out.ctypes.data if out.size else None, nthreads or os.cpu_count() or 1)
    if rc != 0:
        raise RuntimeError("mbref_shap rejected its arguments")
    return out


def shapley_bruteforce(model: OracleModel, x: np.ndarray) -> np.ndarray:
    """Exact Shapley values of one row from their definition, as an
    independent check of the TreeSHAP restatement: the value of a coalition S
    is the tree's expectation with the features outside S integrated out by
    node cover fractions (Lundberg et al. 2020, Algorithm 1; a node with zero
    cover gives its children fraction 0, as the reference does), and
    phi_j = sum over S not containing j of |S|!(M-|S|-1)!/M! (v(S+j) - v(S)).
    Pure Python, exponential in the number of features: tiny models only.
    Returns float64 (K, F + 1), the last column the expected value v({})."""
    from itertools import combinations
    from math import factorial

    F, K = model.num_features, model.num_classes
    x = np.asarray(x, dtype=np.float32)

    def goes_left(t, g, v):
        fl = int(model.flags[g])
        if (fl & 2) and model.has_mask[t]:
            c = model.num_bins - 1
            if np.isfinite(v):
                r = np.rint(v)
                if 0 <= r < model.num_bins - 1:
                    c = int(r)
            return (int(model.catmask[g * 8 + c // 32]) >> (c % 32)) & 1 == 1
        if np.isnan(v):
            return (fl & 1) != 0
        return bool(v <= model.threshold[g])

    def expect(t, n, S):
        b = int(model.tree_off[t])
        f = int(model.feature[b + n])
        if f < 0:
            return float(model.leaf[b + n])
        left, right = 2 * n + 1, 2 * n + 2
        if f in S:
            return expect(t, left if goes_left(t, b + n, x[f]) else right, S)
        cn = float(model.cover[b + n])
        # cover fractions, 0 below a node no training row reached (SHAP.swift:241-242)
        fl = float(model.cover[b + left]) / cn if cn > 0 else 0.0
        fr = float(model.cover[b + right]) / cn if cn > 0 else 0.0
        return fl * expect(t, left, S) + fr * expect(t, right, S)

    out = np.zeros((K, F + 1))
    for k in range(K):
        out[k, F] = float(model.base_scores[k])
    for t in range(model.num_trees):
        if not model.has_cover[t] or not model.cover[model.tree_off[t]] > 0:
            continue
        k = t % K
        v = {}
        for r in range(F + 1):
            for S in combinations(range(F), r):
                v[S] = expect(t, 0, set(S))
        out[k, F] += v[()]
        for j in range(F):
            others = [i for i in range(F) if i != j]
            for r in range(F):
                w = factorial(r) * factorial(F - r - 1) / factorial(F)
                for S in combinations(others, r):
                    Sj = tuple(sorted(S + (j,)))
                    out[k, j] += w * (v[Sj] - v[S])
    return out


# ---- binned data (oracle/mbbinned.c restating Shaders.swift:37-76, 1741-1781) ----

def bin_data(X, edges, num_bins: int, categorical, layout: str = "row") -> np.ndarray:
    """Tiled uint8 bins, ceil(F/8) * 8 * rows bytes (bin_data, Shaders.swift:41-76)."""
    lib = _load()
    X = np.ascontiguousarray(X, dtype=np.float32)
    if layout == "row":
        rows, cols = X.shape
        lay, ld = 1, cols
    else:
        cols, rows = X.shape
        lay, ld = 0, rows
    edges = np.ascontiguousarray(edges, dtype=np.float32)
    cat = np.zeros(cols, np.uint8)
    cat[list(categorical)] = 1
    out = np.empty(((cols + 7) // 8) * 8 * rows, dtype=np.uint8)
    if lib.mbref_bin_data(_ptr(X), rows, cols, ld, lay, _ptr(edges), num_bins, _ptr(cat),
                          _ptr(out)) != 0:
        raise RuntimeError("mbref_bin_data rejected its arguments")
    return out


@dataclass
class SplitForest:
    """Trees in the trainer's split form (NodeSplit, Shaders.swift:466)."""
    tree_off: np.ndarray   # int64[T+1]
    feature: np.ndarray    # int32[N], < 0 for leaves
    bin: np.ndarray        # uint32[N]
    flags: np.ndarray      # uint32[N]
    catmask: np.ndarray    # uint32[N*8]
    leaf: np.ndarray       # float32[N]


def split_form(model: OracleModel, edges, num_bins: int) -> SplitForest:
    """A model's trees in split form against a dataset's edges: each numeric
    threshold is the edge it was trained at (Booster.swift:938 writes
    threshold = edges[f * (numBins - 2) + bin]); the first matching edge."""
    ne = num_bins - 2
    edges = np.asarray(edges, dtype=np.float32).reshape(-1, ne)
    N = len(model.feature)
    sb = np.zeros(N, np.uint32)
    mask = np.zeros(N * 8, np.uint32)
    for t in range(model.num_trees):
        for g in range(int(model.tree_off[t]), int(model.tree_off[t + 1])):
            f = int(model.feature[g])
            if f < 0:
                continue
            if (model.flags[g] & 2) and model.has_mask[t]:
                mask[g * 8:(g + 1) * 8] = model.catmask[g * 8:(g + 1) * 8]
                continue
            hit = np.nonzero(edges[f] == model.threshold[g])[0]
            if not hit.size:
                raise ValueError(f"threshold {model.threshold[g]!r} of feature {f} is not a bin edge")
            sb[g] = hit[0]
    fl = model.flags.astype(np.uint32).copy()
    for t in range(model.num_trees):
        if not model.has_mask[t]:   # a categorical flag without a mask routes numerically
            a, b = int(model.tree_off[t]), int(model.tree_off[t + 1])
            fl[a:b] &= ~np.uint32(2)
    return SplitForest(model.tree_off, model.feature, sb, fl, mask, model.leaf)


def predict_binned(bins: np.ndarray, rows: int, num_bins: int, sf: SplitForest, max_depth: int,
                   K: int = 1, preds: np.ndarray | None = None, want_leaf: bool = False):
    """predict_tree_binned over every tree in order into class-major preds
    (K x rows, float32, updated in place) and/or assign_leaves indices (T x rows)."""
    lib = _load()
    T = len(sf.tree_off) - 1
    leaf = np.empty((T, rows), np.int32) if want_leaf else None
    if lib.mbref_predict_binned(_ptr(np.ascontiguousarray(bins, np.uint8)), rows, num_bins, T,
                                _ptr(sf.tree_off), _ptr(sf.feature), _ptr(sf.bin),
                                _ptr(sf.flags), _ptr(sf.catmask), _ptr(sf.leaf), max_depth, K,
                                _ptr(preds), _ptr(leaf)) != 0:
        raise RuntimeError("mbref_predict_binned rejected its arguments")
    return leaf


def compute_edges(X, num_bins: int, categorical=(), layout: str = "row",
                  sample_cap: int = 200_000) -> np.ndarray:
    """Binner.computeEdges (Sources/MacBoost/Binner.swift:25-60): per numeric
    feature every max(1, rows // sample_cap)-th value, NaNs dropped, sorted;
    edge k (k < num_bins - 2) = sample[min(m - 1, (k + 1) * m // (num_bins - 1))].
    Categorical and all-NaN features keep zeros.  cols x (num_bins - 2) fp32."""
    a = np.asarray(X, dtype=np.float32)
    fm = a.T if layout == "row" else a
    cols, rows = fm.shape
    data_bins = num_bins - 1
    ne = data_bins - 1
    step = max(1, rows // sample_cap)
    edges = np.zeros((cols, ne), np.float32)
    cats = set(int(c) for c in categorical)
    k = np.arange(ne, dtype=np.int64)
    for f in range(cols):
        if f in cats:
            continue
        s = fm[f, ::step]
        s = s[~np.isnan(s)]
        m = s.size
        if m == 0:
            continue
        s = np.sort(s, kind="stable")
        edges[f] = s[np.minimum(m - 1, (k + 1) * m // data_bins)]
    return edges.reshape(-1)


def make_dataset(X, labels, num_bins: int, categorical=(), layout: str = "row"):
    """MacBooster.makeDataset (Sources/MacBoost/Booster.swift:392-434) without
    its error checks: (edges, tiled bins)."""
    edges = compute_edges(X, num_bins, categorical, layout)
    return edges, bin_data(X, edges, num_bins, categorical, layout)


def write_mbds(path, bins, rows: int, cols: int, num_bins: int, categorical, feature_names,
               edges, labels) -> None:
    """A .mbds file as BinnedDataset.save writes it (Sources/MacBoost/Dataset.swift:26-39)."""
    import struct
    # JSONEncoder: compact, UTF-8 as is, "/" escaped
    names = (json.dumps(list(feature_names), separators=(",", ":"), ensure_ascii=False)
             .replace("/", "\\/").encode() if feature_names is not None else b"")
    with open(path, "wb") as fh:
        fh.write(struct.pack("<III", 0x4D424453, 1, 8))
        fh.write(struct.pack("<QII", rows, cols, num_bins))
        cats = sorted(categorical)
        fh.write(struct.pack("<I", len(cats)))
        for c in cats:
            fh.write(struct.pack("<I", c))
        fh.write(struct.pack("<I", len(names)))
        fh.write(names)
        e = np.ascontiguousarray(edges, np.float32)
        fh.write(struct.pack("<Q", e.size))
        fh.write(e.tobytes())
        lab = np.ascontiguousarray(labels, np.float32)
        fh.write(struct.pack("<Q", lab.size))
        fh.write(lab.tobytes())
        b = np.ascontiguousarray(bins, np.uint8)
        fh.write(struct.pack("<Q", b.size))
        fh.write(b.tobytes())


def predict(model: OracleModel, raw: np.ndarray) -> np.ndarray:
    """`predict` semantics on raw margins: fp32 exp for poisson/tweedie."""
    if model.objective in LOG_LINK_OBJECTIVES:
        return np.exp(raw.astype(np.float32))
    return raw


def predict_cli(model: OracleModel, raw: np.ndarray) -> np.ndarray:
    """What `macboost predict` writes (Sources/MacBoostCLI/main.swift:344-364),
    in float32: `predict` (exp for log-link objectives), then per row a softmax
    (max-shifted, class-order float32 sum, divide) when K > 1, or
    1 / (1 + exp(-x)) for the binary objective.  exp is the float32 rounding
    of the float64 exp (a correctly rounded expf)."""
    def exp32(x):
        return np.exp(np.asarray(x, dtype=np.float64)).astype(np.float32)

    v = np.asarray(raw, dtype=np.float32).reshape(raw.shape[0], -1).copy()
    if model.objective in LOG_LINK_OBJECTIVES:
        v = exp32(v)
    K = v.shape[1]
    if K > 1:
        mx = np.full(v.shape[0], -np.inf, dtype=np.float32)
        for c in range(K):
            mx = np.where(v[:, c] > mx, v[:, c], mx)
        s = np.zeros(v.shape[0], dtype=np.float32)
        for c in range(K):
            v[:, c] = exp32(v[:, c] - mx)
            s = (s + v[:, c]).astype(np.float32)
        return (v / s[:, None]).astype(np.float32)
    if model.objective == 1:
        one = np.float32(1.0)
        return (one / (one + exp32(-v))).astype(np.float32)
    return v


def predict_proba(raw: np.ndarray) -> np.ndarray:
    """MacBoostClassifier.predict_proba formula (__init__.py:439-445), float64."""
    raw = np.asarray(raw).astype(np.float64)
    if raw.ndim == 2 and raw.shape[1] > 1:
        e = np.exp(raw - raw.max(axis=1, keepdims=True))
        return e / e.sum(axis=1, keepdims=True)
    p = 1.0 / (1.0 + np.exp(-raw.reshape(-1)))
    return np.column_stack([1 - p, p])


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in fp32 units-in-the-last-place between two float32 arrays."""
    a = np.ascontiguousarray(a, dtype=np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, dtype=np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)
