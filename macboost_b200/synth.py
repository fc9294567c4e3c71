"""Seeded synthetic MacBoost models and feature matrices for the five benchmark
configurations (BASELINE.json ``configs``).

Models are written in MacBoost's JSON model format -- the ``ModelFile`` keys of
Sources/MacBoost/Booster.swift:2119-2130 (version, objective, numBins,
baseScore, numFeatures, categorical, trees, numClasses, baseScores) with trees
in the implicit-heap layout of Booster.swift:119-146 (feature < 0 marks a leaf,
flags bit0 = missing goes left, bit1 = categorical, catMask 8 words per node or
empty, every array sized 2^(maxDepth+1)-1 as the trainer sizes them at
Booster.swift:517).

Feature data is generated in independent chunks of ``CHUNK`` rows, chunk ``c``
seeded by ``SeedSequence(seed, spawn_key=(c,))``, so any row slice (one GPU's
shard) regenerates on its own without generating the rows before it.

No public dataset is used: each configuration's distributions are stated in
its ``Config.data`` description and reproduced here from the seed.
"""

from __future__ import annotations

import json
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

CHUNK = 1 << 16
EDGES_256 = (np.arange(1, 256, dtype=np.float64) / 256.0).astype(np.float32)


@dataclass(frozen=True)
class Config:
    name: str
    rows: int
    features: int
    trees: int
    classes: int
    objective: int
    output: str            # "raw" | "sigmoid" | "softmax"
    data: str
    model: str
    model_seed: int
    data_seed: int
    extra: dict = field(default_factory=dict)


CONFIGS = {
    "cfg1": Config("cfg1", 500_000, 100, 100, 1, 0, "raw",
                   "500,000 x 100 fp32, iid Uniform[0,1), no NaN",
                   "100 complete depth-6 trees; uniform random split feature; threshold "
                   "uniform over the 255 bin edges k/256; random default-left bit; leaves "
                   "N(0, 0.05^2); base 0; L2", 101, 1001),
    "cfg2": Config("cfg2", 10_000_000, 28, 100, 1, 1, "sigmoid",
                   "10,000,000 x 28 fp32; f0-20 LogNormal(0, 0.5), f21-27 N(0, 1)",
                   "100 complete depth-6 trees; thresholds from the feature's empirical "
                   "k/256 quantiles (k=1..255) of a seeded 100k-row sample; leaves "
                   "N(0, 0.1^2); base margin -0.1; binary logistic (sigmoid)", 102, 1002),
    "cfg3": Config("cfg3", 1_000_000, 100, 100, 1, 0, "raw",
                   "1,000,000 x 100; cols 0-79 Uniform[0,1) with NaN p=0.2; cols 80-99 "
                   "integer codes 0-31 from a truncated Zipf(1.1) stored as fp32",
                   "100 complete depth-6 trees; numeric splits on bin edges with random "
                   "default; categorical splits (cols 80-99) with random 32-bit subsets and "
                   "bits 32-255 equal to the node's random default; leaves N(0, 0.05^2); L2",
                   103, 1003),
    "cfg4": Config("cfg4", 10_000_000, 100, 1000, 10, 7, "softmax",
                   "10,000,000 x 100 fp32 Uniform[0,1) with NaN p=0.05",
                   "10 classes x 100 rounds = 1,000 complete depth-6 trees, tree t scores "
                   "class t % 10; bin-edge thresholds; leaves N(0, 0.05^2); base scores 0; "
                   "softmax", 104, 1004),
    "cfg5": Config("cfg5", 50_000_000, 100, 500, 1, 0, "raw",
                   "50,000,000 x 100 fp32 Uniform[0,1) with NaN p=0.1",
                   "500 leaf-wise trees of 255 leaves: a uniformly chosen splittable leaf "
                   "(depth < 12, the reference's maxDepth cap) is split until 255 leaves; "
                   "bin-edge thresholds; random default; leaves N(0, 0.02^2); raw margin",
                   105, 1005, {"max_depth": 12, "num_leaves": 255}),
}


# --------------------------------------------------------------------------
# feature data
# --------------------------------------------------------------------------

_ZIPF_P = (np.arange(1, 33, dtype=np.float64)) ** -1.1
_ZIPF_CDF = np.cumsum(_ZIPF_P / _ZIPF_P.sum())


def _chunk_rows(cfg: Config, rng: np.random.Generator, n: int) -> np.ndarray:
    """n rows of cfg's distribution, row-major (n, F) float32."""
    F = cfg.features
    if cfg.name == "cfg1":
        return rng.random((n, F), dtype=np.float32)
    if cfg.name == "cfg2":
        x = np.empty((n, F), dtype=np.float32)
        x[:, :21] = rng.lognormal(0.0, 0.5, (n, 21)).astype(np.float32)
        x[:, 21:] = rng.standard_normal((n, 7), dtype=np.float32)
        return x
    if cfg.name == "cfg3":
        x = np.empty((n, F), dtype=np.float32)
        num = rng.random((n, 80), dtype=np.float32)
        num[rng.random((n, 80)) < 0.2] = np.nan
        x[:, :80] = num
        u = rng.random((n, 20))
        codes = np.searchsorted(_ZIPF_CDF, u, side="right")
        x[:, 80:] = np.minimum(codes, 31).astype(np.float32)
        return x
    p_nan = {"cfg4": 0.05, "cfg5": 0.10}[cfg.name]
    x = rng.random((n, F), dtype=np.float32)
    x[rng.random((n, F), dtype=np.float32) < p_nan] = np.nan
    return x


def make_data(cfg: Config | str, rows: int | None = None, row_start: int = 0,
              seed: int | None = None, layout: str = "feature", out: np.ndarray | None = None,
              threads: int | None = None) -> np.ndarray:
    """Rows [row_start, row_start+rows) of the config's feature matrix.

    layout="feature" returns (F, rows) feature-major (the C ABI's layout);
    layout="row" returns (rows, F).  ``out`` may be a preallocated (e.g. pinned)
    float32 array of that shape."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    rows = cfg.rows if rows is None else rows
    seed = cfg.data_seed if seed is None else seed
    F = cfg.features
    shape = (F, rows) if layout == "feature" else (rows, F)
    if out is None:
        out = np.empty(shape, dtype=np.float32)
    assert out.shape == shape and out.dtype == np.float32
    first, last = row_start // CHUNK, (row_start + rows + CHUNK - 1) // CHUNK

    def work(c):
        rng = np.random.default_rng(np.random.SeedSequence(seed, spawn_key=(c,)))
        block = _chunk_rows(cfg, rng, CHUNK)
        a = max(row_start, c * CHUNK)
        b = min(row_start + rows, (c + 1) * CHUNK)
        src = block[a - c * CHUNK:b - c * CHUNK]
        if layout == "feature":
            out[:, a - row_start:b - row_start] = src.T
        else:
            out[a - row_start:b - row_start] = src

    nthreads = threads or min(32, os.cpu_count() or 1)
    if last - first <= 1 or nthreads == 1:
        for c in range(first, last):
            work(c)
    else:
        with ThreadPoolExecutor(nthreads) as ex:
            list(ex.map(work, range(first, last)))
    return out


# --------------------------------------------------------------------------
# models
# --------------------------------------------------------------------------

def _empty_tree(n_nodes: int, with_mask: bool) -> dict:
    return {
        "feature": np.full(n_nodes, -1, dtype=np.int32),
        "threshold": np.zeros(n_nodes, dtype=np.float32),
        "leaf": np.zeros(n_nodes, dtype=np.float32),
        "flags": np.zeros(n_nodes, dtype=np.uint8),
        "catMask": np.zeros(n_nodes * 8, dtype=np.uint32) if with_mask else None,
    }


def _split(tree: dict, n: int, rng: np.random.Generator, feat: int, thr_choices,
           cat_features: frozenset):
    tree["feature"][n] = feat
    dl = int(rng.integers(0, 2))
    if feat in cat_features:
        tree["flags"][n] = 2 | dl
        words = np.zeros(8, dtype=np.uint32)
        bits = rng.random(32) < 0.5
        words[0] = np.uint32(np.sum(bits.astype(np.uint64) << np.arange(32, dtype=np.uint64)))
        if dl:
            words[1:] = 0xFFFFFFFF          # unseen / missing codes follow the default
        tree["catMask"][n * 8:(n + 1) * 8] = words
    else:
        tree["flags"][n] = dl
        choices = thr_choices[feat] if isinstance(thr_choices, list) else thr_choices
        tree["threshold"][n] = choices[int(rng.integers(0, len(choices)))]


def _complete_tree(rng, depth: int, F: int, thr_choices, sigma: float,
                   cat_features: frozenset = frozenset(), with_mask: bool = False) -> dict:
    n_nodes = (1 << (depth + 1)) - 1
    tree = _empty_tree(n_nodes, with_mask)
    for n in range((1 << depth) - 1):
        _split(tree, n, rng, int(rng.integers(0, F)), thr_choices, cat_features)
    first_leaf = (1 << depth) - 1
    tree["leaf"][first_leaf:] = (rng.standard_normal(1 << depth) * sigma).astype(np.float32)
    return tree


def _leafwise_tree(rng, num_leaves: int, max_depth: int, F: int, thr_choices,
                   sigma: float) -> dict:
    n_nodes = (1 << (max_depth + 1)) - 1
    tree = _empty_tree(n_nodes, False)
    leaves = [0]
    depth = {0: 0}
    while len(leaves) < num_leaves:
        splittable = [i for i, n in enumerate(leaves) if depth[n] < max_depth]
        if not splittable:
            break
        k = splittable[int(rng.integers(0, len(splittable)))]
        n = leaves.pop(k)
        _split(tree, n, rng, int(rng.integers(0, F)), thr_choices, frozenset())
        for ch in (2 * n + 1, 2 * n + 2):
            depth[ch] = depth[n] + 1
            leaves.append(ch)
    vals = (rng.standard_normal(len(leaves)) * sigma).astype(np.float32)
    for n, v in zip(sorted(leaves), vals):
        tree["leaf"][n] = v
    return tree


def _quantile_edges(cfg: Config, seed: int) -> list:
    """Per feature, the empirical k/256 quantiles (k = 1..255) of a 100k-row
    seeded sample, picked like Binner.swift:47-51 (sorted sample, index
    min(m-1, k*m/256))."""
    sample = make_data(cfg, rows=100_000, seed=seed, layout="row")
    out = []
    for f in range(cfg.features):
        s = np.sort(sample[:, f][~np.isnan(sample[:, f])])
        m = len(s)
        idx = np.minimum(m - 1, (np.arange(1, 256) * m) // 256)
        out.append(s[idx].astype(np.float32))
    return out


def make_model(cfg: Config | str, trees: int | None = None, seed: int | None = None) -> dict:
    """The config's model as a MacBoost ModelFile dict (numpy arrays inside)."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    T = cfg.trees if trees is None else trees
    seed = cfg.model_seed if seed is None else seed
    rng = np.random.default_rng(seed)
    F = cfg.features
    cats: frozenset = frozenset()
    base = [0.0] * cfg.classes
    if cfg.name == "cfg1":
        tl = [_complete_tree(rng, 6, F, EDGES_256, 0.05) for _ in range(T)]
    elif cfg.name == "cfg2":
        edges = _quantile_edges(cfg, seed + 7_000_000)
        tl = [_complete_tree(rng, 6, F, edges, 0.1) for _ in range(T)]
        base = [float(np.float32(-0.1))]
    elif cfg.name == "cfg3":
        cats = frozenset(range(80, 100))
        tl = [_complete_tree(rng, 6, F, EDGES_256, 0.05, cats, with_mask=True)
              for _ in range(T)]
    elif cfg.name == "cfg4":
        tl = [_complete_tree(rng, 6, F, EDGES_256, 0.05) for _ in range(T)]
    elif cfg.name == "cfg5":
        tl = [_leafwise_tree(rng, cfg.extra["num_leaves"], cfg.extra["max_depth"], F,
                             EDGES_256, 0.02) for _ in range(T)]
    else:
        raise KeyError(cfg.name)
    model = {
        "version": 1,
        "objective": cfg.objective,
        "numBins": 256,
        "baseScore": base[0],
        "numFeatures": F,
        "categorical": sorted(cats),
        "trees": tl,
        "numClasses": cfg.classes,
        "baseScores": base,
    }
    return model


def add_covers(model: dict, X: np.ndarray) -> dict:
    """Give every tree a `cover` array: the number of rows of X (row-major,
    numFeatures columns) that reach each node, which is what a trainer with
    unit hessians stores (Booster.swift:126).  Routing as the predictor:
    categorical mask bit, NaN to the default side, else v <= threshold."""
    X = np.asarray(X, dtype=np.float32)
    data_bins = int(model["numBins"]) - 1
    for t in model["trees"]:
        feat = np.asarray(t["feature"], dtype=np.int64)
        thr = np.asarray(t["threshold"], dtype=np.float32)
        flags = np.asarray(t["flags"], dtype=np.int64)
        mask = t.get("catMask")
        mask = None if mask is None or len(mask) == 0 else np.asarray(mask, dtype=np.uint64)
        cover = np.zeros(len(feat), dtype=np.float64)
        idx = np.arange(len(X))
        node = np.zeros(len(X), dtype=np.int64)
        while idx.size:
            np.add.at(cover, node, 1.0)
            f = feat[node]
            inner = f >= 0
            idx, node, f = idx[inner], node[inner], f[inner]
            if not idx.size:
                break
            v = X[idx, f]
            fl = flags[node]
            with np.errstate(invalid="ignore"):
                left = np.where(np.isnan(v), (fl & 1) != 0, v <= thr[node])
                if mask is not None:
                    cat = (fl & 2) != 0
                    if cat.any():
                        vc = v[cat]
                        r = np.rint(vc)
                        ok = np.isfinite(vc) & (r >= 0) & (r < data_bins)
                        code = np.where(ok, r, data_bins).astype(np.int64)
                        w = mask[node[cat] * 8 + code // 32]
                        left[cat] = ((w >> (code % 32).astype(np.uint64)) & 1) == 1
            node = 2 * node + 1 + (~left).astype(np.int64)
        t["cover"] = cover.astype(np.float32)
    return model


def _fmt_list(a: np.ndarray) -> str:
    # float32 values are written as the exact repr of their float64 value, so
    # any reader that parses to float64 and rounds to float32 recovers them.
    if a.dtype == np.float32:
        return "[" + ",".join(map(repr, a.astype(np.float64).tolist())) + "]"
    return "[" + ",".join(map(str, a.tolist())) + "]"


def model_to_json(model: dict) -> str:
    """Serialise a ModelFile dict (numpy arrays allowed) to JSON text."""
    parts = ['{"version":%d,"objective":%d,"numBins":%d,"baseScore":%s,"numFeatures":%d,'
             % (model["version"], model["objective"], model["numBins"],
                repr(float(np.float32(model["baseScore"]))), model["numFeatures"])]
    parts.append('"categorical":%s,' % json.dumps([int(c) for c in model["categorical"]]))
    if model.get("featureNames") is not None:
        parts.append('"featureNames":%s,' % json.dumps(model["featureNames"]))
    parts.append('"trees":[')
    for i, t in enumerate(model["trees"]):
        if i:
            parts.append(",")
        mask = t.get("catMask")
        cover = t.get("cover")
        parts.append('{"feature":%s,"threshold":%s,"leaf":%s,"flags":%s,"catMask":%s%s}' % (
            _fmt_list(np.asarray(t["feature"], dtype=np.int32)),
            _fmt_list(np.asarray(t["threshold"], dtype=np.float32)),
            _fmt_list(np.asarray(t["leaf"], dtype=np.float32)),
            _fmt_list(np.asarray(t["flags"], dtype=np.uint8)),
            "[]" if mask is None or len(mask) == 0 else _fmt_list(np.asarray(mask, np.uint32)),
            "" if cover is None else ',"cover":' + _fmt_list(np.asarray(cover, np.float32))))
    parts.append("]")
    if model.get("numClasses") is not None:
        parts.append(',"numClasses":%d' % model["numClasses"])
    if model.get("baseScores") is not None:
        parts.append(',"baseScores":[%s]' % ",".join(
            repr(float(np.float32(b))) for b in model["baseScores"]))
    parts.append("}")
    return "".join(parts)


def write_model(model: dict, path) -> str:
    text = model_to_json(model)
    with open(path, "w") as fh:
        fh.write(text)
    return str(path)
