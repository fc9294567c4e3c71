"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a checkout that has the MacBoost reference sources next to it:

    python tests/golden/make_golden.py /path/to/macboost

It imports the reference's own Python predictor (``python/macboost/_pyinfer.py``
``PyModel``) and classifier (``python/macboost/__init__.py``
``MacBoostClassifier.predict_proba``, pure-Python backend) and records, for
each model / input pair:

* ``raw``   -- ``PyModel.predict_raw(X)``   (fp32 margins, reference order)
* ``pred``  -- ``PyModel.predict(X)``       (exp for poisson / tweedie)
* ``leaf``  -- final heap index per (row, tree), from a loop that is the
               reference's level-synchronous walk (_pyinfer.py:62-70) with the
               node kept per tree and routing by ``PyModel._goes_left_at``
* ``proba`` -- ``MacBoostClassifier.predict_proba(X)`` (float64)

The fixtures are committed; the tests read them and never need the reference.
"""

from __future__ import annotations

import gzip
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from macboost_b200 import synth  # noqa: E402

F32 = np.float32


def leaf_indices(pm, X):
    """Heap index reached in every tree: _pyinfer.py:62-70 keeping `node`."""
    n = X.shape[0]
    out = np.empty((n, pm.num_trees), dtype=np.int32)
    for t, tree in enumerate(pm.trees):
        node = np.zeros(n, dtype=np.int64)
        active = tree["feature"][node] >= 0
        while active.any():
            idx = np.nonzero(active)[0]
            cur = node[idx]
            v = X[idx, tree["feature"][cur]]
            left = pm._goes_left_at(tree, cur, v)
            node[idx] = 2 * cur + 1 + (~left).astype(np.int64)
            active[idx] = tree["feature"][node[idx]] >= 0
        out[:, t] = node
    return out


def tree(feature, threshold, leaf, flags, catmask=None):
    n = len(feature)
    assert len(threshold) == n and len(leaf) == n and len(flags) == n
    return {"feature": np.asarray(feature, np.int32),
            "threshold": np.asarray(threshold, np.float64).astype(F32),
            "leaf": np.asarray(leaf, np.float64).astype(F32),
            "flags": np.asarray(flags, np.uint8),
            "catMask": None if catmask is None else np.asarray(catmask, np.uint32)}


def mask_words(bits, fill_high=None):
    w = np.zeros(8, dtype=np.uint64)
    for b in bits:
        w[b // 32] |= np.uint64(1) << np.uint64(b % 32)
    if fill_high is not None:
        w[1:] = 0xFFFFFFFF if fill_high else 0
    return w.astype(np.uint32)


def edge_model(objective=0, K=1, base=None):
    """Hand-built trees that pin each routing rule of the reference walk."""
    tiny = float(np.float32(1e-40))           # a denormal threshold
    T = []
    # A: complete depth 2; root x0 <= 0.5 (NaN left), x1 <= 0 (NaN right),
    #    x2 <= -1.5 (NaN left)
    T.append(tree([0, 1, 2, -1, -1, -1, -1], [0.5, 0.0, -1.5, 0, 0, 0, 0],
                  [0, 0, 0, 1.0, 2.0, 3.0, 4.0], [1, 0, 1, 0, 0, 0, 0]))
    # B: root is a leaf
    T.append(tree([-1], [0.0], [0.25], [0]))
    # C: categorical on x3, 32-bit subset {0, 2, 5, 31}, codes >= 32 and the
    #    missing bin follow bit 255 (set): a compressible mask
    n = 3
    cm = np.zeros(8 * n, np.uint32)
    cm[0:8] = mask_words([0, 2, 5, 31], fill_high=True)
    T.append(tree([3, -1, -1], [0, 0, 0], [0, -8.0, 8.0], [2, 0, 0], cm))
    # D: denormal threshold on x0 and an unbalanced right spine on x1
    T.append(tree([0, -1, 1, -1, -1, -1, 2] + [-1] * 8,
                  [tiny, 0, 2.0, 0, 0, 0, 0.5] + [0] * 8,
                  [0, 16.0, 0, 0, 0, 32.0, 0] + [0, 0, 0, 0, 0, 0, 64.0, 128.0],
                  [0, 0, 1, 0, 0, 0, 0] + [0] * 8))
    # E: categorical on x3 with a mask that is NOT uniform above bit 31
    #    (codes 40 and 254 go left, 255 = missing goes right)
    cm = np.zeros(8 * 3, np.uint32)
    cm[0:8] = mask_words([1, 3, 40, 254])
    T.append(tree([3, -1, -1], [0, 0, 0], [0, 0.5, -0.5], [3, 0, 0], cm))
    # F: node flagged categorical in a tree without catMask -> numeric routing
    T.append(tree([2, -1, -1], [0.0, 0, 0], [0, -0.125, 0.125], [2, 0, 0]))
    # G: threshold exactly representable ties (v == thr goes left), -0.0
    T.append(tree([1, 0, -1, -1, -1], [-0.0, 0.75, 0, 0, 0], [0, 0, 1e-3, 2e-3, 3e-3],
                  [0, 0, 0, 0, 0]))
    # H: huge / infinite thresholds never occur in files (JSON cannot hold
    #    them); use the largest finite float instead
    T.append(tree([2, -1, -1], [float(np.finfo(F32).max), 0, 0], [0, 0.0625, -0.0625],
                  [0, 0, 0]))
    # pad the forest so multiclass variants see several trees per class
    T = T * 2 if K > 1 else T
    if base is None:
        base = [0.0] * K
    return {"version": 1, "objective": objective, "numBins": 256,
            "baseScore": base[0], "numFeatures": 4, "categorical": [3],
            "trees": T, "numClasses": K, "baseScores": base}


def edge_inputs(seed=7):
    """Rows that hit every rule above, plus seeded random rows with specials."""
    nan, inf = np.nan, np.inf
    den = float(np.float32(1e-45))
    rows = [
        [0.5, 0.0, -1.5, 0.0], [0.5000001, -0.0, -1.5, 2.0], [nan, nan, nan, nan],
        [-inf, inf, -inf, inf], [inf, -inf, inf, -inf], [den, 1.0, 0.0, 5.0],
        [-den, -1.0, 0.0, 31.0], [0.0, 2.0, 3.0, -0.5], [1e-40, 0.75, 0.5, -0.6],
        [float(np.float32(1e-40)), 0.0, 0.5, 2.5], [2.0, 0.5, 0.5, 3.5], [0.25, 0.25, 0, 254.5],
        [0.1, 0.9, 0.1, 255.0], [0.1, 0.9, 0.1, 1e9], [0.1, 0.9, 0.1, 40.0],
        [0.1, 0.9, 0.1, 254.0], [0.1, 0.9, 0.1, 253.5], [0.1, 0.9, 0.1, 32.0],
        [0.1, 0.9, 0.1, 0.5], [0.1, 0.9, 0.1, 1.5], [0.1, 0.9, 0.1, -1.0],
        [0.1, 0.9, float(np.finfo(F32).max), 3e38], [0.1, 0.9, -0.0, 1e30],
        [0.1, 0.9, 0.0, -1e30],
    ]
    rng = np.random.default_rng(seed)
    r = rng.uniform(-3, 3, (488, 4)).astype(F32)
    r[:, 3] = rng.integers(-3, 300, 488).astype(F32) + rng.choice(
        [0.0, 0.5, -0.5, 0.25], 488).astype(F32)
    special = rng.choice([nan, inf, -inf, den, -den, 0.0, -0.0, 0.5], size=r.shape)
    pick = rng.random(r.shape) < 0.15
    r[pick] = special[pick]
    return np.vstack([np.asarray(rows, dtype=F32), r]).astype(F32)


CASES = {
    # name: (model builder, input builder)
    "edge_l2": (lambda: edge_model(0, 1), edge_inputs),
    "edge_binary": (lambda: edge_model(1, 1, [float(F32(-0.3))]), edge_inputs),
    "edge_poisson": (lambda: edge_model(5, 1, [float(F32(0.125))]), edge_inputs),
    "edge_multiclass": (lambda: edge_model(7, 3, [0.5, -0.25, 1.0]), edge_inputs),
    "cfg1_small": (lambda: synth.make_model("cfg1", trees=100),
                   lambda: synth.make_data("cfg1", rows=512, layout="row", seed=11)),
    "cfg2_small": (lambda: synth.make_model("cfg2", trees=100),
                   lambda: synth.make_data("cfg2", rows=1024, layout="row", seed=12)),
    "cfg3_small": (lambda: synth.make_model("cfg3", trees=100),
                   lambda: synth.make_data("cfg3", rows=512, layout="row", seed=13)),
    "cfg4_small": (lambda: synth.make_model("cfg4", trees=200),
                   lambda: synth.make_data("cfg4", rows=512, layout="row", seed=14)),
    "cfg5_small": (lambda: synth.make_model("cfg5", trees=6),
                   lambda: synth.make_data("cfg5", rows=512, layout="row", seed=15)),
}


def main(ref_root: str):
    sys.path.insert(0, str(Path(ref_root) / "python"))
    os.environ["MACBOOST_FORCE_PYTHON"] = "1"
    from macboost import MacBoostClassifier          # reference package
    from macboost._pyinfer import PyModel            # reference predictor

    for name, (mk_model, mk_x) in CASES.items():
        model = mk_model()
        X = np.ascontiguousarray(mk_x(), dtype=F32)
        text = synth.model_to_json(model)
        mpath = HERE / f"{name}.model.json.gz"
        with gzip.open(mpath, "wt") as fh:
            fh.write(text)
        tmp = HERE / f".{name}.tmp.json"
        tmp.write_text(text)
        try:
            pm = PyModel(str(tmp))
            raw = np.asarray(pm.predict_raw(X), dtype=F32).reshape(X.shape[0], -1)
            pred = np.asarray(pm.predict(X), dtype=F32).reshape(X.shape[0], -1)
            leaf = leaf_indices(pm, X)
            clf = MacBoostClassifier.load_model(str(tmp))
            proba = np.asarray(clf.predict_proba(X), dtype=np.float64)
        finally:
            tmp.unlink()
        np.savez_compressed(HERE / f"{name}.npz", X=X, raw=raw, pred=pred,
                            leaf=leaf.astype(np.int16 if leaf.max() < 32767 else np.int32),
                            proba=proba)
        print(f"{name}: X{X.shape} raw{raw.shape} leaf{leaf.shape} "
              f"proba{proba.shape} trees={pm.num_trees} K={pm.num_classes}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <macboost source root>")
    main(sys.argv[1])
