"""Randomised parity: seeded random MacBoost models and rows, through every
kernel family the planner can pick, against the oracle (leaf indices and raw
margins bit for bit, transforms within 2 ulp).

Models vary what the benchmark configs hold fixed: class count, numBins,
complete depths 0-8 and leaf-wise trees to depth 12, root-is-leaf trees,
categorical masks (full and 32-bit), default directions; thresholds include
values the rows hit exactly, +-0.0, denormals and large magnitudes; rows include
NaN, +-Inf, +-0.0, denormals and categorical ids outside the code range.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import O, assert_bitwise, assert_ulp
from macboost_b200 import synth

pytestmark = pytest.mark.gpu

PLANS = ["", "codes=0", "codes=0,planes=0", "codes=1", "codes=0,top=1",
         "codes=0,planes=0,top=1", "codes=0,planes=0,pay=0"]
SPECIAL = np.float32([0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38, 0.5, -0.5, 1.0])


def _thresholds(rng, n):
    t = rng.standard_normal(n).astype(np.float32)
    pick = rng.random(n)
    t = np.where(pick < 0.15, SPECIAL[rng.integers(0, len(SPECIAL), n)], t)
    with np.errstate(over="ignore"):     # the discarded branch may overflow
        t = np.where((pick > 0.15) & (pick < 0.3), np.round(t * 4) / 4, t)   # values rows hit
    return t.astype(np.float32)


def _tree(rng, F, cats, nb, leafwise):
    depth = int(rng.integers(0, 9)) if not leafwise else 12
    n_nodes = (1 << (depth + 1)) - 1
    feat = np.full(n_nodes, -1, np.int32)
    flags = np.zeros(n_nodes, np.uint8)
    thr = np.zeros(n_nodes, np.float32)
    mask = np.zeros(n_nodes * 8, np.uint32)
    use_mask = bool(cats) and rng.random() < 0.8
    if leafwise:
        leaves, dep = [0], {0: 0}
        for _ in range(int(rng.integers(1, 60))):
            cand = [i for i, n in enumerate(leaves) if dep[n] < depth]
            if not cand:
                break
            n = leaves.pop(cand[int(rng.integers(0, len(cand)))])
            feat[n] = -2                                  # marked internal
            for ch in (2 * n + 1, 2 * n + 2):
                dep[ch] = dep[n] + 1
                leaves.append(ch)
        internal = np.nonzero(feat == -2)[0]
    else:
        internal = np.arange((1 << depth) - 1)
    for n in internal:
        f = int(rng.integers(0, F))
        feat[n] = f
        dl = int(rng.integers(0, 2))
        if f in cats and use_mask:
            flags[n] = 2 | dl
            w = rng.integers(0, 2**32, 8, dtype=np.uint64).astype(np.uint32)
            if rng.random() < 0.5:
                w[1:] = 0xFFFFFFFF if dl else 0           # a 32-bit mask
            mask[n * 8:(n + 1) * 8] = w
        else:
            flags[n] = dl
            thr[n] = _thresholds(rng, 1)[0]
    leaf = (rng.standard_normal(n_nodes) * 0.3).astype(np.float32)
    leaf[rng.random(n_nodes) < 0.05] = np.float32(-0.0)
    return {"feature": feat, "threshold": thr, "leaf": leaf, "flags": flags,
            "catMask": mask if use_mask else None}


def random_model(seed):
    rng = np.random.default_rng(seed)
    F = int(rng.integers(1, 41))
    K = int(rng.choice([1, 1, 2, 3, 5]))
    nb = int(rng.choice([4, 16, 64, 256]))
    cats = set(int(c) for c in rng.choice(F, size=int(rng.integers(0, min(F, 4) + 1)),
                                           replace=False)) if F > 1 else set()
    objective = 7 if K > 2 else int(rng.choice([0, 1, 5]))
    leafwise = rng.random() < 0.35
    T = K * int(rng.integers(1, 25))
    trees = [_tree(rng, F, cats, nb, leafwise and rng.random() < 0.8) for _ in range(T)]
    base = [float(np.float32(b)) for b in rng.standard_normal(K) * 0.1]
    return {"version": 1, "objective": objective, "numBins": nb, "baseScore": base[0],
            "numFeatures": F, "categorical": sorted(cats), "trees": trees,
            "numClasses": K, "baseScores": base}, rng


def random_rows(rng, model, n):
    F = model["numFeatures"]
    X = (rng.standard_normal((n, F)) * 1.5).astype(np.float32)
    X = np.where(rng.random((n, F)) < 0.1, np.round(X * 4) / 4, X).astype(np.float32)
    sp = rng.random((n, F))
    X[sp < 0.04] = np.nan
    X[(sp >= 0.04) & (sp < 0.05)] = np.inf
    X[(sp >= 0.05) & (sp < 0.06)] = -np.inf
    X[(sp >= 0.06) & (sp < 0.08)] = SPECIAL[rng.integers(0, len(SPECIAL), 1)][0]
    for c in model["categorical"]:
        ids = rng.integers(-3, model["numBins"] + 5, n).astype(np.float32)
        ids[rng.random(n) < 0.1] += np.float32(0.5)     # halves: round to even
        ids[rng.random(n) < 0.05] = np.nan
        X[:, c] = ids
    if rng.random() < 0.3:                              # some inputs without NaN
        X = np.where(np.isnan(X), np.float32(0.0), X)
    return X


@pytest.mark.parametrize("seed", range(24))
def test_random_models_every_plan(gpu, oracle_built, seed, monkeypatch):
    core = gpu
    model, rng = random_model(1000 + seed)
    text = synth.model_to_json(model)
    om = O.model_from_dict(json.loads(text))
    X = random_rows(rng, model, int(rng.integers(1, 3000)))
    raw_o, leaf_o = O.predict_raw(om, X, want_leaf=True)
    ran = 0
    for plan in PLANS:
        monkeypatch.setenv("MACBOOST_PLAN", plan)
        try:
            h = core.load_json(text)
        except core.MacBoostError as e:
            if "not applicable" in str(e):
                continue
            raise
        ran += 1
        assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), raw_o, f"seed {seed} {plan!r}")
        assert np.array_equal(core.predict_ex(h, X, kind=core.KIND_LEAF), leaf_o), \
            f"seed {seed} {plan!r} leaf"
    assert ran >= 3
    monkeypatch.delenv("MACBOOST_PLAN")
    h = core.load_json(text)
    with np.errstate(over="ignore", invalid="ignore"):
        want_p = O.predict(om, raw_o)
        want_cli = O.predict_cli(om, raw_o)
        want_proba = O.predict_proba(raw_o if om.num_classes > 1 else raw_o[:, 0])
    assert_ulp(core.predict_ex(h, X, kind=core.KIND_PREDICT), want_p, 2, f"seed {seed} predict")
    assert_ulp(core.predict_ex(h, X, kind=core.KIND_CLI), want_cli, 2, f"seed {seed} cli")
    assert_ulp(core.predict_ex(h, X, kind=core.KIND_PROBA), want_proba.astype(np.float32), 2,
               f"seed {seed} proba")
