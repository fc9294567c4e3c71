"""TreeSHAP oracle on the CPU: the recursive restatement (oracle/mbshap.c,
Sources/MacBoost/SHAP.swift:170-326) pinned to exact Shapley values computed
from their definition, the local-accuracy property the reference's tests use
(Tests/MacBoostTests/ObjectiveTests.swift:400-425), and the library's checks
on cover arrays (no GPU needed)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import O
from macboost_b200 import synth


def tiny_model(seed: int, K: int = 1, F: int = 5, depth: int = 4, trees: int = 4,
               zero_cover_leaf: bool = False):
    """Complete trees over few features (so paths repeat features), one
    categorical feature, NaNs in the data, covers from routing the data."""
    rng = np.random.default_rng(seed)
    tl = [synth._complete_tree(rng, depth, F, synth.EDGES_256, 0.3, frozenset({F - 1}),
                               with_mask=True) for _ in range(trees * K)]
    m = {"version": 1, "objective": 7 if K > 1 else 0, "numBins": 256,
         "baseScore": 0.25, "numFeatures": F, "categorical": [F - 1], "trees": tl,
         "numClasses": K, "baseScores": [0.25 + 0.5 * k for k in range(K)]}
    X = rng.random((600, F)).astype(np.float32)
    X[:, F - 1] = rng.integers(0, 32, 600)
    X[rng.random((600, F)) < 0.1] = np.nan
    synth.add_covers(m, X)
    if zero_cover_leaf:   # a leaf no training row reached
        m["trees"][0]["cover"][(1 << depth) - 1] = 0.0
    return m, X


@pytest.mark.parametrize("seed,K", [(1, 1), (2, 1), (3, 3)])
def test_oracle_matches_shapley_definition(oracle_built, seed, K):
    m, X = tiny_model(seed, K=K)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    F = om.num_features
    got = O.predict_contrib(om, X[:25]).reshape(25, K, F + 1)
    for i in range(25):
        want = O.shapley_bruteforce(om, X[i])
        np.testing.assert_allclose(got[i], want, rtol=2e-6, atol=2e-7, err_msg=f"row {i}")


def test_local_accuracy(oracle_built):
    """Per class, contributions + expected value == the raw margin."""
    for cfg, trees, rows in (("cfg2", 40, 300), ("cfg3", 30, 300), ("cfg4", 60, 100),
                             ("cfg5", 10, 100)):
        m = synth.make_model(cfg, trees=trees)
        synth.add_covers(m, synth.make_data(cfg, rows=2000, seed=17, layout="row"))
        om = O.model_from_dict(json.loads(synth.model_to_json(m)))
        X = synth.make_data(cfg, rows=rows, seed=3, layout="row")
        K, F = om.num_classes, om.num_features
        c = O.predict_contrib(om, X).reshape(rows, K, F + 1).astype(np.float64)
        raw = O.predict_raw(om, X).astype(np.float64)
        np.testing.assert_allclose(c.sum(axis=2), raw, atol=2e-5, err_msg=cfg)


def test_uncovered_trees_and_zero_covers(oracle_built):
    """Trees with an empty cover array take no part; a zero-cover node gives
    zero fractions below it (SHAP.swift:241-242)."""
    m, X = tiny_model(4, zero_cover_leaf=True)
    m["trees"][1]["cover"] = None            # written without a cover array
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    assert list(om.has_cover) == [1, 0, 1, 1]
    got = O.predict_contrib(om, X[:10])
    for i in range(10):
        want = O.shapley_bruteforce(om, X[i])
        np.testing.assert_allclose(got[i], want[0], rtol=2e-6, atol=2e-7)


def test_cover_length_is_checked(lib_built):
    core = lib_built
    m, X = tiny_model(5)
    m["trees"][2]["cover"] = np.ones(7, np.float32)
    h = core.load_json(synth.model_to_json(m))
    with pytest.raises(core.MacBoostError, match="tree 2 has 7 cover values for 31 nodes"):
        core.predict_contrib(h, X[:4])
    with pytest.raises(ValueError, match="cover values"):
        O.model_from_dict(json.loads(synth.model_to_json(m)))
