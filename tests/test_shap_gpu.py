"""GPU TreeSHAP contributions (macboost_predict_contrib) against the oracle.

Bar: every contribution and expected value within max(2 ulp fp32, 1e-9) of
the float64 oracle (oracle/mbshap.c, the recursive TreeSHAP of
Sources/MacBoost/SHAP.swift:170-326) rounded to float32.  The kernel also
computes in float64 but by a different summation (leaf paths instead of
recursion), so results differ from the oracle only in the last bit of
float32 or by float64 rounding on values that cancel to nearly zero.  The
reference's own GPU-vs-CPU test allows 5e-3 (ObjectiveTests.swift:457-459).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import O
from macboost_b200 import synth
from test_shap_oracle import tiny_model

pytestmark = pytest.mark.gpu
ATOL = 1e-9


def assert_contrib_close(got, want, what):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, what
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    ulp = np.spacing(np.abs(want)).astype(np.float64)
    bad = ~((d <= 2 * ulp) | (d <= ATOL))
    assert not bad.any(), (f"{what}: {int(bad.sum())} values off; worst {d.max():.3e} at "
                           f"{np.unravel_index(int(np.argmax(np.where(bad, d, 0))), d.shape)}")
    return float(np.mean(got.view(np.uint32) == want.view(np.uint32)))


def covered(cfg, trees, seed=17, sample=4000):
    m = synth.make_model(cfg, trees=trees)
    synth.add_covers(m, synth.make_data(cfg, rows=sample, seed=seed, layout="row"))
    text = synth.model_to_json(m)
    return text, O.model_from_dict(json.loads(text))


CASES = {"cfg1": (100, 1500), "cfg2": (100, 3000), "cfg3": (100, 1500), "cfg4": (300, 300),
         "cfg5": (60, 300)}


@pytest.mark.parametrize("cfg", sorted(CASES))
def test_contrib_vs_oracle(gpu, oracle_built, cfg):
    core = gpu
    trees, rows = CASES[cfg]
    text, om = covered(cfg, trees)
    h = core.load_json(text)
    X = synth.make_data(cfg, rows=rows, row_start=321, layout="row")
    want = O.predict_contrib(om, X)
    got = core.predict_contrib_ex(h, X, layout="row", devices=[0])
    exact = assert_contrib_close(got, want, cfg)
    assert exact > 0.95, f"{cfg}: only {exact:.3f} of values bit-identical"
    # local accuracy against the engine's own margins
    K, F = om.num_classes, om.num_features
    raw = core.predict_ex(h, X, kind=core.KIND_RAW)
    s = got.reshape(rows, K, F + 1).astype(np.float64).sum(axis=2)
    np.testing.assert_allclose(s, raw, atol=3e-5, err_msg=f"{cfg} local accuracy")


@pytest.mark.parametrize("seed,K", [(1, 1), (3, 3), (6, 1)])
def test_contrib_tiny_models_vs_definition(gpu, oracle_built, seed, K):
    """Repeated features on a path, categorical splits, NaNs, a zero-cover
    leaf, a tree without covers: against the oracle and the Shapley definition."""
    core = gpu
    m, X = tiny_model(seed, K=K, zero_cover_leaf=True)
    if seed == 6:
        m["trees"][1]["cover"] = None
    text = synth.model_to_json(m)
    om = O.model_from_dict(json.loads(text))
    h = core.load_json(text)
    got = core.predict_contrib_ex(h, X, devices=[0])
    assert_contrib_close(got, O.predict_contrib(om, X), f"tiny seed={seed}")
    F = om.num_features
    for i in range(0, 40, 7):
        want = O.shapley_bruteforce(om, X[i])
        np.testing.assert_allclose(got[i].reshape(K, F + 1), want, rtol=2e-6, atol=2e-7)


def test_reference_signature_layouts_and_repeatability(gpu, oracle_built):
    """macboost_predict_contrib (feature-major, the reference binding's call)
    equals the row-major form bit for bit, and runs repeat bit for bit."""
    core = gpu
    text, om = covered("cfg3", 50)
    h = core.load_json(text)
    X = synth.make_data("cfg3", rows=2049, row_start=5, layout="row")
    a = core.predict_contrib(h, X)
    b = core.predict_contrib_ex(h, X, layout="row")
    c = core.predict_contrib_ex(h, np.ascontiguousarray(X.T), layout="feature")
    d = core.predict_contrib(h, X)
    for other, what in ((b, "row-major"), (c, "feature-major ex"), (d, "repeat")):
        assert np.array_equal(a.view(np.uint32), other.view(np.uint32)), what


@pytest.mark.parametrize("rows", [1, 31, 127, 129, 1000])
def test_contrib_ragged_rows(gpu, oracle_built, rows):
    core = gpu
    text, om = covered("cfg2", 30)
    h = core.load_json(text)
    X = synth.make_data("cfg2", rows=rows, row_start=77, layout="row")
    assert_contrib_close(core.predict_contrib_ex(h, X), O.predict_contrib(om, X), f"rows={rows}")


def test_contrib_without_covers_is_bias_only(gpu):
    core = gpu
    m = synth.make_model("cfg1", trees=10)
    h = core.load_json(synth.model_to_json(m))
    X = synth.make_data("cfg1", rows=100, layout="row")
    out = core.predict_contrib(h, X)
    assert np.all(out[:, :-1] == 0) and np.all(out[:, -1] == np.float32(m["baseScores"][0]))


def test_contrib_wide_model_global_accumulators(gpu, oracle_built):
    """Too many features for shared-memory accumulators: the kernel keeps
    them in global memory; same results."""
    core = gpu
    F = 900
    rng = np.random.default_rng(12)
    tl = [synth._complete_tree(rng, 6, F, synth.EDGES_256, 0.05) for _ in range(40)]
    m = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.0, "numFeatures": F,
         "categorical": [], "trees": tl, "numClasses": 1, "baseScores": [0.0]}
    Xs = rng.random((3000, F)).astype(np.float32)
    synth.add_covers(m, Xs)
    text = synth.model_to_json(m)
    om = O.model_from_dict(json.loads(text))
    h = core.load_json(text)
    X = rng.random((700, F)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    assert_contrib_close(core.predict_contrib_ex(h, X), O.predict_contrib(om, X), "wide")


def test_contrib_multi_device(gpu, oracle_built):
    core = gpu
    n = core.device_count()
    text, om = covered("cfg2", 40)
    h = core.load_json(text)
    X = synth.make_data("cfg2", rows=3001, layout="row")
    one = core.predict_contrib_ex(h, X, devices=[0])
    many = core.predict_contrib_ex(h, X, devices=list(range(min(n, 4))))
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))


def test_contrib_device_entry_point(gpu, oracle_built):
    """macboost_predict_contrib_device on device buffers (feature-major with a
    padded stride, and row-major) equals the host-memory call bit for bit."""
    core = gpu
    from test_gpu_parity import _cudart
    cu = _cudart()
    text, om = covered("cfg3", 40)
    h = core.load_json(text)
    rows, F = 3001, om.num_features
    X = synth.make_data("cfg3", rows=rows, row_start=9, layout="row")
    want = core.predict_contrib_ex(h, X)
    W = want.shape[1]
    ld = 3008
    fm = np.zeros((F, ld), np.float32)
    fm[:, :rows] = X.T
    for src, layout, stride in ((fm, core.LAYOUT_FEATURE_MAJOR, ld),
                                (np.ascontiguousarray(X), core.LAYOUT_ROW_MAJOR, F)):
        dx = cu.alloc(src.nbytes)
        dout = cu.alloc(rows * W * 4)
        try:
            cu.h2d(dx, src)
            core.predict_contrib_device(h, 0, dx, rows, F, stride, dout, layout=layout)
            core.check_device(h, 0)
            got = cu.d2h(dout, rows * W, np.float32).reshape(rows, W)
        finally:
            cu.free(dx)
            cu.free(dout)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"layout {layout}"


def test_estimator_predict_contrib(gpu, oracle_built, tmp_path):
    """MacBoostRegressor.predict_contrib equals the reference-signature call."""
    core = gpu
    from macboost_b200 import MacBoostRegressor
    text, om = covered("cfg1", 20)
    p = tmp_path / "m.json"
    p.write_text(text)
    m = MacBoostRegressor.load_model(p, devices=[0])
    X = synth.make_data("cfg1", rows=500, row_start=3, layout="row")
    got = m.predict_contrib(X)
    want = core.predict_contrib(core.load(p), X)
    assert got.shape == (500, om.num_features + 1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("seed", range(10))
def test_contrib_random_models(gpu, oracle_built, seed):
    """Random models of the predict fuzz test (categorical masks, NaN, +-Inf,
    root-is-leaf trees, 1-5 classes) with covers from routed rows."""
    core = gpu
    from test_fuzz_gpu import random_model, random_rows
    model, rng = random_model(5000 + seed)
    synth.add_covers(model, random_rows(rng, model, 2000))
    text = synth.model_to_json(model)
    om = O.model_from_dict(json.loads(text))
    X = random_rows(rng, model, 700)
    got = core.predict_contrib_ex(core.load_json(text), X)
    assert_contrib_close(got, O.predict_contrib(om, X), f"seed {seed}")


def test_contrib_deep_paths_generic_kernel(gpu, oracle_built):
    """Leaf-wise trees deeper than 12 (paths through more than 12 distinct
    features) run the kernel's generic run-time-U path."""
    core = gpu
    rng = np.random.default_rng(77)
    F = 40
    tl = [synth._leafwise_tree(rng, 200, 16, F, synth.EDGES_256, 0.1) for _ in range(12)]
    m = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.0, "numFeatures": F,
         "categorical": [], "trees": tl, "numClasses": 1, "baseScores": [0.0]}
    Xs = rng.random((4000, F)).astype(np.float32)
    synth.add_covers(m, Xs)
    text = synth.model_to_json(m)
    om = O.model_from_dict(json.loads(text))
    depth = max(int(np.log2(len(t["feature"]) + 1)) - 1 for t in tl)
    assert depth == 16
    X = rng.random((900, F)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    got = core.predict_contrib_ex(core.load_json(text), X)
    assert_contrib_close(got, O.predict_contrib(om, X), "deep")
