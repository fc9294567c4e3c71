"""The oracle (oracle/mbref.c + oracle/oracle.py) pinned to the reference.

The golden fixtures were produced by the reference's own predictor
(python/macboost/_pyinfer.py PyModel) and classifier
(python/macboost/__init__.py predict_proba); see tests/golden/make_golden.py.
"""

import numpy as np
import pytest

from conftest import (O, assert_bitwise, golden_arrays, golden_names, golden_oracle_model)

CASES = golden_names()


def test_fixtures_present():
    assert {"edge_l2", "edge_binary", "edge_poisson", "edge_multiclass", "cfg1_small",
            "cfg2_small", "cfg3_small", "cfg4_small", "cfg5_small"} <= set(CASES)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("layout", ["row", "feature"])
def test_oracle_matches_reference(oracle_built, name, layout):
    g = golden_arrays(name)
    m = golden_oracle_model(name)
    X = g["X"] if layout == "row" else np.ascontiguousarray(g["X"].T)
    raw, leaf = O.predict_raw(m, X, layout=layout, want_leaf=True)
    assert_bitwise(raw, g["raw"], f"{name} raw margins")
    assert np.array_equal(leaf, g["leaf"].astype(np.int32)), f"{name} leaf indices"
    with np.errstate(over="ignore"):
        assert_bitwise(O.predict(m, raw), g["pred"], f"{name} predict")
    proba = O.predict_proba(raw if m.num_classes > 1 else raw[:, 0])
    assert np.array_equal(proba, g["proba"]), f"{name} predict_proba"


@pytest.mark.parametrize("nthreads", [1, 3, 8])
def test_oracle_thread_split_invariant(oracle_built, nthreads):
    g = golden_arrays("cfg2_small")
    m = golden_oracle_model("cfg2_small")
    raw = O.predict_raw(m, g["X"], nthreads=nthreads)
    assert_bitwise(raw, g["raw"], "thread split")


def test_oracle_detects_planted_mistake(oracle_built):
    """A wrong oracle must fail the comparison: flip one threshold on the CPU."""
    g = golden_arrays("cfg1_small")
    m = golden_oracle_model("cfg1_small")
    internal = np.nonzero(m.feature >= 0)[0]
    m.threshold[internal[0]] = np.float32(-1.0)  # root of tree 0 now sends all right
    raw = O.predict_raw(m, g["X"])
    assert not np.array_equal(raw.view(np.uint32), g["raw"].view(np.uint32))


def test_ulp_distance():
    a = np.array([1.0, -0.0, 0.0, -1.0], dtype=np.float32)
    b = np.nextafter(a, np.float32(np.inf))
    assert list(O.ulp_distance(a, b)) == [1, 1, 1, 1]
    assert O.ulp_distance(np.float32([0.0]), np.float32([-0.0]))[0] == 0
