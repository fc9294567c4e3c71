"""Binned data on the CPU: the .mbds reader against files written by the
oracle's restatement of BinnedDataset.save (Sources/MacBoost/Dataset.swift:
26-39), its error messages, and the binned oracle (oracle/mbbinned.c,
Shaders.swift:37-76 and 1741-1781) pinned to the float predictor oracle:
binning rows and walking the model's trees in split form gives the float
predictor's margins bit for bit."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from conftest import O, assert_bitwise
from macboost_b200 import synth

NUM_BINS = 64


def binned_model(seed=0, F=20, trees=30, depth=5, K=1, cats=(18, 19), num_bins=NUM_BINS):
    """A model whose numeric thresholds are the dataset's bin edges, plus the
    rows and edges of that dataset."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((3000, F)).astype(np.float32)
    for c in cats:
        X[:, c] = rng.integers(0, min(32, num_bins - 1), len(X))
    X[rng.random(X.shape) < 0.07] = np.nan
    E = O.compute_edges(X, num_bins, cats).reshape(F, num_bins - 2)
    thr = [E[f] for f in range(F)]
    tl = [synth._complete_tree(rng, depth, F, thr, 0.1, frozenset(cats), with_mask=True)
          for _ in range(trees * K)]
    m = {"version": 1, "objective": 7 if K > 1 else 1, "numBins": num_bins, "baseScore": 0.0,
         "numFeatures": F, "categorical": sorted(cats), "trees": tl, "numClasses": K,
         "baseScores": [0.05 * k for k in range(K)]}
    return m, X, E


@pytest.mark.parametrize("K", [1, 3])
def test_binned_oracle_equals_float_oracle(oracle_built, K):
    m, X, E = binned_model(seed=K, K=K)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    cats = m["categorical"]
    bins = O.bin_data(X, E, NUM_BINS, cats)
    sf = O.split_form(om, E, NUM_BINS)
    rows = len(X)
    preds = np.tile(np.asarray(m["baseScores"], np.float32)[:, None], (1, rows)).copy()
    leaf = O.predict_binned(bins, rows, NUM_BINS, sf, max_depth=6, K=K, preds=preds,
                            want_leaf=True)
    raw, raw_leaf = O.predict_raw(om, X, want_leaf=True)
    assert_bitwise(preds.T, raw, "binned margins vs float margins")
    assert np.array_equal(leaf.T, raw_leaf)


def test_bin_data_oracle_rules(oracle_built):
    """NaN -> missing bin, categorical clamp(rint), numeric first edge >= v."""
    E = np.array([[0.0, 1.0, 1.0, 2.0], [0, 0, 0, 0]], np.float32).reshape(2, 4)
    X = np.array([[np.nan, 3.6], [-5.0, -2.4], [0.0, 7.0], [1.0, 1e30], [1.5, -np.inf],
                  [2.0, np.inf], [9.0, 2.5]], np.float32)
    b = O.bin_data(X, E.ravel(), 6, [1]).reshape(1, len(X), 8)[0]
    assert b[:, 0].tolist() == [5, 0, 0, 1, 3, 3, 4]
    assert b[:, 1].tolist() == [4, 0, 4, 4, 0, 4, 2]
    assert not b[:, 2:].any()


def write_dataset(tmp_path, seed=3, rows=500, cols=13, num_bins=NUM_BINS, names=True):
    rng = np.random.default_rng(seed)
    bins = rng.integers(0, num_bins, ((cols + 7) // 8) * 8 * rows).astype(np.uint8)
    edges = np.sort(rng.random((cols, num_bins - 2)), axis=1).astype(np.float32)
    labels = rng.random(rows).astype(np.float32)
    fn = [f"feat é{i}" for i in range(cols)] if names else None
    p = tmp_path / "d.mbds"
    O.write_mbds(p, bins, rows, cols, num_bins, [5, 2], fn, edges, labels)
    return p, bins, edges, labels, fn


def test_mbds_reader(lib_built, tmp_path):
    core = lib_built
    p, bins, edges, labels, names = write_dataset(tmp_path)
    d = core.Dataset(p)
    assert (d.rows, d.cols, d.num_bins) == (500, 13, NUM_BINS)
    assert d.categorical == [2, 5]
    assert d.feature_names == names
    assert np.array_equal(d.bins, bins)
    assert np.array_equal(d.edges, edges.ravel())
    assert np.array_equal(d.labels, labels)
    p2, *_ = write_dataset(tmp_path, names=False)
    assert core.Dataset(p2).feature_names is None


def test_mbds_errors(lib_built, tmp_path):
    core = lib_built
    p, *_ = write_dataset(tmp_path)
    raw = p.read_bytes()
    cases = {
        "bad_magic": (b"XXXX" + raw[4:], "Invalid input: not a MacBoost dataset (.mbds) file"),
        "bad_version": (raw[:4] + struct.pack("<I", 2) + raw[8:],
                        "Invalid input: unsupported .mbds version"),
        "bad_tile": (raw[:8] + struct.pack("<I", 16) + raw[12:],
                     "Invalid input: .mbds tile width mismatch"),
        "truncated": (raw[:-10], "Invalid input: truncated .mbds file"),
        "empty": (b"", "Invalid input: truncated .mbds file"),
    }
    for name, (data, msg) in cases.items():
        q = tmp_path / f"{name}.mbds"
        q.write_bytes(data)
        with pytest.raises(core.MacBoostError) as ei:
            core.Dataset(q)
        assert str(ei.value) == msg, name
    # rows field one larger than the arrays: sizes inconsistent
    rows = struct.unpack_from("<Q", raw, 12)[0]
    q = tmp_path / "sizes.mbds"
    q.write_bytes(raw[:12] + struct.pack("<Q", rows + 1) + raw[20:])
    with pytest.raises(core.MacBoostError, match=r"^Invalid input: .mbds sizes are inconsistent$"):
        core.Dataset(q)
    with pytest.raises(core.MacBoostError, match="cannot read"):
        core.Dataset(tmp_path / "absent.mbds")


def test_split_form_needs_edge_thresholds(lib_built, tmp_path):
    """A model whose thresholds are not the dataset's edges is rejected before
    any device work (no GPU needed for the check)."""
    core = lib_built
    m, X, E = binned_model(seed=9)
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    p = tmp_path / "x.mbds"
    O.write_mbds(p, bins, len(X), X.shape[1], NUM_BINS, m["categorical"], None, E,
                 np.zeros(len(X), np.float32))
    d = core.Dataset(p)
    m["trees"][3]["threshold"][0] = np.float32(0.123456)
    h = core.load_json(synth.model_to_json(m))
    with pytest.raises(core.MacBoostError, match="is not one of the dataset's bin edges"):
        core.predict_dataset(h, d, core.KIND_RAW)
    m2 = dict(m, numBins=128)
    h2 = core.load_json(synth.model_to_json(m2))
    with pytest.raises(core.MacBoostError, match="numBins 128, the dataset has 64"):
        core.predict_dataset(h2, d, core.KIND_RAW)
