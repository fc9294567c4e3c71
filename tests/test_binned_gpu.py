"""Binned data on the GPU: bin_data and the binned tree walk
(predict_tree_binned / assign_leaves) bit for bit against the oracle
(oracle/mbbinned.c), and a model predicted on a .mbds dataset equal to the
float predictor on the rows the bins came from."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import O, assert_bitwise
from macboost_b200 import synth
from test_binned_cpu import NUM_BINS, binned_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", ["row", "feature"])
def test_bin_data_vs_oracle(gpu, oracle_built, layout):
    core = gpu
    rng = np.random.default_rng(4)
    rows, cols, nb = 20_011, 21, 256
    X = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    X[:, 3] = rng.integers(-5, 300, rows)               # categorical ids, some outside the range
    X[:, 4] = np.float32([1e30, -1e30, np.inf, -np.inf, 2.5, -0.4, 3.5, 7.49][0])
    X[::7, 4] = np.float32(-1e30)
    X[rng.random(X.shape) < 0.05] = np.nan
    X[::11, 9] = np.inf
    X[::13, 9] = -np.inf
    E = np.sort(rng.standard_normal((cols, nb - 2)) * 3, axis=1).astype(np.float32)
    E[5, 100:140] = E[5, 100]                            # repeated edges
    E[6] = rng.standard_normal(nb - 2).astype(np.float32)  # unsorted: the search is replayed verbatim
    cats = [3, 4]
    Xin = X if layout == "row" else np.ascontiguousarray(X.T)
    got = core.bin_data(Xin, E, nb, cats, layout=layout)
    want = O.bin_data(Xin, E, nb, cats, layout=layout)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("K,max_depth", [(1, 6), (3, 6), (1, 3)])
def test_tree_binned_vs_oracle(gpu, oracle_built, K, max_depth):
    core = gpu
    m, X, E = binned_model(seed=10 + K, K=K)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    sf = O.split_form(om, E, NUM_BINS)
    rows, cols = X.shape
    rng = np.random.default_rng(1)
    start = rng.standard_normal(K * rows).astype(np.float32)
    want = start.copy()
    want_leaf = O.predict_binned(bins, rows, NUM_BINS, sf, max_depth, K, want, want_leaf=True)
    got = start.copy()
    got_leaf = core.predict_tree_binned(bins, rows, cols, NUM_BINS, sf.tree_off, sf.feature,
                                        sf.bin, sf.flags, sf.catmask, sf.leaf, max_depth, K,
                                        preds=got, want_leaf=True)
    assert_bitwise(got, want, "class-major preds")
    assert np.array_equal(got_leaf, want_leaf)
    # one tree per call, as the trainer uses it, gives the same sums
    per = start.copy()
    T = len(sf.tree_off) - 1
    for t in range(T):
        a, b = int(sf.tree_off[t]), int(sf.tree_off[t + 1])
        part = per.reshape(K, rows)[t % K].copy()
        core.predict_tree_binned(bins, rows, cols, NUM_BINS, [0, b - a], sf.feature[a:b],
                                 sf.bin[a:b], sf.flags[a:b], sf.catmask[a * 8:b * 8],
                                 sf.leaf[a:b], max_depth, 1, preds=part)
        per.reshape(K, rows)[t % K] = part
    assert_bitwise(per, want, "tree by tree")


def test_tree_binned_rejects_bad_splits(gpu, oracle_built):
    core = gpu
    m, X, E = binned_model(seed=2)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    sf = O.split_form(om, E, NUM_BINS)
    rows, cols = X.shape
    feat = sf.feature.copy()
    feat[0] = cols + 5                                   # root names a missing feature
    with pytest.raises(core.MacBoostError, match="outside the bin matrix"):
        core.predict_tree_binned(bins, rows, cols, NUM_BINS, sf.tree_off, feat, sf.bin,
                                 sf.flags, sf.catmask, sf.leaf, 6, 1,
                                 preds=np.zeros(rows, np.float32))


@pytest.mark.parametrize("K", [1, 3])
def test_predict_dataset_equals_float_predict(gpu, oracle_built, tmp_path, K):
    core = gpu
    m, X, E = binned_model(seed=20 + K, K=K, trees=60)
    text = synth.model_to_json(m)
    om = O.model_from_dict(json.loads(text))
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    p = tmp_path / "x.mbds"
    O.write_mbds(p, bins, len(X), X.shape[1], NUM_BINS, m["categorical"], None, E,
                 np.zeros(len(X), np.float32))
    d = core.Dataset(p)
    h = core.load_json(text)
    assert_bitwise(core.predict_dataset(h, d, core.KIND_RAW), O.predict_raw(om, X), "raw")
    for kind in (core.KIND_PREDICT, core.KIND_PROBA, core.KIND_CLI):
        assert_bitwise(core.predict_dataset(h, d, kind), core.predict_ex(h, X, kind=kind),
                       f"kind {kind}")
    assert np.array_equal(core.predict_dataset(h, d, core.KIND_LEAF),
                          core.predict_ex(h, X, kind=core.KIND_LEAF))


def _split_arrays(sf):
    return [np.ascontiguousarray(sf.tree_off, np.int64), np.ascontiguousarray(sf.feature, np.int32),
            np.ascontiguousarray(sf.bin, np.uint32), np.ascontiguousarray(sf.flags, np.uint32),
            np.ascontiguousarray(sf.catmask, np.uint32), np.ascontiguousarray(sf.leaf, np.float32)]


@pytest.mark.parametrize("trees,depth", [(40, 5), (1, 10), (260, 5)])
def test_tree_binned_record_staging_and_fallback(gpu, oracle_built, trees, depth):
    """The walk stages a call's trees in shared memory when they fit and reads
    the split arrays otherwise: through the host call (all nodes counted: 40
    trees of 63 nodes staged, 260 trees, 16,380 nodes, too many) and the
    device call (8 KB of records: one 63-node tree staged per call, a 2,047-node
    tree too large), against the oracle, preds and leaf indices bit for bit."""
    core = gpu
    from test_gpu_parity import _cudart
    m, X, E = binned_model(seed=60 + depth, trees=trees, depth=depth)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    sf = O.split_form(om, E, NUM_BINS)
    rows, cols = X.shape
    start = np.random.default_rng(2).standard_normal(rows).astype(np.float32)
    want = start.copy()
    want_leaf = O.predict_binned(bins, rows, NUM_BINS, sf, depth, 1, want, want_leaf=True)
    got = start.copy()
    got_leaf = core.predict_tree_binned(bins, rows, cols, NUM_BINS, sf.tree_off, sf.feature,
                                        sf.bin, sf.flags, sf.catmask, sf.leaf, depth, 1,
                                        preds=got, want_leaf=True)
    assert_bitwise(got, want, "host call")
    assert np.array_equal(got_leaf, want_leaf)
    # the device entry point, one tree per call as a GPU trainer calls it
    cu = _cudart()
    T = len(sf.tree_off) - 1
    arrs = _split_arrays(sf)
    dbins = cu.alloc(bins.nbytes)
    dpreds = cu.alloc(rows * 4)
    dleaf = cu.alloc(rows * 4)
    dstatus = cu.alloc(4)
    dptrs = [cu.alloc(max(a.nbytes, 4)) for a in arrs]
    try:
        cu.h2d(dbins, np.ascontiguousarray(bins))
        cu.h2d(dpreds, start)
        cu.h2d(dstatus, np.zeros(1, np.uint32))
        for d, a in zip(dptrs, arrs):
            cu.h2d(d, a)
        leaves = []
        for t in range(min(T, 12)):
            a0, a1 = int(sf.tree_off[t]), int(sf.tree_off[t + 1])
            off = np.array([a0, a1], np.int64)
            doff = cu.alloc(16)
            try:
                cu.h2d(doff, off)
                core.predict_tree_binned_device(
                    dbins, rows, cols, NUM_BINS, 1, doff, dptrs[1], dptrs[2], dptrs[3], dptrs[4],
                    dptrs[5], depth, 1, 0, dpreds, dleaf, dstatus)
                leaves.append(cu.d2h(dleaf, rows, np.int32))
            finally:
                cu.free(doff)
        status = cu.d2h(dstatus, 1, np.uint32)[0]
        preds = cu.d2h(dpreds, rows, np.float32)
    finally:
        for d in [dbins, dpreds, dleaf, dstatus, *dptrs]:
            cu.free(d)
    assert status == 0
    n = min(T, 12)
    part = start.copy()
    part_leaf = O.predict_binned(bins, rows, NUM_BINS, O.SplitForest(
        tree_off=sf.tree_off[:n + 1], feature=sf.feature, bin=sf.bin, flags=sf.flags,
        catmask=sf.catmask, leaf=sf.leaf), depth, 1, part, want_leaf=True)
    assert_bitwise(preds, part, "device call, tree by tree")
    for t in range(n):
        assert np.array_equal(leaves[t], part_leaf[t]), f"tree {t} leaves"


def test_bin_data_device_entry_point(gpu, oracle_built):
    """macboost_bin_data_device on device buffers (feature-major with a padded
    stride, and row-major) equals the host call byte for byte."""
    core = gpu
    from test_gpu_parity import _cudart
    cu = _cudart()
    rng = np.random.default_rng(14)
    rows, cols, nb, ld = 5001, 19, 64, 5008
    X = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    X[:, 2] = rng.integers(-2, 70, rows)
    X[rng.random(X.shape) < 0.05] = np.nan
    E = np.sort(rng.standard_normal((cols, nb - 2)), axis=1).astype(np.float32)
    cats = np.zeros(cols, np.uint8)
    cats[2] = 1
    want = core.bin_data(X, E, nb, [2], layout="row")
    fm = np.zeros((cols, ld), np.float32)
    fm[:, :rows] = X.T
    for src, layout, stride in ((fm, core.LAYOUT_FEATURE_MAJOR, ld),
                                (np.ascontiguousarray(X), core.LAYOUT_ROW_MAJOR, cols)):
        bufs = [cu.alloc(src.nbytes), cu.alloc(E.nbytes), cu.alloc(cols), cu.alloc(want.nbytes)]
        try:
            cu.h2d(bufs[0], src)
            cu.h2d(bufs[1], E)
            cu.h2d(bufs[2], cats)
            core.bin_data_device(bufs[0], rows, cols, stride, layout, bufs[1], nb, bufs[2], 0,
                                 bufs[3])
            got = cu.d2h(bufs[3], want.size, np.uint8)
        finally:
            for b in bufs:
                cu.free(b)
        assert np.array_equal(got, want), f"layout {layout}"
