"""The persistent kernels' steady state against the oracle.

A launch sizes its grid to one wave of resident CTAs, so on the row counts a
test can check every CTA (and every warp of the per-warp pipeline) would take
one row tile at most and the loop body would run once.  After its first tile
(two tiles, CTA-wide loops) each warp or CTA claims the next from the launch's
per-stream counters ("claim=0": a fixed order), and both orders are covered.  MACBOOST_PLAN "grid=N"
caps the CTAs of a launch; with two CTAs each one loops over many tiles, so
these tests reach what a 10M-row launch runs: the per-warp loop's later
chunks (mbarrier phase flips, buffer release and prefetch into the other
buffer), the streamed forest's wrap from its last block to block 0 of the next
tile, and the host path's double-buffered chunks ("chunk=N").  Every family
(complete with one and two tile buffers, streamed complete, explicit, binned
codes, TreeSHAP, the binned-data walk) is compared with the oracle: margins
and leaf indices bit-exact, as the reference's own GPU-vs-CPU test asks of a
whole batch (Tests/MacBoostTests/FeatureTests.swift:284-301).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import O, assert_bitwise, assert_ulp
from macboost_b200 import synth

pytestmark = pytest.mark.gpu


def _loops(desc, rows, grid):
    """Tiles (or 32-row chunks, per-warp pipeline) each CTA or warp walks."""
    R = desc["rows_per_tile"]
    if desc["blocks"] == 1 and not desc["codes"]:
        return (rows + 31) // 32 // (grid * (R // 32))
    return (rows + R - 1) // R // grid


CASES = [
    # (config, trees, rows, plan): every family of the forest kernel
    ("cfg2", None, 50_000, "codes=0,bufs=1,grid=2"),     # resident, per-warp, 1 buffer
    ("cfg2", None, 50_000, "codes=0,bufs=2,grid=2"),     # resident, per-warp, 2 buffers
    ("cfg2", None, 40_000, "codes=0,planes=0,grid=3"),   # no NaN planes (NaN-free chunk test)
    ("cfg3", None, 30_000, "codes=0,grid=2"),            # categorical, streamed or resident
    ("cfg4", 300, 20_000, "codes=0,bufs=1,grid=2"),      # streamed blocks, 1 tile buffer
    ("cfg4", 300, 20_000, "codes=0,bufs=2,grid=2"),      # streamed blocks, 2 tile buffers
    ("cfg5", 120, 12_000, "grid=2"),                     # explicit (leaf-wise) layout
    ("cfg2", None, 30_000, "codes=1,grid=2"),            # binned codes, resident
    ("cfg4", 1000, 12_000, "codes=1,grid=2"),            # binned codes, streamed
    ("cfg2", None, 50_000, "codes=0,claim=0,grid=2"),    # per-warp, fixed chunk order
    ("cfg4", 300, 20_000, "codes=0,claim=0,grid=2"),     # CTA tiles, fixed tile order
]


@pytest.mark.parametrize("cfg,trees,rows,plan", CASES)
def test_persistent_loop_vs_oracle(gpu, oracle_built, monkeypatch, cfg, trees, rows, plan):
    core = gpu
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    text = synth.model_to_json(synth.make_model(cfg, trees=trees))
    h = core.load_json(text)
    desc = json.loads(core.describe(h))
    grid = int(plan.split("grid=")[1].split(",")[0])
    assert desc["grid_cap"] == grid
    assert desc["codes"] == ("codes=1" in plan)
    if "bufs=" in plan:
        assert desc["tile_buffers"] == int(plan.split("bufs=")[1].split(",")[0])
    if cfg == "cfg4":
        assert desc["blocks"] > 1, "the cfg4 forest should stream in blocks"
    if cfg == "cfg2" and "codes=0" in plan and "planes=0" not in plan:
        assert desc["blocks"] == 1, "the cfg2 forest should be resident (per-warp pipeline)"
    loops = _loops(desc, rows, grid)
    assert loops >= 4, f"only {loops} trips round the persistent loop"
    om = O.model_from_dict(json.loads(text))
    X = synth.make_data(cfg, rows=rows, row_start=5_000_017, layout="feature")
    raw_o, leaf_o = O.predict_raw(om, X, layout="feature", want_leaf=True)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW, layout="feature"), raw_o,
                   f"{cfg} {plan} raw")
    leaf = core.predict_ex(h, X, kind=core.KIND_LEAF, layout="feature")
    assert np.array_equal(leaf, leaf_o), f"{cfg} {plan} leaf indices"
    proba = core.predict_ex(h, X, kind=core.KIND_PROBA, layout="feature")
    ref = O.predict_proba(raw_o if om.num_classes > 1 else raw_o[:, 0]).astype(np.float32)
    assert_ulp(proba, ref, 2, f"{cfg} {plan} proba")


@pytest.mark.parametrize("plan", ["grid=2,chunk=4096", "grid=3,chunk=1000,bufs=2"])
def test_host_chunks_vs_oracle(gpu, oracle_built, monkeypatch, plan):
    """A host-memory predict in many chunks (two streams, two buffers each,
    the D2H of chunk c queued after chunk c+1), row- and feature-major."""
    core = gpu
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    text = synth.model_to_json(synth.make_model("cfg2"))
    h = core.load_json(text)
    assert json.loads(core.describe(h))["chunk_rows"] == int(plan.split("chunk=")[1].split(",")[0])
    om = O.model_from_dict(json.loads(text))
    rows = 21_003                              # 6 and 22 chunks, the last one ragged
    X = synth.make_data("cfg2", rows=rows, row_start=3_000_001, layout="row")
    want = O.predict_raw(om, X)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), want, f"{plan} row-major")
    assert_bitwise(core.predict_ex(h, np.ascontiguousarray(X.T), kind=core.KIND_RAW,
                                   layout="feature"), want, f"{plan} feature-major")
    n = core.device_count()
    if n > 1:
        devs = list(range(min(n, 4)))
        assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW, devices=devs), want,
                       f"{plan} devices={devs}")


@pytest.mark.parametrize("cfg,plan", [
    ("cfg2", "grid=2,chunk=1024"),                 # accumulators in shared memory
    ("cfg1", "grid=2,chunk=1024"),                 # 100 features: accumulators in global memory
    ("cfg2", "grid=3,chunk=1024,shapglobal=2"),    # global accumulators forced
    ("cfg1", "chunk=1000"),                        # two streams' chunks overlapping, full grid
    ("cfg1", "grid=3,shapdense=0"),                # the 154-register global build
    ("cfg4", "grid=3,chunk=1024,shapdense=1"),     # the 128-register build, 10 classes
])
def test_contrib_persistent_loop(gpu, oracle_built, monkeypatch, cfg, plan):
    """TreeSHAP's persistent CTAs over many row tiles and host chunks (the
    chunks of the two streams use separate global accumulator regions)."""
    from test_shap_gpu import assert_contrib_close, covered
    core = gpu
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    text, om = covered(cfg, 40)
    h = core.load_json(text)
    X = synth.make_data(cfg, rows=3000, row_start=77_777, layout="row")
    want = O.predict_contrib(om, X)
    got = core.predict_contrib_ex(h, X, layout="row", devices=[0])
    assert assert_contrib_close(got, want, f"contrib {cfg} {plan}") > 0.95
    # the device entry point on the same handle (accumulator region 0, waits)
    Xf = np.ascontiguousarray(X.T)
    got_d = core.predict_contrib_ex(h, Xf, layout="feature", devices=[0])
    assert assert_contrib_close(got_d, want, f"contrib {cfg} {plan} feature-major") > 0.95


def test_binned_walk_persistent_loop(gpu, oracle_built, monkeypatch):
    """The binned-data walk's staged kernel (256-row tiles) over 6 tiles per CTA."""
    from test_binned_cpu import NUM_BINS, binned_model
    core = gpu
    monkeypatch.setenv("MACBOOST_PLAN", "grid=2")
    m, X, E = binned_model(seed=31)
    om = O.model_from_dict(json.loads(synth.model_to_json(m)))
    bins = O.bin_data(X, E, NUM_BINS, m["categorical"])
    sf = O.split_form(om, E, NUM_BINS)
    rows, cols = X.shape
    start = np.random.default_rng(2).standard_normal(rows).astype(np.float32)
    want = start.copy()
    want_leaf = O.predict_binned(bins, rows, NUM_BINS, sf, 5, 1, want, want_leaf=True)
    got = start.copy()
    got_leaf = core.predict_tree_binned(bins, rows, cols, NUM_BINS, sf.tree_off, sf.feature,
                                        sf.bin, sf.flags, sf.catmask, sf.leaf, 5, 1, preds=got,
                                        want_leaf=True)
    assert_bitwise(got, want, "binned preds grid=2")
    assert np.array_equal(got_leaf, want_leaf)
