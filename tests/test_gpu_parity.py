"""GPU parity: the CUDA path through the C ABI against the reference's golden
vectors and the oracle.

Bars: leaf indices and raw margins bit-exact;
transformed outputs (sigmoid / softmax / exp) within 2 ulp fp32 of the
reference formula evaluated in float64 (python/macboost/__init__.py:439-445)
or fp32 exp (Booster.swift:1995-1997, _pyinfer.py:93-95).
"""

import ctypes
import json

import numpy as np
import pytest

from conftest import (O, assert_bitwise, assert_ulp, golden_arrays, golden_names,
                      golden_oracle_model, golden_text)
from macboost_b200 import synth

pytestmark = pytest.mark.gpu
ULP = 2  # tolerance for transformed outputs, fp32 units in the last place


@pytest.mark.parametrize("name", golden_names())
def test_golden_all_kinds(gpu, tmp_path, name):
    core = gpu
    g = golden_arrays(name)
    path = tmp_path / "m.json"
    path.write_text(golden_text(name))
    h = core.load(path)
    X = g["X"]
    K = g["raw"].shape[1]
    raw = core.predict_ex(h, X, kind=core.KIND_RAW)
    assert_bitwise(raw, g["raw"], f"{name} raw")
    raw_f = core.predict_ex(h, np.ascontiguousarray(X.T), kind=core.KIND_RAW, layout="feature")
    assert_bitwise(raw_f, g["raw"], f"{name} raw (feature-major)")
    leaf = core.predict_ex(h, X, kind=core.KIND_LEAF)
    assert np.array_equal(leaf, g["leaf"].astype(np.int32)), f"{name} leaf indices"
    pred = core.predict_ex(h, X, kind=core.KIND_PREDICT)
    assert_ulp(pred, g["pred"], ULP, f"{name} predict")
    if not name.endswith("poisson"):
        assert_bitwise(pred, g["pred"], f"{name} predict (no transform)")
    proba = core.predict_ex(h, X, kind=core.KIND_PROBA)
    assert_ulp(proba, g["proba"].astype(np.float32), ULP, f"{name} proba")
    # the reference-signature entry point (feature-major copy, macboost_predict)
    ref_sig = core.predict(h, X).reshape(-1, K)
    assert_bitwise(ref_sig, pred, f"{name} macboost_predict vs kind=predict")
    assert_ulp(ref_sig, g["pred"], ULP, f"{name} macboost_predict")


CFG_ROWS = {"cfg1": 20_000, "cfg2": 50_000, "cfg3": 20_000, "cfg4": 4_000, "cfg5": 6_000}


@pytest.fixture(scope="module")
def cfg_models():
    return {}


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
def test_config_models_vs_oracle(gpu, oracle_built, cfg, cfg_models):
    """Full-size models of the five benchmark configs on seeded row samples."""
    core = gpu
    model = synth.make_model(cfg)
    text = synth.model_to_json(model)
    h = core.load_json(text)
    om = O.model_from_dict(json.loads(text))
    n = CFG_ROWS[cfg]
    X = synth.make_data(cfg, rows=n, row_start=12_345, layout="feature")
    raw_o, leaf_o = O.predict_raw(om, X, layout="feature", want_leaf=True)
    raw = core.predict_ex(h, X, kind=core.KIND_RAW, layout="feature")
    assert_bitwise(raw, raw_o, f"{cfg} raw")
    leaf = core.predict_ex(h, X, kind=core.KIND_LEAF, layout="feature")
    assert np.array_equal(leaf, leaf_o), f"{cfg} leaf"
    proba = core.predict_ex(h, X, kind=core.KIND_PROBA, layout="feature")
    ref = O.predict_proba(raw_o if om.num_classes > 1 else raw_o[:, 0]).astype(np.float32)
    assert_ulp(proba, ref, ULP, f"{cfg} proba")


@pytest.mark.parametrize("rows", [1, 3, 4, 31, 255, 257, 511, 513, 1000, 4099])
def test_ragged_row_counts(gpu, oracle_built, rows):
    core = gpu
    name = "cfg2_small"
    h = core.load_json(golden_text(name))
    om = golden_oracle_model(name)
    X = synth.make_data("cfg2", rows=rows, row_start=777, layout="row")
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), O.predict_raw(om, X),
                   f"rows={rows}")


def test_zero_rows(gpu):
    core = gpu
    h = core.load_json(golden_text("cfg1_small"))
    out = core.predict_ex(h, np.zeros((0, 100), np.float32), kind=core.KIND_RAW)
    assert out.shape == (0, 1)


def test_device_entry_point_alignment_paths(gpu, oracle_built):
    """Device-resident input: aligned (bulk copies) and misaligned (plain
    loads) base addresses and strides give identical results."""
    core = gpu
    from macboost_b200 import _core
    cudart = _cudart()
    h = core.load_json(golden_text("cfg3_small"))
    om = golden_oracle_model("cfg3_small")
    rows, F = 3001, 100
    X = synth.make_data("cfg3", rows=rows, layout="feature")
    ref = O.predict_raw(om, X, layout="feature")
    for ld, offset in [(3004, 0), (3001, 0), (3004, 1), (3010, 3)]:
        buf = np.zeros((F, ld), np.float32)
        buf[:, :rows] = X
        flat = np.concatenate([np.zeros(offset, np.float32), buf.ravel()])
        dx = cudart.alloc(flat.nbytes)
        dout = cudart.alloc(rows * 4)
        try:
            cudart.h2d(dx, flat)
            _core.predict_device(h, 0, dx + 4 * offset, rows, F, ld, dout, kind=core.KIND_RAW)
            core.check_device(h, 0)
            out = cudart.d2h(dout, rows, np.float32)
        finally:
            cudart.free(dx)
            cudart.free(dout)
        assert_bitwise(out.reshape(rows, 1), ref, f"ld={ld} offset={offset}")


def test_deterministic_and_leaf_consistent(gpu):
    core = gpu
    h = core.load_json(golden_text("cfg4_small"))
    X = synth.make_data("cfg4", rows=5000, layout="row")
    a = core.predict_ex(h, X, kind=core.KIND_RAW)
    b = core.predict_ex(h, X, kind=core.KIND_RAW)
    assert_bitwise(a, b, "repeat")
    # margins recomputed on the host from the GPU's leaf indices, in tree order
    leaf = core.predict_ex(h, X, kind=core.KIND_LEAF)
    m = json.loads(golden_text("cfg4_small"))
    K = m["numClasses"]
    acc = np.tile(np.asarray(m["baseScores"], np.float32), (X.shape[0], 1))
    for t, tree in enumerate(m["trees"]):
        lv = np.asarray(tree["leaf"], np.float64).astype(np.float32)
        acc[:, t % K] += lv[leaf[:, t]]
    assert_bitwise(a, acc, "margins from leaf indices")


def test_multi_device_sharding(gpu, oracle_built):
    core = gpu
    n = core.device_count()
    h = core.load_json(golden_text("cfg2_small"))
    om = golden_oracle_model("cfg2_small")
    X = synth.make_data("cfg2", rows=10_007, layout="row")
    ref = O.predict_raw(om, X)
    devs = list(range(min(n, 4)))
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW, devices=devs), ref,
                   f"devices={devs}")
    with pytest.raises(core.MacBoostError, match="listed twice"):
        core.predict_ex(h, X, kind=core.KIND_RAW, devices=[0, 0])
    with pytest.raises(core.MacBoostError, match="does not exist"):
        core.predict_ex(h, X, kind=core.KIND_RAW, devices=[n + 3])


def test_pinned_buffers(gpu, oracle_built):
    core = gpu
    h = core.load_json(golden_text("cfg1_small"))
    om = golden_oracle_model("cfg1_small")
    X = core.pinned_empty((7000, 100))
    X[:] = synth.make_data("cfg1", rows=7000, layout="row")
    out = core.pinned_empty((7000, 1))
    core.predict_ex(h, X, kind=core.KIND_RAW, out=out)
    assert_bitwise(out, O.predict_raw(om, np.asarray(X)), "pinned")


class _Cudart:
    """Minimal device-memory helpers over the CUDA runtime (test plumbing)."""

    def __init__(self):
        import glob
        import os
        cands = sorted(glob.glob("/usr/local/cuda/lib64/libcudart.so*")) + ["libcudart.so.12"]
        last = None
        for c in cands:
            try:
                self.lib = ctypes.CDLL(c if os.path.exists(c) else c)
                break
            except OSError as e:
                last = e
        else:
            raise last
        self.lib.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
        self.lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_int]
        self.lib.cudaFree.argtypes = [ctypes.c_void_p]

    def alloc(self, n):
        p = ctypes.c_void_p()
        assert self.lib.cudaMalloc(ctypes.byref(p), n) == 0
        return p.value

    def h2d(self, d, a):
        assert self.lib.cudaMemcpy(d, a.ctypes.data, a.nbytes, 1) == 0

    def d2h(self, d, n, dt):
        out = np.empty(n, dt)
        assert self.lib.cudaMemcpy(out.ctypes.data, d, out.nbytes, 2) == 0
        return out

    def free(self, d):
        self.lib.cudaFree(d)


_CUDART = None


def _cudart():
    global _CUDART
    if _CUDART is None:
        _CUDART = _Cudart()
    return _CUDART


@pytest.mark.parametrize("plan", ["codes=0", "codes=0,planes=0", "codes=1", "codes=1,G=8",
                                  "codes=0,top=1", "codes=0,planes=0,top=1", "codes=0,top=0",
                                  "codes=0,planes=0,pay=0", "codes=0,planes=0,top=1,pay=0"])
@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_every_layout_vs_oracle(gpu, oracle_built, cfg, plan, monkeypatch):
    """Each kernel family (fp32 tiles with NaN planes, fp32 with default-left
    flags, the default direction as the record word or by a shift of its flag
    bit, binned codes; the first two levels from shared memory or from the
    kernel parameter), forced through MACBOOST_PLAN, against the oracle."""
    core = gpu
    if cfg == "cfg4" and "G=8" in plan:
        pytest.skip("10 classes walk 10 trees per group")
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    trees = {"cfg4": 300}.get(cfg)
    text = synth.model_to_json(synth.make_model(cfg, trees=trees))
    h = core.load_json(text)
    desc = json.loads(core.describe(h))
    assert desc["codes"] == ("codes=1" in plan)
    if "planes=0" in plan:
        assert desc["nan_planes"] is False
    if "top=1" in plan and desc["layout"] == "complete":
        assert desc["top_params"] is True
    if "top=0" in plan:
        assert desc["top_params"] is False
    if "pay=0" in plan:
        assert desc["payload_records"] is False
    elif "planes=0" in plan and desc["layout"] == "complete" and cfg != "cfg3":
        assert desc["payload_records"] is True   # no categorical splits, no planes
    om = O.model_from_dict(json.loads(text))
    X = synth.make_data(cfg, rows=5003, row_start=999, layout="row")
    raw_o, leaf_o = O.predict_raw(om, X, want_leaf=True)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), raw_o, f"{cfg} {plan} raw")
    assert np.array_equal(core.predict_ex(h, X, kind=core.KIND_LEAF), leaf_o), f"{cfg} {plan}"


@pytest.mark.parametrize("name", golden_names())
def test_cli_transform_kind(gpu, oracle_built, name):
    """MACBOOST_KIND_CLI: the float32 transform `macboost predict` applies."""
    core = gpu
    g = golden_arrays(name)
    h = core.load_json(golden_text(name))
    m = golden_oracle_model(name)
    with np.errstate(over="ignore"):
        ref = O.predict_cli(m, g["raw"])
    got = core.predict_ex(h, g["X"], kind=core.KIND_CLI)
    assert_ulp(got, ref, ULP, f"{name} cli transform")


@pytest.mark.parametrize("cfg,plan", [("cfg1", "codes=0,planes=0"), ("cfg2", "codes=0,planes=0"),
                                      ("cfg5", "")])
def test_nan_free_tiles(gpu, oracle_built, cfg, plan, monkeypatch):
    """Row tiles without NaN take the walk without default-direction tests;
    tiles with NaN keep them.  Rows with NaN in a few places, so that both kinds
    of tile occur in one call, against the oracle."""
    core = gpu
    if plan:
        monkeypatch.setenv("MACBOOST_PLAN", plan)
    trees = {"cfg5": 60}.get(cfg)
    text = synth.model_to_json(synth.make_model(cfg, trees=trees))
    h = core.load_json(text)
    om = O.model_from_dict(json.loads(text))
    X = synth.make_data(cfg, rows=9001, row_start=31, layout="row")
    X = np.where(np.isnan(X), np.float32(0.5), X).astype(np.float32)
    X[4000:4003, 7] = np.nan                   # one or two tiles with NaN
    X[8999, 2] = np.nan                        # and the last, partial tile
    raw_o, leaf_o = O.predict_raw(om, X, want_leaf=True)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), raw_o, f"{cfg} raw")
    assert np.array_equal(core.predict_ex(h, X, kind=core.KIND_LEAF), leaf_o), f"{cfg} leaf"


@pytest.mark.parametrize("depth", [3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("plan", ["codes=0,G=8", "codes=0,G=8,planes=0", "codes=0,G=8,top=1",
                                  "codes=0,G=8,planes=0,top=1", "codes=0,G=8,top=0"])
def test_fixed_depth_builds(gpu, oracle_built, depth, plan, monkeypatch):
    """Single-class forests of depth 4-8 in 8-tree groups run the fixed-depth
    kernel builds (depth 3: the run-time-depth build), with and without NaN
    planes and top-level parameters, categorical splits and NaN rows (tiles
    with and without NaN), against the oracle."""
    core = gpu
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    rng = np.random.default_rng(700 + depth)
    F, cats = 30, frozenset({27, 28, 29})
    tl = [synth._complete_tree(rng, depth, F, synth.EDGES_256, 0.1, cats, with_mask=True)
          for _ in range(37)]
    m = {"version": 1, "objective": 1, "numBins": 256, "baseScore": -0.2, "numFeatures": F,
         "categorical": sorted(cats), "trees": tl, "numClasses": 1, "baseScores": [-0.2]}
    text = synth.model_to_json(m)
    h = core.load_json(text)
    om = O.model_from_dict(json.loads(text))
    X = rng.random((20_000, F), dtype=np.float32)
    X[:, 27:] = rng.integers(-2, 260, (20_000, 3))
    X[10_000:][rng.random((10_000, F)) < 0.05] = np.nan     # the second half holds NaN
    raw_o, leaf_o = O.predict_raw(om, X, want_leaf=True)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), raw_o, f"d{depth} {plan} raw")
    assert np.array_equal(core.predict_ex(h, X, kind=core.KIND_LEAF), leaf_o), f"d{depth} leaf"


@pytest.mark.parametrize("wide", [False, True])
def test_explicit_child_encodings(gpu, oracle_built, wide):
    """Explicit-layout records store 8 x the child distance when every
    distance is at most 2047, else the distance itself (a complete depth-12
    tree has distances up to 4095); both walks against the oracle."""
    core = gpu
    rng = np.random.default_rng(91 + wide)
    F = 24
    tl = [synth._leafwise_tree(rng, 120, 11, F, synth.EDGES_256, 0.1) for _ in range(15)]
    if wide:
        tl.insert(7, synth._complete_tree(rng, 12, F, synth.EDGES_256, 0.1))
    m = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.1, "numFeatures": F,
         "categorical": [], "trees": tl, "numClasses": 1, "baseScores": [0.1]}
    text = synth.model_to_json(m)
    h = core.load_json(text)
    d = json.loads(core.describe(h))
    assert d["layout"] == "explicit" and d["compact_children"] is (not wide)
    om = O.model_from_dict(json.loads(text))
    X = rng.random((6000, F), dtype=np.float32)
    X[3000:][rng.random((3000, F)) < 0.1] = np.nan
    raw_o, leaf_o = O.predict_raw(om, X, want_leaf=True)
    assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW), raw_o, f"wide={wide}")
    assert np.array_equal(core.predict_ex(h, X, kind=core.KIND_LEAF), leaf_o)
