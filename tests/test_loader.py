"""Model loading, validation and flattening through the C ABI (no GPU needed).

The loader restates MacBooster.load (Sources/MacBoost/Booster.swift:2144-2162)
and PyModel.__init__ (python/macboost/_pyinfer.py:22-46); arrays are compared
bit for bit with the oracle's json-module reading of the same files.
"""

import ctypes
import json

import numpy as np
import pytest

from conftest import O, golden_names, golden_text
from macboost_b200 import synth


def _load_text(core, text):
    return core.load_json(text)


@pytest.mark.parametrize("name", golden_names())
def test_loader_matches_json_module(lib_built, tmp_path, name):
    core = lib_built
    text = golden_text(name)
    path = tmp_path / "m.json"
    path.write_text(text)
    h = core.load(path)
    ref = O.model_from_dict(json.loads(text))
    assert core.num_trees(h) == ref.num_trees
    assert core.num_features(h) == ref.num_features
    assert core.num_classes(h) == ref.num_classes
    assert core.best_iteration(h) == 0
    # save -> read back with the json module -> identical arrays
    out = tmp_path / "saved.json"
    core.save(h, out)
    back = O.model_from_dict(json.loads(out.read_text()))
    for field in ("feature", "flags", "tree_off", "has_mask", "catmask"):
        assert np.array_equal(getattr(back, field), getattr(ref, field)), field
    for field in ("threshold", "leaf", "base_scores"):
        assert np.array_equal(getattr(back, field).view(np.uint32),
                              getattr(ref, field).view(np.uint32)), field


def test_describe_layouts(lib_built):
    core = lib_built
    h = _load_text(core, golden_text("cfg2_small"))
    d = json.loads(core.describe(h))
    assert d["layout"] == "complete" and d["depth"] == 6 and d["trees"] == 100
    assert d["padded_trees"] % d["group"] == 0 and d["smem_bytes"] <= 232448
    assert d["rows_per_tile"] % 32 == 0
    h5 = _load_text(core, golden_text("cfg5_small"))
    d5 = json.loads(core.describe(h5))
    assert d5["layout"] == "explicit" and d5["depth"] <= 12
    h4 = _load_text(core, golden_text("cfg4_small"))
    d4 = json.loads(core.describe(h4))
    assert d4["classes"] == 10 and d4["group"] == 10


def test_streaming_plan_for_large_forest(lib_built):
    core = lib_built
    m = synth.make_model("cfg4", trees=1000)
    d = json.loads(core.describe(core.load_json(synth.model_to_json(m))))
    assert d["blocks"] > 1 and d["plan"].endswith("forest streamed in tree blocks")
    assert d["smem_bytes"] <= 232448


def test_feature_importance_matches_reference_rule(lib_built):
    core = lib_built
    text = golden_text("cfg1_small")
    h = core.load_json(text)
    m = json.loads(text)
    split = np.zeros(m["numFeatures"], np.float32)
    for t in m["trees"]:
        stack = [0]
        while stack:  # Booster.swift:1926-1940 stack order
            n = stack.pop()
            if t["feature"][n] < 0:
                continue
            split[t["feature"][n]] += 1
            stack += [2 * n + 1, 2 * n + 2]
    assert np.array_equal(core.feature_importance(h, "split"), split)
    assert np.array_equal(core.feature_importance(h, "gain"), np.zeros_like(split))


BASE = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.5, "numFeatures": 2,
        "categorical": [],
        "trees": [{"feature": [0, -1, -1], "threshold": [0.5, 0, 0], "leaf": [0, 1, 2],
                   "flags": [0, 0, 0], "catMask": []}]}


def _variant(**kw):
    m = json.loads(json.dumps(BASE))
    for k, v in kw.items():
        if k.startswith("tree_"):
            m["trees"][0][k[5:]] = v
        elif v is None:
            m.pop(k, None)
        else:
            m[k] = v
    return json.dumps(m)


def test_minimal_model_loads(lib_built):
    h = lib_built.load_json(_variant())
    assert lib_built.num_trees(h) == 1 and lib_built.num_classes(h) == 1


@pytest.mark.parametrize("text,needle", [
    ("{", "malformed"),
    ("[]", "expected '{'"),
    (_variant(version=2), "version"),
    (_variant(objective=9), "objective"),
    (_variant(numBins=3), "numBins"),
    (_variant(numBins=257), "numBins"),
    (_variant(numFeatures=None), "lacks"),
    (_variant(trees=None), "lacks"),
    (_variant(tree_feature=[5, -1, -1]), "feature"),
    (_variant(tree_feature=[0]), "lengths differ"),
    (_variant(tree_feature=[0], tree_threshold=[0.5], tree_leaf=[0], tree_flags=[0]),
     "children outside"),
    (_variant(tree_catMask=[0] * 7), "8 words"),
    (_variant(tree_flags=[256, 0, 0]), "flags"),
    (_variant(numClasses=3), "baseScores"),
    (_variant(numClasses=2, baseScores=[0.0]), "baseScores has 1"),
    (_variant(numClasses=129, baseScores=[0.0] * 129), "numClasses"),
    (_variant(baseScore=1e39), "does not fit"),
    (_variant().replace('"baseScore": 0.5', '"baseScore": NaN'), "malformed"),
    (_variant(tree_feature=[], tree_threshold=[], tree_leaf=[], tree_flags=[]), "empty tree"),
    (_variant() + "x", "trailing"),
])
def test_invalid_models_rejected(lib_built, text, needle):
    with pytest.raises(lib_built.MacBoostError) as ei:
        lib_built.load_json(text)
    assert needle in str(ei.value)


def test_lenient_forms_accepted(lib_built):
    core = lib_built
    # numClasses 0 means one class (_pyinfer.py:31); integral decimals for
    # integer fields; unknown keys ignored; unreachable nodes are not checked.
    h = core.load_json(_variant(numClasses=0, extra={"x": [1, 2]},
                                tree_feature=[0, -1, -1, 99, 99, 99, 99],
                                tree_threshold=[0.5] + [0] * 6, tree_leaf=[0, 1, 2, 0, 0, 0, 0],
                                tree_flags=[0] * 7))
    assert core.num_classes(h) == 1
    h2 = core.load_json(_variant().replace('"numFeatures": 2', '"numFeatures": 2.0'))
    assert core.num_features(h2) == 2


def test_missing_file_and_null_handles(lib_built):
    core = lib_built
    with pytest.raises(core.MacBoostError, match="cannot open"):
        core.load("/nonexistent/dir/model.json")
    lib = core._lib
    for fn in ("macboost_num_trees", "macboost_num_features", "macboost_num_classes",
               "macboost_best_iteration"):
        assert getattr(lib, fn)(None) == -1
    err = ctypes.c_char_p()
    assert lib.macboost_predict(None, None, 1, 1, None, ctypes.byref(err)) == -1
    assert core._take_error(err) == "null argument"


def test_training_entry_points_report_unsupported(lib_built):
    lib = lib_built._lib
    lib.macboost_train.restype = ctypes.c_void_p
    err = ctypes.c_char_p()
    assert not lib.macboost_train(None, None, 0, 0, 0, None, None, None, 0, None,
                                  ctypes.byref(err))
    assert "not supported" in lib_built._take_error(err)


def test_cols_mismatch_is_an_error(lib_built):
    core = lib_built
    h = core.load_json(_variant())
    with pytest.raises(core.MacBoostError, match="model expects 2 features, got 3"):
        core.predict(h, np.zeros((4, 3), np.float32))


def test_plan_thread_bounds_by_class_count(lib_built):
    """Tiles of up to 768 threads for one or two classes, 640 for three or
    four, 512 for five to eight (their kernels' register budgets)."""
    core = lib_built
    rng = np.random.default_rng(3)
    for K, cap in ((1, 768), (2, 768), (3, 640), (4, 640), (5, 512), (8, 512)):
        tl = [synth._complete_tree(rng, 4, 6, synth.EDGES_256, 0.1) for _ in range(4 * K)]
        m = {"version": 1, "objective": 7 if K > 2 else 1, "numBins": 256, "baseScore": 0.0,
             "numFeatures": 6, "categorical": [], "trees": tl, "numClasses": K,
             "baseScores": [0.0] * K}
        d = json.loads(core.describe(core.load_json(synth.model_to_json(m))))
        assert d["rows_per_tile"] <= cap, (K, d["rows_per_tile"])


def test_explicit_child_encoding_choice(lib_built):
    """Explicit records hold 8 x the child distance when every distance is at
    most 2047; a complete depth-12 tree (distances up to 4095) keeps the plain
    distance."""
    core = lib_built
    rng = np.random.default_rng(5)
    leafwise = [synth._leafwise_tree(rng, 100, 11, 10, synth.EDGES_256, 0.1) for _ in range(3)]
    base = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.0, "numFeatures": 10,
            "categorical": [], "numClasses": 1, "baseScores": [0.0]}
    d = json.loads(core.describe(core.load_json(synth.model_to_json({**base, "trees": leafwise}))))
    assert d["layout"] == "explicit" and d["compact_children"] is True
    wide = leafwise + [synth._complete_tree(rng, 12, 10, synth.EDGES_256, 0.1)]
    d = json.loads(core.describe(core.load_json(synth.model_to_json({**base, "trees": wide}))))
    assert d["layout"] == "explicit" and d["compact_children"] is False


def test_plan_restrictions_from_the_environment(lib_built, monkeypatch):
    """MACBOOST_PLAN restricts the planner when a model is loaded: grid (CTAs per
    launch), chunk (rows per host chunk) and claim=0 (fixed chunk order) are
    recorded in the plan; without them the plan has none."""
    core = lib_built
    text = golden_text("cfg2_small")
    d = json.loads(core.describe(core.load_json(text)))
    assert "grid_cap" not in d and "chunk_rows" not in d and "claim" not in d
    monkeypatch.setenv("MACBOOST_PLAN", "grid=3,chunk=4096,claim=0,bufs=2")
    d = json.loads(core.describe(core.load_json(text)))
    assert d["grid_cap"] == 3 and d["chunk_rows"] == 4096 and d["claim"] is False
    assert d["tile_buffers"] == 2


def test_payload_records_choice(lib_built, monkeypatch):
    """Without NaN planes or categorical splits, complete-layout records carry
    the default direction as the walk's fmax operand, a float at or below
    -2^127 for default-left nodes; a forest with a default-left threshold below
    -2^127 would have values under it and keeps the shifted-flag route."""
    core = lib_built
    monkeypatch.setenv("MACBOOST_PLAN", "planes=0,codes=0")

    def describe(threshold, default_left):
        rng = np.random.default_rng(11)
        tl = [synth._complete_tree(rng, 4, 6, synth.EDGES_256, 0.1) for _ in range(8)]
        tl[3]["threshold"][2] = np.float32(threshold)
        tl[3]["flags"][2] = default_left
        m = {"version": 1, "objective": 0, "numBins": 256, "baseScore": 0.0,
             "numFeatures": 6, "categorical": [], "trees": tl, "numClasses": 1,
             "baseScores": [0.0]}
        d = json.loads(core.describe(core.load_json(synth.model_to_json(m))))
        assert d["layout"] == "complete" and d["nan_planes"] is False
        return d["payload_records"]

    assert describe(0.5, 1) is True
    assert describe(-1.7e38, 1) is True          # above -2^127 = -1.7014118e38
    assert describe(-1.71e38, 0) is True         # default right: the operand is a NaN
    assert describe(-1.71e38, 1) is False
    assert describe(-3.4e38, 1) is False
    monkeypatch.setenv("MACBOOST_PLAN", "planes=0,codes=0,pay=0")
    assert describe(0.5, 1) is False
