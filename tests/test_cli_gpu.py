"""`macboost predict` end to end on the GPU: text input through the CLI
readers, the engine, and the prediction file, against the oracle
(Sources/MacBoostCLI/main.swift:317-371 restated in oracle/table_ref.py and
oracle.predict_cli).

Outputs without a transform (regression margins, --raw) must match the
oracle's file byte for byte; sigmoid / softmax / exp outputs within 2 ulp
fp32 of the oracle's float32 transform.
"""

from __future__ import annotations

import json
import math
import subprocess

import numpy as np
import pytest

from conftest import O, ROOT, assert_ulp, golden_arrays, golden_names, golden_text
from macboost_b200 import synth
from oracle import table_ref as T

pytestmark = pytest.mark.gpu
ULP = 2
CLI = ROOT / "macboost_b200" / "macboost"


def _csv(X, names, delim=","):
    lines = [delim.join(names)]
    for row in X:
        lines.append(delim.join("" if math.isnan(v) else "%.9g" % v for v in row))
    return "\n".join(lines) + "\n"


def _run(*args):
    r = subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return r


def _read_preds(path, k):
    lines = path.read_text().splitlines()
    head = lines[0]
    want = ",".join(f"class_{c}" for c in range(k)) if k > 1 else "prediction"
    assert head == want
    return np.array([[np.float32(v) for v in ln.split(",")] for ln in lines[1:]], np.float32)


def _compare(path, ref: np.ndarray, k: int, exact: bool, what: str):
    if exact:
        assert path.read_text() == T.prediction_text(ref, k), what
    else:
        assert_ulp(_read_preds(path, k), ref.reshape(-1, k), ULP, what)


@pytest.mark.parametrize("name", golden_names())
def test_cli_predict_golden(gpu, tmp_path, name):
    g = golden_arrays(name)
    text = golden_text(name)
    m = json.loads(text)
    om = O.model_from_dict(m)
    K = om.num_classes
    model = tmp_path / "m.json"
    model.write_text(text)
    X = g["X"]
    data = tmp_path / "x.csv"
    data.write_text(_csv(X, [f"c{i}" for i in range(X.shape[1])]))
    raw = g["raw"]
    with np.errstate(over="ignore"):
        cli_ref = O.predict_cli(om, raw)
    transformed = K > 1 or om.objective in (1, 5, 6)
    out = tmp_path / "p.csv"
    r = _run("predict", "--model", model, "--data", data, "--output", out)
    assert r.stdout.strip() == f"wrote {X.shape[0]} predictions to {out}"
    _compare(out, cli_ref, K, not transformed, f"{name} cli")
    # --raw: predict semantics (exp kept for the log-link objectives)
    _run("predict", "--model", model, "--data", data, "--output", out, "--raw")
    with np.errstate(over="ignore"):
        pred = O.predict(om, raw)
    _compare(out, pred, K, om.objective not in (5, 6), f"{name} --raw")


def test_cli_feature_names_tsv_and_libsvm(gpu, tmp_path):
    """Columns matched by name (shuffled, with extra and label columns), TSV
    input, and LibSVM input through --format."""
    m = json.loads(golden_text("cfg3_small"))
    F = m["numFeatures"]
    names = [f"f{i}" for i in range(F)]
    m["featureNames"] = names
    model = tmp_path / "named.json"
    model.write_text(json.dumps(m))
    om = O.model_from_dict(m)
    X = synth.make_data("cfg3", rows=2500, row_start=42, layout="row")
    ref = O.predict_raw(om, X)
    rng = np.random.default_rng(0)
    perm = rng.permutation(F)
    cols = ["label", "junk"] + [names[j] for j in perm]
    table = np.column_stack([np.zeros(len(X)), np.ones(len(X)), X[:, perm]]).astype(np.float32)
    out = tmp_path / "p.csv"
    for delim, fname in ((",", "x.csv"), ("\t", "x.tsv")):
        data = tmp_path / fname
        data.write_text(_csv(table, cols, delim))
        _run("predict", "--model", model, "--data", data, "--output", out)
        _compare(out, ref, 1, True, f"by name, delimiter {delim!r}")
    # LibSVM: every value written (NaN as "nan"); columns label, f0, f1, ...
    lines = []
    for row in X:
        lines.append("0 " + " ".join(f"{j}:{'nan' if math.isnan(v) else '%.9g' % v}"
                                     for j, v in enumerate(row)))
    svm = tmp_path / "x.svm"
    svm.write_text("\n".join(lines) + "\n")
    _run("predict", "--model", model, "--data", svm, "--output", out, "--format", "libsvm")
    _compare(out, ref, 1, True, "libsvm")
    _run("predict", "--model", model, "--data", svm, "--output", out, "--format", "auto")
    _compare(out, ref, 1, True, "libsvm (auto)")


def test_cli_predict_through_the_c_abi(gpu, tmp_path):
    """macboost_cli_predict from Python on a larger multiclass table."""
    core = gpu
    text = synth.model_to_json(synth.make_model("cfg4", trees=200))
    om = O.model_from_dict(json.loads(text))
    X = synth.make_data("cfg4", rows=20_000, row_start=5, layout="row")
    data = tmp_path / "x.csv"
    data.write_text(_csv(X, [f"c{i}" for i in range(X.shape[1])]))
    h = core.load_json(text)
    out = tmp_path / "p.csv"
    assert core.cli_predict(h, data, out, devices=[0]) == len(X)
    raw = O.predict_raw(om, X)
    with np.errstate(over="ignore"):
        _compare(out, O.predict_cli(om, raw), om.num_classes, False, "cfg4 softmax")
    assert core.cli_predict(h, data, out, raw=True) == len(X)
    _compare(out, raw, om.num_classes, True, "cfg4 --raw")
