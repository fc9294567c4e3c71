"""Making binned datasets on the GPU against the oracle: quantile edges
(Binner.computeEdges, Sources/MacBoost/Binner.swift:25-60) and bins
(bin_data, Shaders.swift:41-76) bit for bit, the .mbds file byte for byte
against the oracle's restatement of BinnedDataset.save (Sources/MacBoost/
Dataset.swift:26-39), `macboost dataset` (Sources/MacBoostCLI/main.swift:
134-154) end to end, and the trainer's round trip: a model whose thresholds
are the dataset's edges predicts on the dataset exactly as on the rows."""

from __future__ import annotations

import json
import re
import subprocess

import numpy as np
import pytest

from conftest import O, ROOT, assert_bitwise
from macboost_b200 import synth
from test_cli_gpu import _csv

pytestmark = pytest.mark.gpu
CLI = ROOT / "macboost_b200" / "macboost"


def _matrix(rng, rows, cols, cats, nb):
    X = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    X[rng.random(X.shape) < 0.08] = np.nan
    for c in cats:
        X[:, c] = rng.integers(0, nb - 1, rows)
        X[rng.random(rows) < 0.05, c] = np.nan
    if cols > 2 and 2 not in cats:
        X[:, 2] = np.nan                                   # all-NaN feature
    if cols > 4 and 4 not in cats:
        X[:, 4] = np.where(rng.random(rows) < 0.5, np.float32(0.0), np.float32(-0.0))
        X[::17, 4] = np.float32(1.5)
    if cols > 5 and 5 not in cats:
        X[::9, 5] = np.inf
        X[::10, 5] = -np.inf
    return X


@pytest.mark.parametrize("rows,cols,nb", [(20_011, 9, 256), (450_013, 6, 16), (1, 3, 4),
                                          (7, 17, 64)])
def test_make_dataset_vs_oracle(gpu, oracle_built, rows, cols, nb):
    """450k rows sample every 2nd value for the edges (step = rows / 200000)."""
    core = gpu
    rng = np.random.default_rng(rows)
    cats = [c for c in (1, cols - 1) if c != 2 and c != 4]
    X = _matrix(rng, rows, cols, cats, nb)
    y = rng.standard_normal(rows).astype(np.float32)
    d = core.Dataset.make(X, y, num_bins=nb, categorical=cats)
    E, B = O.make_dataset(X, y, nb, cats)
    assert (d.rows, d.cols, d.num_bins) == (rows, cols, nb)
    assert np.array_equal(d.edges.view(np.uint32), E.view(np.uint32)), "edges"
    assert np.array_equal(d.bins, B), "bins"
    assert np.array_equal(d.labels.view(np.uint32), y.view(np.uint32))
    assert d.categorical == sorted(set(cats)) and d.feature_names is None
    dm = core.Dataset.make(np.ascontiguousarray(X.T), y, num_bins=nb, categorical=cats,
                           layout="feature")
    assert np.array_equal(dm.bins, B) and np.array_equal(dm.edges.view(np.uint32),
                                                         E.view(np.uint32))


def test_save_matches_oracle_bytes(gpu, oracle_built, tmp_path):
    core = gpu
    rng = np.random.default_rng(8)
    rows, cols, nb = 3001, 11, 64
    cats = [3, 7]
    X = _matrix(rng, rows, cols, cats, nb)
    y = rng.integers(0, 2, rows).astype(np.float32)
    names = [f"col/{i}" if i % 3 else f'q"{i}' for i in range(cols)]
    d = core.Dataset.make(X, y, num_bins=nb, categorical=[7, 3, 7], feature_names=names)
    got = tmp_path / "g.mbds"
    d.save(got)
    E, B = O.make_dataset(X, y, nb, cats)
    want = tmp_path / "w.mbds"
    O.write_mbds(want, B, rows, cols, nb, cats, names, E, y)
    assert got.read_bytes() == want.read_bytes()
    back = core.Dataset(got)
    assert back.feature_names == names and back.categorical == cats
    assert np.array_equal(back.bins, B)
    # without names: an empty names block
    d2 = core.Dataset.make(X, y, num_bins=nb, categorical=cats)
    d2.save(got)
    O.write_mbds(want, B, rows, cols, nb, cats, None, E, y)
    assert got.read_bytes() == want.read_bytes()


@pytest.mark.parametrize("delim,fmt", [(",", None), ("\t", "tsv")])
def test_cli_dataset_end_to_end(gpu, oracle_built, tmp_path, delim, fmt):
    """`macboost dataset` on a text table equals makeDataset on the parsed
    columns: label column split off, categorical names mapped to features."""
    core = gpu
    rng = np.random.default_rng(31)
    rows, cols, nb = 5003, 8, 32
    X = _matrix(rng, rows, cols, [1, 6], nb)
    y = rng.standard_normal(rows).astype(np.float32)
    names = [f"x{i}" for i in range(cols)]
    table = np.concatenate([X[:, :3], y[:, None], X[:, 3:]], axis=1)   # label in the middle
    data = tmp_path / ("t.tsv" if fmt else "t.csv")
    data.write_text(_csv(table, names[:3] + ["target"] + names[3:], delim))
    out = tmp_path / "t.mbds"
    args = ["dataset", "--data", data, "--output", out, "--label", "target",
            "--categorical", "x6,x1", "--bins", str(nb)]
    if fmt:
        args += ["--format", fmt]
    r = subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert re.fullmatch(rf"binned {rows} rows x {cols} features into {re.escape(str(out))} "
                        r"in \d+\.\d\ds\n", r.stdout), r.stdout
    # the text holds each value to 9 significant digits: parse it back the same way
    parsed = np.array([[np.float32(v) if v else np.nan for v in line.split(delim)]
                       for line in data.read_text().splitlines()[1:]], np.float32)
    Xp = np.concatenate([parsed[:, :3], parsed[:, 4:]], axis=1)
    yp = parsed[:, 3]
    E, B = O.make_dataset(Xp, yp, nb, [1, 6])
    want = tmp_path / "w.mbds"
    O.write_mbds(want, B, rows, cols, nb, [1, 6], names, E, yp)
    assert out.read_bytes() == want.read_bytes()
    assert core.cli_dataset(data, tmp_path / "api.mbds", label="target", categorical="x6,x1",
                            num_bins=nb, fmt=fmt or "auto") == (rows, cols)
    assert (tmp_path / "api.mbds").read_bytes() == want.read_bytes()


def test_cli_dataset_libsvm_defaults(gpu, oracle_built, tmp_path):
    """LibSVM input names its columns label, f0, f1, ...; --bins that is no
    integer falls back to 256 (Int(String) ?? 256)."""
    core = gpu
    rng = np.random.default_rng(5)
    rows, F = 700, 6
    X = np.full((rows, F), np.nan, np.float32)
    lines = []
    for i in range(rows):
        y = int(rng.integers(0, 2))
        feats = sorted(rng.choice(F, size=int(rng.integers(1, F + 1)), replace=False))
        parts = [str(y)]
        for f in feats:
            v = np.float32(rng.standard_normal())
            X[i, f] = v
            parts.append(f"{f + 1}:{float(v)!r}")
        lines.append((y, " ".join(parts)))
    p = tmp_path / "d.svm"
    p.write_text("\n".join(line for _, line in lines) + "\n")
    out = tmp_path / "d.mbds"
    r = subprocess.run([str(CLI), "dataset", "--data", str(p), "--output", str(out), "--bins",
                        "12.5"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    d = core.Dataset(out)
    y = np.float32([yy for yy, _ in lines])
    # CSV.readLibSVM: missing entries are 0, not NaN
    X0 = np.where(np.isnan(X), np.float32(0.0), X)
    E, B = O.make_dataset(X0, y, 256, [])
    assert d.num_bins == 256 and d.feature_names == [f"f{i}" for i in range(F)]
    assert np.array_equal(d.edges.view(np.uint32), E.view(np.uint32))
    assert np.array_equal(d.bins, B) and np.array_equal(d.labels, y)


@pytest.mark.parametrize("K", [1, 3])
def test_predict_on_made_dataset(gpu, oracle_built, K):
    """The trainer's round trip: thresholds taken from the dataset's edges
    route the binned rows as the float predictor routes the raw rows."""
    core = gpu
    rng = np.random.default_rng(40 + K)
    rows, F, nb, cats = 30_000, 12, 64, (10, 11)
    X = _matrix(rng, rows, F, cats, nb)
    X[np.isinf(X)] = np.float32(3e38)      # model JSON holds finite thresholds only
    y = np.zeros(rows, np.float32)
    d = core.Dataset.make(X, y, num_bins=nb, categorical=cats)
    E = d.edges.reshape(F, nb - 2)
    thr = [E[f] for f in range(F)]
    tl = [synth._complete_tree(rng, 6, F, thr, 0.1, frozenset(cats), with_mask=True)
          for _ in range(40 * K)]
    m = {"version": 1, "objective": 7 if K > 1 else 0, "numBins": nb, "baseScore": 0.0,
         "numFeatures": F, "categorical": sorted(cats), "trees": tl, "numClasses": K,
         "baseScores": [0.1 * k for k in range(K)]}
    text = synth.model_to_json(m)
    om = O.model_from_dict(json.loads(text))
    h = core.load_json(text)
    assert_bitwise(core.predict_dataset(h, d, core.KIND_RAW), O.predict_raw(om, X), "raw")
    assert np.array_equal(core.predict_dataset(h, d, core.KIND_LEAF),
                          core.predict_ex(h, X, kind=core.KIND_LEAF))
