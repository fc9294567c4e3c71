"""Making binned datasets (MacBooster.makeDataset, Sources/MacBoost/
Booster.swift:392-434; `macboost dataset`, Sources/MacBoostCLI/main.swift:
134-154) on the CPU: the oracle's quantile edges pinned to a plain-Python
restatement of Binner.computeEdges (Sources/MacBoost/Binner.swift:25-60),
feature names through the .mbds writer and reader, and every check that
fails before a GPU is touched, with the reference's messages."""

from __future__ import annotations

import math
import re
import struct
import subprocess

import numpy as np
import pytest

from conftest import O, ROOT

CLI = ROOT / "macboost_b200" / "macboost"


def edges_loop(cols_values, num_bins, categorical=(), sample_cap=200_000):
    """Binner.computeEdges as plain Python: Python's sort is stable, as the
    reference's Array.sort is, so equal keys (-0.0 and 0.0) keep their order."""
    data_bins = num_bins - 1
    ne = data_bins - 1
    out = []
    for f, col in enumerate(cols_values):
        if f in categorical:
            out.extend([0.0] * ne)
            continue
        step = max(1, len(col) // sample_cap)
        sample = sorted(v for v in col[::step] if not math.isnan(v))
        if not sample:
            out.extend([0.0] * ne)
            continue
        m = len(sample)
        out.extend(sample[min(m - 1, ((k + 1) * m) // data_bins)] for k in range(ne))
    return np.float32(out)


@pytest.mark.parametrize("num_bins,sample_cap", [(4, 200_000), (16, 7), (256, 200_000),
                                                 (64, 100)])
def test_compute_edges_oracle_vs_loop(num_bins, sample_cap):
    rng = np.random.default_rng(num_bins)
    rows, cols = 1500, 7
    X = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    X[:, 2] = np.nan                                       # all-NaN feature
    X[:, 3] = rng.integers(0, 5, rows)                     # categorical
    X[:, 4] = np.where(rng.random(rows) < 0.5, np.float32(0.0), np.float32(-0.0))
    X[::11, 5] = np.inf
    X[::13, 5] = -np.inf
    X[:, 6] = np.round(X[:, 6])                            # many ties
    got = O.compute_edges(X, num_bins, categorical=[3], sample_cap=sample_cap)
    want = edges_loop([list(map(float, X[:, f].astype(np.float64))) for f in range(cols)],
                      num_bins, {3}, sample_cap)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    fm = O.compute_edges(np.ascontiguousarray(X.T), num_bins, [3], "feature", sample_cap)
    assert np.array_equal(got.view(np.uint32), fm.view(np.uint32))


def test_mbds_feature_names_escaping(lib_built, tmp_path):
    """Names as JSONEncoder writes them ("/" escaped, UTF-8 as is) read back."""
    core = lib_built
    names = ["a/b", 'q"uote', "back\\slash", "tab\there", "ünï", "ctl\x01", "", "x"]
    rows, cols, nb = 5, len(names), 16
    bins = np.zeros(((cols + 7) // 8) * 8 * rows, np.uint8)
    p = tmp_path / "n.mbds"
    O.write_mbds(p, bins, rows, cols, nb, [], names, np.zeros(cols * (nb - 2), np.float32),
                 np.zeros(rows, np.float32))
    raw = p.read_bytes()
    (nlen,) = struct.unpack_from("<I", raw, 32)
    text = raw[36:36 + nlen].decode()
    assert '"a\\/b"' in text and "ünï" in text and "\\u0001" in text
    assert core.Dataset(p).feature_names == names


def test_dataset_make_errors(lib_built):
    """makeDataset's checks, in the reference's order, before any device work."""
    core = lib_built
    rng = np.random.default_rng(1)
    X = rng.standard_normal((50, 4)).astype(np.float32)
    y = np.zeros(50, np.float32)
    for nb in (3, 257, -1):
        with pytest.raises(core.MacBoostError,
                           match=rf"^Invalid input: numBins must be in 4\.\.\.256, got {nb}$"):
            core.Dataset.make(X, y, num_bins=nb)
    with pytest.raises(core.MacBoostError, match=r"^Invalid input: dataset shapes inconsistent "
                                                 r"\(rows=0, cols=4, X=0, y=0\)$"):
        core.Dataset.make(X[:0], y[:0])
    for bad, text in ((np.nan, "nan"), (np.inf, "inf"), (-np.inf, "-inf")):
        yb = y.copy()
        yb[7] = bad
        yb[9] = np.nan
        with pytest.raises(core.MacBoostError, match=rf"^Invalid input: label at row 7 is "
                                                     rf"{text}; labels must be finite$"):
            core.Dataset.make(X, yb)
    Xc = X.copy()
    Xc[:, 1] = rng.integers(0, 15, 50)
    Xc[:, 3] = rng.integers(0, 15, 50)
    Xc[4, 1] = np.nan                                     # NaN ids are skipped
    Xc[5, 1] = 14.5                                       # rounds to even: 14, inside 0..<15
    Xc[6, 1] = -0.4                                       # rounds to -0.0, inside
    for col, v, shown in ((1, 15.5, "15.5"), (1, -0.6, "-0.6"), (3, 300.0, "300.0"),
                          (3, -np.inf, "-inf"), (1, 1e20, "1e+20")):
        Xb = Xc.copy()
        Xb[10, col] = v
        Xb[20, 3 if col == 1 else 1] = 99.0               # a later feature is bad too
        first = min(col, 3 if col == 1 else 1)
        shown_first = shown if first == col else "99.0"
        with pytest.raises(core.MacBoostError,
                           match=rf"^Categorical feature {first} has value "
                                 rf"{re.escape(shown_first)}; expected integer ids in "
                                 r"0\.\.<15 or NaN$"):
            core.Dataset.make(Xb, y, num_bins=16, categorical=[3, 1])


def _run(*args, env=None):
    return subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True,
                          timeout=120, env=env)


def test_cli_dataset_errors_before_the_gpu(lib_built, tmp_path):
    d = tmp_path / "t.csv"
    d.write_text("a,b,label,c\n1,2,0,3\n4,,1,5\n")
    out = tmp_path / "o.mbds"
    for args, msg in [
            (("dataset",), "error: --data is required"),
            (("dataset", "--data", d), "error: --output is required (e.g. train.mbds)"),
            (("dataset", "--data", d, "--output", out, "--format", "xml"),
             "error: unknown --format 'xml' (auto | csv | tsv | libsvm)"),
            (("dataset", "--data", tmp_path / "absent.csv", "--output", out),
             f"error: CSV I/O error: cannot read {tmp_path / 'absent.csv'}"),
            (("dataset", "--data", d, "--output", out, "--label", "y"),
             "error: label column 'y' not found; columns: a, b, label, c"),
            (("dataset", "--data", d, "--output", out, "--categorical", "a,label"),
             "error: categorical column 'label' not found among features"),
            (("dataset", "--data", d, "--output", out, "--bins", "3"),
             "error: Invalid input: numBins must be in 4...256, got 3"),
            (("dataset", "--data", d, "--output", out, "--bins", "99999999999"),
             "error: Invalid input: numBins must be in 4...256, got 99999999999"),
            (("dataset", "--data", d, "--output", out, "--bins", "-4"),
             "error: Invalid input: numBins must be in 4...256, got -4"),
            (("dataset", "--data", d, "--output", out, "--label", "b"),
             "error: Invalid input: label at row 1 is nan; labels must be finite"),
            (("dataset", "--data", d, "--output", out, "--categorical", "c", "--bins", "5"),
             "error: Categorical feature 2 has value 5.0; expected integer ids in 0..<4 or NaN")]:
        r = _run(*args)
        assert r.returncode == 1 and r.stderr.strip() == msg, (args, r.stderr)
    assert not out.exists()
    # a header-only table: the reader refuses it (CSV.swift), before makeDataset's
    # shape check
    h = tmp_path / "h.csv"
    h.write_text("a,label\n")
    r = _run("dataset", "--data", h, "--output", out)
    assert r.stderr.strip() == "error: Malformed CSV: no data rows"
    # a table of only the label column: no features
    h.write_text("label\n1\n")
    r = _run("dataset", "--data", h, "--output", out)
    assert r.stderr.strip() == ("error: Invalid input: dataset shapes inconsistent "
                                "(rows=1, cols=0, X=0, y=1)")


def test_cli_dataset_abi_errors(lib_built, tmp_path):
    core = lib_built
    d = tmp_path / "t.svm"
    d.write_text("1 1:0.5 3:2\n0 2:1\n")
    # LibSVM tables name their columns label, f0, f1, ... (CSV.readLibSVM)
    with pytest.raises(core.MacBoostError, match="categorical column 'f9' not found"):
        core.cli_dataset(d, tmp_path / "o.mbds", categorical="f9")
    with pytest.raises(core.MacBoostError, match="numBins must be in 4...256, got 2"):
        core.cli_dataset(d, tmp_path / "o.mbds", categorical="f0,,f2", num_bins=2)
