"""CLI text input and output on the CPU: the library's CSV / TSV / LibSVM
readers and prediction writer against the oracle's restatement of
Sources/MacBoostCLI/CSV.swift, and the `macboost` command's argument and
error handling (everything that runs before a GPU is needed)."""

from __future__ import annotations

import json
import math
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden_text
from oracle import table_ref as T

CLI = ROOT / "macboost_b200" / "macboost"


def _same(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _check(core, tmp_path, data: bytes, fmt: str, suffix: str = ".csv"):
    p = tmp_path / f"t{suffix}"
    p.write_bytes(data)
    try:
        ref = T.read_table(p, fmt)
    except T.TableError as e:
        with pytest.raises(core.MacBoostError) as ei:
            core.read_table(p, fmt)
        assert str(ei.value) == str(e)
        return None
    names, vals = core.read_table(p, fmt)
    assert names == ref[0]
    assert _same(vals, ref[1]), f"{data!r}\n{vals}\n{ref[1]}"
    return names, vals


CSV_CASES = {
    "basic": b"a, b ,c\n1,2,3\n4,5,6\n",
    "tsv": b"a\tb\n1\t2\n3\t4\n",
    "crlf": b"a,b\r\n1,2\r\n3,4\r\n",
    "blank_and_cr_lines": b"a,b\n\n1,2\n\r\n3,4\n\n\n",
    "missing_tokens": b"a,b,c\nNA,,nan\n-inf,inf,abc\n1.5x,0x1p3,  7\n",
    "extra_fields": b"a,b\n1,2,3,4\n5,6\n",
    "short_row": b"a,b,c\n1,2,3\n4,5\n6\n",
    "no_data_rows": b"a,b\n\n\n",
    "empty_file": b"",
    "no_final_newline": b"a,b\n1,2",
    "blank_field_reads_next_line": b"a,b\n1, \n2,3\n",
    "tab_header_comma_data": b"a\tb\n1,2\t3\n",
    "number_forms": (b"a,b,c,d,e,f,g,h\n+1,.5,5.,1e5,1e,1e+,-0,00012\n"
                     b"1.5E-3,infinity,-NaN,nan(123),0x1.8p1,1e-50,3.5e38,1e39\n"),
    "trailing_delimiter": b"a,b,\n1,2,3\n",
    "quoted": b'"a","b"\n"1",2\n',
    "unicode_header": " name　,x , y\n1,2,3\n".encode(),
    "only_header_no_newline": b"a,b",
    "lone_cr_line_end": b"a,b\n1,2\r3,4\r",
}


@pytest.mark.parametrize("case", sorted(CSV_CASES))
def test_csv_cases(lib_built, tmp_path, case):
    _check(lib_built, tmp_path, CSV_CASES[case], "csv")


LIBSVM_CASES = {
    "one_based": b"1 1:0.5 3:2\n0 2:1.5\n",
    "zero_based": b"1 0:0.5 2:2\n0 1:1.5\n",
    "qid_and_comments": b"# comment\n1 qid:3 1:0.5 # trailing 9:9\n0 2:1 3:4\n",
    "crlf_blank": b"1 1:1\r\n\r\n0 2:2\r\n",
    "no_label": b"1:0.5 2:3\n",
    "no_pairs": b"1\n0\n",
    "negative_index": b"1 -1:2 3:1\n",
    "duplicate_index": b"1 2:1 2:5\n",
    "bad_value": b"1 2:abc 3:1\n",
    "min_index_five": b"1 5:1 7:2\n",
    "tabs": b"1\t1:1\t2:2\n-1\t3:3\n",
    "empty": b"",
}


@pytest.mark.parametrize("case", sorted(LIBSVM_CASES))
def test_libsvm_cases(lib_built, tmp_path, case):
    _check(lib_built, tmp_path, LIBSVM_CASES[case], "libsvm", ".svm")


def test_auto_format_by_extension(lib_built, tmp_path):
    r = _check(lib_built, tmp_path, LIBSVM_CASES["one_based"], "auto", ".libsvm")
    assert r[0][0] == "label"
    r = _check(lib_built, tmp_path, CSV_CASES["basic"], "auto", ".txt")
    assert r[0] == ["a", "b", "c"]


def test_io_errors(lib_built, tmp_path):
    core = lib_built
    for p in (tmp_path / "absent.csv", tmp_path):
        with pytest.raises(core.MacBoostError, match=r"^CSV I/O error: cannot read "):
            core.read_table(p)


def _number_strings(rng, n):
    """Numeric text in the forms tables hold, plus double-rounding traps."""
    out = []
    f = (rng.standard_normal(n) * 10.0 ** rng.integers(-12, 12, n)).astype(np.float32)
    for fmt in ("%.9g", "%.6g", "%.17g", "%e", "%.3f", "%.12e"):
        out += [fmt % x for x in f[: n // 8]]
    out += [repr(float(x)) for x in rng.standard_normal(n // 8) * 1e3]
    out += [str(int(x)) for x in rng.integers(-10**12, 10**12, n // 16)]
    out += ["%d.%0*d" % (rng.integers(0, 1000), int(k), rng.integers(0, 10**int(k)))
            for k in rng.integers(1, 18, n // 16)]
    # strings whose nearest double is exactly halfway between two float32
    pos = np.abs(f[: n // 8]).astype(np.float32)
    pos = pos[(pos > 1e-30) & (pos < 1e30)]
    nxt = np.nextafter(pos, np.float32(np.inf))
    mids = (pos.astype(np.float64) + nxt.astype(np.float64)) / 2
    out += [repr(float(m)) for m in mids]
    out += ["%.8e" % m for m in mids]
    out += ["%.15e" % m for m in mids] + ["%.16g" % m for m in mids]   # 16 digits: fast path
    return out


def test_field_conversion_matches_strtof(lib_built, tmp_path):
    """The reader's fast decimal path gives strtof's value for every string."""
    rng = np.random.default_rng(7)
    strs = _number_strings(rng, 80_000)
    p = tmp_path / "n.csv"
    p.write_text("x\n" + "\n".join(strs) + "\n")
    names, vals = lib_built.read_table(p)
    assert vals.shape == (len(strs), 1)
    ref = np.empty(len(strs), np.float32)
    for i, s in enumerate(strs):
        b = T._Buf(s.encode())
        v, end = b.strtof(0)
        ref[i] = v if end > 0 else np.nan
    bad = np.nonzero(vals[:, 0].view(np.uint32) != ref.view(np.uint32))[0]
    assert bad.size == 0, [(strs[i], vals[i, 0], ref[i]) for i in bad[:10]]


def test_random_table_roundtrip(lib_built, tmp_path):
    rng = np.random.default_rng(3)
    X = rng.standard_normal((3000, 7)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    lines = ["f0,f1,f2,f3,f4,f5,label"]
    for row in X:
        lines.append(",".join("" if math.isnan(v) else "%.9g" % v for v in row))
    data = ("\n".join(lines) + "\n").encode()
    names, vals = _check(lib_built, tmp_path, data, "csv")
    assert _same(vals, X)


def test_prediction_text(lib_built, tmp_path):
    core = lib_built
    rng = np.random.default_rng(11)
    bits = rng.integers(0, 2**32, 60_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    special = np.float32([0.0, -0.0, np.nan, np.inf, -np.inf, 1e-4, 9.9999e-5, 2**24, 2**24 + 2,
                          1e7, 1e-45, 3.4028235e38, 0.1, 1.0, 100.0, 123.25, -5e-5])
    for k, v in ((1, np.concatenate([bits, special])), (3, bits[:30_000]), (10, bits[:20_000])):
        p = tmp_path / f"p{k}.csv"
        core.write_predictions(v.reshape(-1, k) if k > 1 else v, p)
        assert p.read_text() == T.prediction_text(v, k), f"k={k}"


def _run(*args, cwd=None):
    return subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True,
                          cwd=cwd, timeout=120)


def test_cli_commands_and_flags(lib_built):
    r = _run("--version")
    assert r.returncode == 0 and r.stdout.strip() == "macboost 1.0.0"
    r = _run()
    assert r.returncode == 0 and "macboost predict" in r.stdout
    for args, msg in [(("frobnicate",), "error: unknown command 'frobnicate'"),
                      (("predict",), "error: --model is required"),
                      (("predict", "--model", "m.json"), "error: --data is required"),
                      (("predict", "model.json"), "error: unexpected argument 'model.json'"),
                      (("predict", "--model"), "error: missing value for --model"),
                      (("train", "--data", "x.csv"), "error: `macboost train` is not supported"),
                      (("predict", "--model", "m", "--data", "d", "--format", "xml"),
                       "error: unknown --format 'xml'")]:
        r = _run(*args)
        assert r.returncode == 1 and r.stderr.startswith(msg), (args, r.stderr)


def _model_with_names(tmp_path, names):
    m = json.loads(golden_text("cfg2_small"))
    m["featureNames"] = names
    p = tmp_path / "named.json"
    p.write_text(json.dumps(m))
    return p, m


def test_cli_errors_before_the_gpu(lib_built, tmp_path):
    m = json.loads(golden_text("cfg2_small"))
    F = m["numFeatures"]
    model = tmp_path / "m.json"
    model.write_text(json.dumps(m))
    # a model file that does not load
    r = _run("predict", "--model", tmp_path / "nope.json", "--data", "x.csv")
    assert r.returncode == 1 and r.stderr.startswith("error: ")
    # missing input file
    r = _run("predict", "--model", model, "--data", tmp_path / "absent.csv")
    assert r.returncode == 1
    assert r.stderr.strip() == f"error: CSV I/O error: cannot read {tmp_path / 'absent.csv'}"
    # too few columns (no feature names in the model)
    few = tmp_path / "few.csv"
    few.write_text(",".join(f"c{i}" for i in range(F - 1)) + "\n" +
                   ",".join("1" for _ in range(F - 1)) + "\n")
    r = _run("predict", "--model", model, "--data", few)
    assert r.stderr.strip() == f"error: model expects {F} features, CSV has {F - 1} columns"
    # by-name mapping: a missing column
    names = [f"feat_{i}" for i in range(F)]
    named, _ = _model_with_names(tmp_path, names)
    hdr = names[:-1] + ["other"]
    d = tmp_path / "named.csv"
    d.write_text(",".join(hdr) + "\n" + ",".join("0.5" for _ in hdr) + "\n")
    r = _run("predict", "--model", named, "--data", d)
    assert r.stderr.strip() == (f"error: Malformed CSV: column '{names[-1]}' required by the "
                                f"model is missing")
    # a short row is reported before the missing column (the table is read first)
    d.write_text(",".join(hdr) + "\n" + ",".join("0.5" for _ in hdr) + "\n1,2\n")
    r = _run("predict", "--model", named, "--data", d)
    assert r.stderr.strip() == (f"error: Malformed CSV: row 2 has fewer fields than the header "
                                f"({len(hdr)})")
    # the oracle's column mapping gives the same verdicts
    with pytest.raises(T.TableError, match="required by the model is missing"):
        T.column_map(hdr, F, names)
    assert T.column_map(["x"] + names, F, names) == list(range(1, F + 1))


def test_cli_importance(lib_built, tmp_path):
    core = lib_built
    F = json.loads(golden_text("cfg3_small"))["numFeatures"]
    names = [f"n{i}" for i in range(F)]
    m = json.loads(golden_text("cfg3_small"))
    m["featureNames"] = names
    p = tmp_path / "m.json"
    p.write_text(json.dumps(m))
    r = _run("importance", "--model", p)
    assert r.returncode == 0, r.stderr
    h = core.load(p)
    assert core.feature_names(h) == names
    gain = core.feature_importance(h, "gain")
    split = core.feature_importance(h, "split")
    order = sorted(range(F), key=lambda i: -gain[i])      # stable, by gain descending
    want = ["feature".ljust(24) + "gain".ljust(14) + "splits"]
    want += [names[i].ljust(24) + ("%.1f" % gain[i]).ljust(14) + "%.0f" % split[i]
             for i in order]
    assert r.stdout.splitlines() == want
