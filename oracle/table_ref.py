"""CPU restatement of MacBoost's CLI text readers, prediction writer and
predict command (TEST INFRASTRUCTURE ONLY).

Only tests/ import this module; the product (``macboost_b200``) never does.

* ``read_csv`` restates ``CSV.read`` (Sources/MacBoostCLI/CSV.swift:48-118) and
  ``read_libsvm`` restates ``CSV.readLibSVM`` (CSV.swift:126-217) as plain
  Python loops over the file's bytes.  Fields are converted by the C
  library's own ``strtof`` / ``strtol`` called in place on the same
  NUL-terminated buffer (through ctypes), exactly as the Swift code calls
  them, so every quirk of those functions (leading blanks, hex, inf/nan)
  is the C library's.
* ``swift_description`` restates how Swift prints a Float (shortest
  round-trip digits; exponent form below 1e-4 or above 2^24); the digits
  come from numpy's Dragon4 in "unique" mode.
* ``prediction_text`` restates ``CSV.writePredictions`` (CSV.swift:219-224)
  and the multiclass branch of ``runPredict`` (MacBoostCLI/main.swift:357-361).
* ``column_map`` restates runPredict's feature-to-column mapping
  (main.swift:327-342).
Sized for small cases (thousands of rows): pure-Python loops.
"""

from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

_libc = ctypes.CDLL(ctypes.util.find_library("c") or "libc.so.6")
_libc.strtof.restype = ctypes.c_float
_libc.strtof.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
_libc.strtol.restype = ctypes.c_long
_libc.strtol.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]

# Unicode White_Space: what Swift's CharacterSet.whitespacesAndNewlines trims
_WS = "".join(chr(c) for c in [*range(0x09, 0x0E), 0x20, 0x85, 0xA0, 0x1680,
                               *range(0x2000, 0x200B), 0x2028, 0x2029, 0x202F, 0x205F,
                               0x3000])


class TableError(Exception):
    """A reader error; str() is the message the reference prints."""


class _Buf:
    """The file's bytes + '\\n' + NUL (CSV.swift:52-53) in C memory."""

    def __init__(self, data: bytes):
        self.b = data + b"\n\0"
        self.c = ctypes.create_string_buffer(self.b, len(self.b))
        self.base = ctypes.addressof(self.c)

    def strtof(self, off: int):
        end = ctypes.c_void_p()
        v = _libc.strtof(self.base + off, ctypes.byref(end))
        return np.float32(v), end.value - self.base

    def strtol(self, off: int):
        end = ctypes.c_void_p()
        v = _libc.strtol(self.base + off, ctypes.byref(end), 10)
        return int(v), end.value - self.base


def read_csv(data: bytes):
    """CSV.read: returns (header, float32 (rows, cols)) or raises TableError."""
    buf = _Buf(data)
    b = buf.b
    n = len(b) - 1
    pos = 0
    while pos < n and b[pos] != 0x0A:
        pos += 1
    if pos >= n:
        raise TableError("Malformed CSV: no header line")
    line = b[:pos].decode("utf-8")
    delim = "\t" if "\t" in line else ","
    dbyte = ord(delim)
    header = [s.strip(_WS) for s in line.split(delim)]
    cols = len(header)
    starts = []
    p = pos + 1
    while p < n:
        if b[p] != 0x0A and b[p] != 0x0D:
            starts.append(p)
        while p < n and b[p] != 0x0A:
            p += 1
        p += 1
    rows = len(starts)
    if rows == 0:
        raise TableError("Malformed CSV: no data rows")
    out = np.full((rows, cols), np.nan, dtype=np.float32)
    bad = None
    for i, q in enumerate(starts):
        for c in range(cols):
            fs = q
            is_end = False
            while True:
                ch = b[q]
                if ch == dbyte:
                    break
                if ch == 0x0A or ch == 0x0D:
                    is_end = True
                    break
                q += 1
            if q > fs:
                v, end = buf.strtof(fs)
                if end > fs:
                    out[i, c] = v
            if is_end:
                if c + 1 < cols and bad is None:
                    bad = i
                break
            q += 1
    if bad is not None:
        raise TableError(f"Malformed CSV: row {bad + 1} has fewer fields than the header "
                         f"({cols})")
    return header, out


def _pairs(buf: _Buf, start: int):
    """forEachPair (CSV.swift:156-181): (label, [(idx, value), ...])."""
    b = buf.b
    label, q = buf.strtof(start)
    pairs = []
    while True:
        while b[q] == 0x20 or b[q] == 0x09:
            q += 1
        if b[q] in (0x0A, 0x0D, 0x23):
            break
        idx, idx_end = buf.strtol(q)
        if idx_end == q or b[idx_end] != 0x3A:
            skip = q
            while b[skip] not in (0x20, 0x09, 0x0A, 0x0D):
                skip += 1
            q = skip
            continue
        v, q = buf.strtof(idx_end + 1)
        pairs.append((idx, v))
    return label, pairs


def read_libsvm(data: bytes):
    """CSV.readLibSVM: returns (header, float32 (rows, 1 + features))."""
    buf = _Buf(data)
    b = buf.b
    n = len(b) - 1
    starts = []
    p = 0
    while p < n:
        if b[p] not in (0x0A, 0x0D, 0x23):
            starts.append(p)
        while p < n and b[p] != 0x0A:
            p += 1
        p += 1
    if not starts:
        raise TableError("Malformed CSV: no data rows")
    parsed = [_pairs(buf, s) for s in starts]
    idxs = [i for _, pr in parsed for i, _ in pr]
    max_idx = max([-1] + idxs)
    min_idx = min(idxs) if idxs else None
    if max_idx < 0:
        raise TableError("Malformed CSV: no idx:value pairs found")
    if min_idx < 0:   # the reference indexes out of bounds here; this build rejects it
        raise TableError(f"Malformed CSV: negative feature index {min_idx}")
    base = 0 if min_idx == 0 else 1
    features = max_idx - base + 1
    out = np.zeros((len(starts), features + 1), dtype=np.float32)
    for i, (label, pr) in enumerate(parsed):
        for idx, v in pr:
            out[i, 1 + idx - base] = v
        out[i, 0] = label
    return ["label"] + [f"f{k}" for k in range(features)], out


def read_table(path, fmt: str = "csv"):
    """loadTable (main.swift:98-110): fmt csv | libsvm | auto (by extension)."""
    data = open(path, "rb").read()
    ext = str(path).rsplit(".", 1)[-1].lower() if "." in str(path) else ""
    if fmt == "libsvm" or (fmt == "auto" and ext in ("svm", "libsvm")):
        return read_libsvm(data)
    return read_csv(data)


def swift_description(v) -> str:
    """How Swift prints a Float (`"\\(v)"`)."""
    v = np.float32(v)
    if np.isnan(v):
        return "nan"
    if np.isinf(v):
        return "-inf" if v < 0 else "inf"
    sign = "-" if np.signbit(v) else ""
    if v == 0:
        return sign + "0.0"
    s = np.format_float_scientific(np.abs(v), unique=True, trim="-", exp_digits=1)
    mant, e = s.split("e")
    exp10 = int(e)
    digits = mant.replace(".", "")
    dexp = exp10 + 1
    if dexp < -3 or abs(float(v)) > 2.0 ** 24:
        frac = "." + digits[1:] if len(digits) > 1 else ""
        return f"{sign}{digits[0]}{frac}e{'-' if exp10 < 0 else '+'}{abs(exp10):02d}"
    if dexp <= 0:
        return sign + "0." + "0" * (-dexp) + digits
    if dexp >= len(digits):
        return sign + digits + "0" * (dexp - len(digits)) + ".0"
    return sign + digits[:dexp] + "." + digits[dexp:]


def prediction_text(preds: np.ndarray, k: int) -> str:
    """The prediction file runPredict writes for (rows, k) float32 values."""
    p = np.asarray(preds, dtype=np.float32).reshape(-1, k)
    if k > 1:
        head = ",".join(f"class_{c}" for c in range(k))
        lines = [",".join(swift_description(x) for x in row) for row in p]
    else:
        head = "prediction"
        lines = [swift_description(x) for x in p[:, 0]]
    return head + "\n" + "".join(ln + "\n" for ln in lines)


def column_map(header, num_features: int, feature_names):
    """runPredict's columns (main.swift:327-342), or raises TableError."""
    if feature_names is not None:
        cols = []
        for name in feature_names:
            if name not in header:
                raise TableError(f"Malformed CSV: column '{name}' required by the model is "
                                 f"missing")
            cols.append(header.index(name))
        return cols
    if len(header) < num_features:
        raise TableError(f"model expects {num_features} features, CSV has {len(header)} "
                         f"columns")
    return list(range(num_features))
