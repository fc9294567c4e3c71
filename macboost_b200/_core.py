"""ctypes bridge to libmacboostc.so, the B200 inference engine's C ABI.

Mirrors the predict subset of MacBoost's python/macboost/_core.py (library
discovery through ``MACBOOST_LIB``, ``MacBoostError``, ``_take_error``,
``_feature_major``, ``_Handle``, ``load`` / ``predict`` / getters) and adds
the engine's additive entry points (output kinds, device lists, row-major and
device-resident input, pinned host buffers).  No PyTorch, no CPU fallback: a
missing library raises ``OSError``, and predicting without a B200 raises
``MacBoostError`` from the library.
"""

from __future__ import annotations

import ctypes
import os
import weakref
from pathlib import Path

import numpy as np

KIND_PREDICT, KIND_RAW, KIND_PROBA, KIND_LEAF, KIND_CLI = 0, 1, 2, 3, 4
LAYOUT_FEATURE_MAJOR, LAYOUT_ROW_MAJOR = 0, 1
FORMATS = {"csv": 0, "tsv": 0, "libsvm": 1, "auto": 2}

_PKG = Path(__file__).resolve().parent


def _find_library() -> str:
    """MACBOOST_LIB, else the in-tree build (python -m macboost_b200.build)."""
    candidates = []
    if env := os.environ.get("MACBOOST_LIB"):
        candidates.append(Path(env))
    candidates.append(_PKG / "libmacboostc.so")
    for c in candidates:
        if c.is_file():
            return str(c)
    raise OSError("libmacboostc.so not found. Build it with `python -m macboost_b200.build` "
                  "or set MACBOOST_LIB.")


_c_char_pp = ctypes.POINTER(ctypes.c_char_p)
_f32_p = ctypes.POINTER(ctypes.c_float)
_i32_p = ctypes.POINTER(ctypes.c_int32)
_lib_instance = None


def _configure(lib):
    P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    sig = {
        "macboost_load": (P, [ctypes.c_char_p, _c_char_pp]),
        "macboost_load_json": (P, [ctypes.c_char_p, I64, _c_char_pp]),
        "macboost_predict": (I32, [P, _f32_p, I64, I64, _f32_p, _c_char_pp]),
        "macboost_predict_ex": (I32, [P, P, I64, I64, I32, I32, _i32_p, I32, P, _c_char_pp]),
        "macboost_predict_device": (I32, [P, I32, P, I64, I64, I64, I32, I32, P, P, _c_char_pp]),
        "macboost_prepare": (I32, [P, _i32_p, I32, _c_char_pp]),
        "macboost_check_device": (I32, [P, I32, _c_char_pp]),
        "macboost_num_classes": (I64, [P]),
        "macboost_num_trees": (I64, [P]),
        "macboost_num_features": (I64, [P]),
        "macboost_best_iteration": (I64, [P]),
        "macboost_output_cols": (I64, [P, I32]),
        "macboost_warnings": (P, [P]),
        "macboost_feature_importance": (I32, [P, I32, _f32_p]),
        "macboost_save": (I32, [P, ctypes.c_char_p, _c_char_pp]),
        "macboost_free": (None, [P]),
        "macboost_free_string": (None, [ctypes.c_char_p]),
        "macboost_describe": (P, [P]),
        "macboost_device_count": (I32, []),
        "macboost_kernel_launches": (ctypes.c_uint64, []),
        "macboost_host_alloc": (P, [I64]),
        "macboost_host_free": (None, [P]),
        "macboost_predict_contrib": (I32, [P, _f32_p, I64, I64, _f32_p, _c_char_pp]),
        "macboost_predict_contrib_ex": (I32, [P, P, I64, I64, I32, _i32_p, I32, P, _c_char_pp]),
        "macboost_predict_contrib_device": (I32, [P, I32, P, I64, I64, I64, I32, P, P,
                                                  _c_char_pp]),
        "macboost_bin_data": (I32, [P, I64, I64, I32, P, I32, P, I32, P, _c_char_pp]),
        "macboost_bin_data_device": (I32, [P, I64, I64, I64, I32, P, I32, P, I32, P, P,
                                           _c_char_pp]),
        "macboost_predict_tree_binned": (I32, [P, I64, I64, I32, I32, P, P, P, P, P, P, I32,
                                               I32, I32, P, P, _c_char_pp]),
        "macboost_predict_tree_binned_device": (I32, [P, I64, I64, I32, I32, P, P, P, P, P, P,
                                                      I32, I32, I32, P, P, P, P, _c_char_pp]),
        "macboost_dataset_load": (P, [ctypes.c_char_p, _c_char_pp]),
        "macboost_dataset_rows": (I64, [P]),
        "macboost_dataset_cols": (I64, [P]),
        "macboost_dataset_num_bins": (I32, [P]),
        "macboost_dataset_bins": (P, [P]),
        "macboost_dataset_edges": (P, [P]),
        "macboost_dataset_labels": (P, [P]),
        "macboost_dataset_num_categorical": (I64, [P]),
        "macboost_dataset_categorical": (I64, [P, I64]),
        "macboost_dataset_num_feature_names": (I64, [P]),
        "macboost_dataset_feature_name": (ctypes.c_char_p, [P, I64]),
        "macboost_dataset_free": (None, [P]),
        "macboost_predict_dataset": (I32, [P, P, I32, _i32_p, I32, P, _c_char_pp]),
        "macboost_dataset_make": (P, [P, I64, I64, P, I32, ctypes.POINTER(I64), I64,
                                      ctypes.POINTER(ctypes.c_char_p), I32, _c_char_pp]),
        "macboost_dataset_save": (I32, [P, ctypes.c_char_p, _c_char_pp]),
        "macboost_cli_dataset": (I32, [ctypes.c_char_p, I32, ctypes.c_char_p, ctypes.c_char_p,
                                       I32, I32, ctypes.c_char_p, ctypes.POINTER(I64),
                                       ctypes.POINTER(I64), _c_char_pp]),
        "macboost_num_feature_names": (I64, [P]),
        "macboost_feature_name": (ctypes.c_char_p, [P, I64]),
        "macboost_table_read": (P, [ctypes.c_char_p, I32, _c_char_pp]),
        "macboost_table_rows": (I64, [P]),
        "macboost_table_cols": (I64, [P]),
        "macboost_table_column_name": (ctypes.c_char_p, [P, I64]),
        "macboost_table_data": (P, [P]),
        "macboost_table_free": (None, [P]),
        "macboost_write_predictions": (I32, [P, I64, I64, ctypes.c_char_p, _c_char_pp]),
        "macboost_cli_predict": (I32, [P, ctypes.c_char_p, I32, I32, _i32_p, I32,
                                       ctypes.c_char_p, ctypes.POINTER(I64), _c_char_pp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


class _LazyLib:
    def __getattr__(self, name):
        global _lib_instance
        if _lib_instance is None:
            lib = ctypes.CDLL(_find_library())
            _configure(lib)
            _lib_instance = lib
        return getattr(_lib_instance, name)


_lib = _LazyLib()


def native_available() -> bool:
    try:
        _lib.macboost_num_trees  # noqa: B018 -- probe the load
        return True
    except OSError:
        return False


def library_path() -> str:
    return _find_library()


class MacBoostError(RuntimeError):
    pass


def _take_error(err: ctypes.c_char_p) -> str:
    msg = err.value.decode() if err.value else "unknown error"
    _lib.macboost_free_string(err)
    return msg


def _feature_major(X) -> tuple[np.ndarray, int, int]:
    """(n, f) array-like -> contiguous feature-major float32 + (rows, cols)."""
    a = np.asarray(X, dtype=np.float32)
    if a.ndim != 2:
        raise ValueError(f"X must be 2-dimensional, got shape {a.shape}")
    rows, cols = a.shape
    return np.ascontiguousarray(a.T), rows, cols


def _f32(a: np.ndarray):
    return a.ctypes.data_as(_f32_p)


class _Handle:
    """Owns a model handle and frees it on GC."""

    def __init__(self, ptr: int):
        self.ptr = ptr

    def __del__(self):
        if getattr(self, "ptr", None):
            try:
                _lib.macboost_free(self.ptr)
            except (AttributeError, TypeError):
                pass  # interpreter shutdown: module globals already cleared
            self.ptr = None


def load(path) -> _Handle:
    err = ctypes.c_char_p()
    ptr = _lib.macboost_load(str(path).encode(), ctypes.byref(err))
    if not ptr:
        raise MacBoostError(_take_error(err))
    return _Handle(ptr)


def load_json(text: str | bytes) -> _Handle:
    data = text.encode() if isinstance(text, str) else bytes(text)
    err = ctypes.c_char_p()
    ptr = _lib.macboost_load_json(data, len(data), ctypes.byref(err))
    if not ptr:
        raise MacBoostError(_take_error(err))
    return _Handle(ptr)


def num_classes(handle: _Handle) -> int:
    return _lib.macboost_num_classes(handle.ptr)


def num_trees(handle: _Handle) -> int:
    return _lib.macboost_num_trees(handle.ptr)


def num_features(handle: _Handle) -> int:
    return _lib.macboost_num_features(handle.ptr)


def best_iteration(handle: _Handle) -> int:
    return _lib.macboost_best_iteration(handle.ptr)


def output_cols(handle: _Handle, kind: int) -> int:
    return _lib.macboost_output_cols(handle.ptr, kind)


def describe(handle: _Handle) -> str:
    p = _lib.macboost_describe(handle.ptr)
    s = ctypes.string_at(p).decode()
    _lib.macboost_free_string(ctypes.cast(p, ctypes.c_char_p))
    return s


def device_count() -> int:
    return _lib.macboost_device_count()


def kernel_launches() -> int:
    return _lib.macboost_kernel_launches()


def predict(handle: _Handle, X) -> np.ndarray:
    """The reference binding's predict (_core.py:210-220): feature-major copy
    of X through macboost_predict; (rows,) for one class else (rows, K)."""
    Xf, rows, cols = _feature_major(X)
    k = _lib.macboost_num_classes(handle.ptr)
    out = np.empty(rows * k, dtype=np.float32)
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict(handle.ptr, _f32(Xf), rows, cols, _f32(out), ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))
    return out.reshape(rows, k) if k > 1 else out


def predict_contrib(handle: _Handle, X) -> np.ndarray:
    """The reference binding's predict_contrib (_core.py:222-231): SHAP
    contributions, (rows, K * (cols + 1)) float32; per class the cols
    contributions then the expected value."""
    Xf, rows, cols = _feature_major(X)
    k = _lib.macboost_num_classes(handle.ptr)
    out = np.empty(rows * k * (cols + 1), dtype=np.float32)
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict_contrib(handle.ptr, _f32(Xf), rows, cols, _f32(out),
                                       ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))
    return out.reshape(rows, k * (cols + 1))


def predict_contrib_ex(handle: _Handle, X, layout: str = "row", devices=None) -> np.ndarray:
    """SHAP contributions with the input layout and device list of predict_ex."""
    a = np.asarray(X, dtype=np.float32)
    if a.ndim != 2:
        raise ValueError(f"X must be 2-dimensional, got shape {a.shape}")
    a = np.ascontiguousarray(a)
    if layout == "row":
        rows, cols = a.shape
        lay = LAYOUT_ROW_MAJOR
    elif layout == "feature":
        cols, rows = a.shape
        lay = LAYOUT_FEATURE_MAJOR
    else:
        raise ValueError("layout must be 'row' or 'feature'")
    k = _lib.macboost_num_classes(handle.ptr)
    out = np.empty((rows, k * (cols + 1)), dtype=np.float32)
    devs = None
    nd = 0
    if devices:
        devs = (ctypes.c_int32 * len(devices))(*devices)
        nd = len(devices)
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict_contrib_ex(handle.ptr, a.ctypes.data, rows, cols, lay, devs, nd,
                                          out.ctypes.data, ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))
    return out


def predict_contrib_device(handle: _Handle, device: int, x_ptr: int, rows: int, cols: int,
                           ld: int, out_ptr: int, layout: int = LAYOUT_FEATURE_MAJOR,
                           stream: int = 0) -> None:
    """Enqueue SHAP contributions on device buffers (raw pointers) on `stream`."""
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict_contrib_device(handle.ptr, device, x_ptr, rows, cols, ld, layout,
                                              out_ptr, stream or None, ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))


def predict_ex(handle: _Handle, X, kind: int = KIND_PREDICT, layout: str = "row",
               devices=None, out: np.ndarray | None = None) -> np.ndarray:
    """Predict with an explicit output kind.

    layout="row": X is (rows, F), passed without a host-side transpose (the
    GPU transposes); layout="feature": X is (F, rows) feature-major.  Returns
    (rows, output_cols(kind)) float32, or int32 for KIND_LEAF."""
    a = np.asarray(X, dtype=np.float32)
    if a.ndim != 2:
        raise ValueError(f"X must be 2-dimensional, got shape {a.shape}")
    a = np.ascontiguousarray(a)
    if layout == "row":
        rows, cols = a.shape
        lay = LAYOUT_ROW_MAJOR
    elif layout == "feature":
        cols, rows = a.shape
        lay = LAYOUT_FEATURE_MAJOR
    else:
        raise ValueError("layout must be 'row' or 'feature'")
    ncol = _lib.macboost_output_cols(handle.ptr, kind)
    if ncol < 0:
        raise ValueError(f"unknown output kind {kind}")
    dt = np.int32 if kind == KIND_LEAF else np.float32
    if out is None:
        out = np.empty((rows, ncol), dtype=dt)
    elif out.dtype != dt or out.size < rows * ncol or not out.flags.c_contiguous:
        raise ValueError("out has the wrong dtype, size or layout")
    devs = None
    nd = 0
    if devices:
        devs = (ctypes.c_int32 * len(devices))(*devices)
        nd = len(devices)
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict_ex(handle.ptr, a.ctypes.data, rows, cols, lay, kind, devs, nd,
                                  out.ctypes.data, ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))
    return out


def predict_device(handle: _Handle, device: int, x_ptr: int, rows: int, cols: int, ld: int,
                   out_ptr: int, kind: int = KIND_RAW, layout: int = LAYOUT_FEATURE_MAJOR,
                   stream: int = 0) -> None:
    """Enqueue a predict on device buffers (raw pointers) on `stream`."""
    err = ctypes.c_char_p()
    rc = _lib.macboost_predict_device(handle.ptr, device, x_ptr, rows, cols, ld, layout, kind,
                                      out_ptr, stream or None, ctypes.byref(err))
    if rc != 0:
        raise MacBoostError(_take_error(err))


def prepare(handle: _Handle, devices=None) -> None:
    devs = None
    nd = 0
    if devices:
        devs = (ctypes.c_int32 * len(devices))(*devices)
        nd = len(devices)
    err = ctypes.c_char_p()
    if _lib.macboost_prepare(handle.ptr, devs, nd, ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


def check_device(handle: _Handle, device: int) -> None:
    err = ctypes.c_char_p()
    if _lib.macboost_check_device(handle.ptr, device, ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


def feature_importance(handle: _Handle, importance_type: str) -> np.ndarray:
    n = _lib.macboost_num_features(handle.ptr)
    out = np.empty(n, dtype=np.float32)
    t = 1 if importance_type == "split" else 0
    if _lib.macboost_feature_importance(handle.ptr, t, _f32(out)) != 0:
        raise MacBoostError("feature_importance failed")
    return out


def save(handle: _Handle, path) -> None:
    err = ctypes.c_char_p()
    if _lib.macboost_save(handle.ptr, str(path).encode(), ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """A numpy array in page-locked host memory (freed with the array)."""
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    ptr = _lib.macboost_host_alloc(max(nbytes, 1))
    if not ptr:
        raise MacBoostError(f"cannot allocate {nbytes} bytes of page-locked host memory")
    buf = (ctypes.c_byte * max(nbytes, 1)).from_address(ptr)
    arr = np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)
    weakref.finalize(buf, _lib.macboost_host_free, ptr)
    return arr


def feature_names(handle: _Handle) -> list[str] | None:
    """The model file's `featureNames`, or None when it has none."""
    n = _lib.macboost_num_feature_names(handle.ptr)
    if n < 0:
        return None
    return [_lib.macboost_feature_name(handle.ptr, i).decode() for i in range(n)]


def _format_code(fmt: str) -> int:
    try:
        return FORMATS[fmt]
    except KeyError:
        raise ValueError(f"unknown format {fmt!r} (csv | tsv | libsvm | auto)") from None


def read_table(path, fmt: str = "csv") -> tuple[list[str], np.ndarray]:
    """A CSV / TSV / LibSVM file read with the CLI's rules: (column names,
    float32 (rows, cols) row-major copy)."""
    err = ctypes.c_char_p()
    t = _lib.macboost_table_read(str(path).encode(), _format_code(fmt), ctypes.byref(err))
    if not t:
        raise MacBoostError(_take_error(err))
    try:
        rows = _lib.macboost_table_rows(t)
        cols = _lib.macboost_table_cols(t)
        names = [_lib.macboost_table_column_name(t, c).decode() for c in range(cols)]
        out = np.empty((rows, cols), dtype=np.float32)
        if out.size:
            ctypes.memmove(out.ctypes.data, _lib.macboost_table_data(t), out.nbytes)
        return names, out
    finally:
        _lib.macboost_table_free(t)


def write_predictions(preds, path) -> None:
    """The CLI's prediction file for (rows,) or (rows, k) float32 values."""
    p = np.ascontiguousarray(preds, dtype=np.float32)
    rows = p.shape[0]
    k = 1 if p.ndim == 1 else int(np.prod(p.shape[1:]))
    err = ctypes.c_char_p()
    if _lib.macboost_write_predictions(p.ctypes.data if p.size else None, rows, max(k, 1),
                                       str(path).encode(), ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


def cli_predict(handle: _Handle, data_path, output_path, fmt: str = "csv", raw: bool = False,
                devices=None) -> int:
    """`macboost predict` on an open model: returns the rows written."""
    devs = None
    nd = 0
    if devices:
        devs = (ctypes.c_int32 * len(devices))(*devices)
        nd = len(devices)
    rows = ctypes.c_int64(0)
    err = ctypes.c_char_p()
    if _lib.macboost_cli_predict(handle.ptr, str(data_path).encode(), _format_code(fmt),
                                 1 if raw else 0, devs, nd, str(output_path).encode(),
                                 ctypes.byref(rows), ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))
    return rows.value


def cli_dataset(data_path, output_path, label: str | None = None, categorical: str | None = None,
                num_bins: int = 256, fmt: str = "auto", device: int = 0) -> tuple[int, int]:
    """`macboost dataset`: bin a table into a .mbds file; returns (rows, features)."""
    rows, cols = ctypes.c_int64(0), ctypes.c_int64(0)
    err = ctypes.c_char_p()
    if _lib.macboost_cli_dataset(str(data_path).encode(), _format_code(fmt),
                                 label.encode() if label is not None else None,
                                 categorical.encode() if categorical is not None else None,
                                 int(num_bins), int(device), str(output_path).encode(),
                                 ctypes.byref(rows), ctypes.byref(cols), ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))
    return rows.value, cols.value


# ---- binned data (the trainer's tiled bin layout) -------------------------

def bin_data(X, edges, num_bins: int, categorical=(), layout: str = "row",
             device: int = 0) -> np.ndarray:
    """Tiled uint8 bins of X (ceil(F/8) * 8 * rows bytes) on `device`."""
    a = np.ascontiguousarray(np.asarray(X, dtype=np.float32))
    if a.ndim != 2:
        raise ValueError(f"X must be 2-dimensional, got shape {a.shape}")
    if layout == "row":
        rows, cols = a.shape
        lay = LAYOUT_ROW_MAJOR
    else:
        cols, rows = a.shape
        lay = LAYOUT_FEATURE_MAJOR
    e = np.ascontiguousarray(edges, dtype=np.float32)
    if e.size != cols * (num_bins - 2):
        raise ValueError(f"edges must hold cols * (num_bins - 2) = {cols * (num_bins - 2)} values")
    cat = np.zeros(cols, np.uint8)
    cat[list(categorical)] = 1
    out = np.empty(((cols + 7) // 8) * 8 * rows, dtype=np.uint8)
    err = ctypes.c_char_p()
    if _lib.macboost_bin_data(a.ctypes.data, rows, cols, lay, e.ctypes.data, num_bins,
                              cat.ctypes.data, device, out.ctypes.data, ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))
    return out


def predict_tree_binned(bins, rows: int, cols: int, num_bins: int, tree_off, feature, split_bin,
                        flags, catmask, leaf, max_depth: int, num_classes: int = 1, preds=None,
                        want_leaf: bool = False, device: int = 0):
    """predict_tree_binned / assign_leaves for every tree in order: updates the
    class-major float32 preds (num_classes x rows) in place and returns the
    tree-major int32 leaf indices (num_trees x rows) when asked."""
    arrs = [np.ascontiguousarray(bins, np.uint8), np.ascontiguousarray(tree_off, np.int64),
            np.ascontiguousarray(feature, np.int32), np.ascontiguousarray(split_bin, np.uint32),
            np.ascontiguousarray(flags, np.uint32), np.ascontiguousarray(catmask, np.uint32),
            np.ascontiguousarray(leaf, np.float32)]
    T = len(arrs[1]) - 1
    if preds is not None and (preds.dtype != np.float32 or not preds.flags.c_contiguous
                              or preds.size != num_classes * rows):
        raise ValueError("preds must be a contiguous float32 array of num_classes * rows")
    li = np.empty((T, rows), np.int32) if want_leaf else None
    err = ctypes.c_char_p()
    if _lib.macboost_predict_tree_binned(
            *[arrs[0].ctypes.data], rows, cols, num_bins, T,
            *[a.ctypes.data for a in arrs[1:]], max_depth, num_classes, device,
            preds.ctypes.data if preds is not None else None,
            li.ctypes.data if li is not None else None, ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))
    return li


def bin_data_device(x_ptr: int, rows: int, cols: int, ld: int, layout: int, edges_ptr: int,
                    num_bins: int, categorical_ptr: int, device: int, bins_ptr: int,
                    stream: int = 0) -> None:
    """macboost_bin_data_device: device pointers, enqueued on `stream`."""
    err = ctypes.c_char_p()
    if _lib.macboost_bin_data_device(x_ptr, rows, cols, ld, layout, edges_ptr, num_bins,
                                     categorical_ptr, device, bins_ptr, stream or None,
                                     ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


def predict_tree_binned_device(bins_ptr: int, rows: int, cols: int, num_bins: int,
                               num_trees: int, tree_off_ptr: int, feature_ptr: int,
                               split_bin_ptr: int, flags_ptr: int, catmask_ptr: int,
                               leaf_ptr: int, max_depth: int, num_classes: int, device: int,
                               preds_ptr: int, leaf_idx_ptr: int, status_ptr: int,
                               stream: int = 0) -> None:
    """macboost_predict_tree_binned_device: every pointer is device memory; the
    walk is enqueued on `stream` and a bad split ORs 2 into the status word."""
    err = ctypes.c_char_p()
    if _lib.macboost_predict_tree_binned_device(
            bins_ptr, rows, cols, num_bins, num_trees, tree_off_ptr, feature_ptr,
            split_bin_ptr, flags_ptr, catmask_ptr, leaf_ptr, max_depth, num_classes, device,
            preds_ptr or None, leaf_idx_ptr or None, status_ptr, stream or None,
            ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))


class Dataset:
    """A MacBoost binned dataset (.mbds) held by the library: loaded from a
    file (`Dataset(path)`) or binned from a matrix (`Dataset.make`)."""

    def __init__(self, path=None, _ptr=None):
        if _ptr is None:
            err = ctypes.c_char_p()
            _ptr = _lib.macboost_dataset_load(str(path).encode(), ctypes.byref(err))
            if not _ptr:
                raise MacBoostError(_take_error(err))
        self.ptr = _ptr
        self.rows = _lib.macboost_dataset_rows(self.ptr)
        self.cols = _lib.macboost_dataset_cols(self.ptr)
        self.num_bins = _lib.macboost_dataset_num_bins(self.ptr)

    def _array(self, fn, dtype, n):
        out = np.empty(n, dtype)
        if n:
            ctypes.memmove(out.ctypes.data, fn(self.ptr), out.nbytes)
        return out

    @property
    def bins(self) -> np.ndarray:
        return self._array(_lib.macboost_dataset_bins, np.uint8,
                           ((self.cols + 7) // 8) * 8 * self.rows)

    @property
    def edges(self) -> np.ndarray:
        return self._array(_lib.macboost_dataset_edges, np.float32,
                           self.cols * (self.num_bins - 2))

    @property
    def labels(self) -> np.ndarray:
        return self._array(_lib.macboost_dataset_labels, np.float32, self.rows)

    @property
    def categorical(self) -> list[int]:
        n = _lib.macboost_dataset_num_categorical(self.ptr)
        return [_lib.macboost_dataset_categorical(self.ptr, i) for i in range(n)]

    @property
    def feature_names(self) -> list[str] | None:
        n = _lib.macboost_dataset_num_feature_names(self.ptr)
        if n < 0:
            return None
        return [_lib.macboost_dataset_feature_name(self.ptr, i).decode() for i in range(n)]

    @classmethod
    def make(cls, X, labels, num_bins: int = 256, categorical=(), feature_names=None,
             layout: str = "row", device: int = 0) -> "Dataset":
        """MacBooster.makeDataset: quantile edges, validation and GPU binning."""
        a = np.asarray(X, dtype=np.float32)
        if a.ndim != 2:
            raise ValueError("X must be 2-D")
        fm = np.ascontiguousarray(a.T if layout == "row" else a)
        cols, rows = fm.shape
        y = np.ascontiguousarray(np.asarray(labels, dtype=np.float32).reshape(-1))
        if y.shape[0] != rows:
            raise ValueError(f"labels hold {y.shape[0]} values for {rows} rows")
        cats = list(categorical)
        carr = (ctypes.c_int64 * max(1, len(cats)))(*cats)
        names = None
        if feature_names is not None:
            if len(feature_names) != cols:
                raise ValueError(f"{len(feature_names)} feature names for {cols} features")
            names = (ctypes.c_char_p * cols)(*[str(n).encode() for n in feature_names])
        err = ctypes.c_char_p()
        ptr = _lib.macboost_dataset_make(fm.ctypes.data, rows, cols, y.ctypes.data,
                                         int(num_bins), carr, len(cats), names, int(device),
                                         ctypes.byref(err))
        if not ptr:
            raise MacBoostError(_take_error(err))
        return cls(_ptr=ptr)

    def save(self, path) -> None:
        """BinnedDataset.save: the .mbds bytes the reference writes."""
        err = ctypes.c_char_p()
        if _lib.macboost_dataset_save(self.ptr, str(path).encode(), ctypes.byref(err)) != 0:
            raise MacBoostError(_take_error(err))

    def __del__(self):
        if getattr(self, "ptr", None):
            try:
                _lib.macboost_dataset_free(self.ptr)
            except (AttributeError, TypeError):
                pass  # interpreter shutdown: module globals already cleared
            self.ptr = None


def predict_dataset(handle: _Handle, dataset: Dataset, kind: int = KIND_PREDICT,
                    devices=None) -> np.ndarray:
    """A model's output of `kind` on every row of a binned dataset."""
    ncol = _lib.macboost_output_cols(handle.ptr, kind)
    if ncol < 0:
        raise ValueError(f"unknown output kind {kind}")
    out = np.empty((dataset.rows, ncol), dtype=np.int32 if kind == KIND_LEAF else np.float32)
    devs = None
    nd = 0
    if devices:
        devs = (ctypes.c_int32 * len(devices))(*devices)
        nd = len(devices)
    err = ctypes.c_char_p()
    if _lib.macboost_predict_dataset(handle.ptr, dataset.ptr, kind, devs, nd, out.ctypes.data,
                                     ctypes.byref(err)) != 0:
        raise MacBoostError(_take_error(err))
    return out
