"""The C-ABI library loads and exports every entry point include/macboost_c.h
declares, and nothing on the product path depends on PyTorch or the oracle."""

import ctypes
import re
import subprocess
import sys

from conftest import ROOT

HEADER = ROOT / "include" / "macboost_c.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(macboost_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_reference_entry_points():
    names = declared_functions()
    # the reference ABI's names (Sources/MacBoostC/CAPI.swift @_cdecl list)
    for n in ("macboost_load", "macboost_predict", "macboost_num_classes", "macboost_num_trees",
              "macboost_num_features", "macboost_best_iteration", "macboost_warnings",
              "macboost_feature_importance", "macboost_save", "macboost_free",
              "macboost_free_string", "macboost_train", "macboost_select_features",
              "macboost_predict_contrib"):
        assert n in names, n


def test_library_exports_every_declared_symbol(lib_built):
    lib = ctypes.CDLL(lib_built.library_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_only_macboost_symbols_exported(lib_built):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_built.library_path()],
                         capture_output=True, text=True, check=True).stdout
    names = [ln.split()[-1] for ln in out.splitlines() if ln.strip()]
    stray = [n for n in names if not n.startswith("macboost_")]
    assert not stray, stray[:10]


def test_library_has_sm100a_code_and_no_torch(lib_built):
    out = subprocess.run(["ldd", lib_built.library_path()], capture_output=True,
                         text=True).stdout
    assert "torch" not in out and "libcudart" not in out  # static runtime, no PyTorch
    code = ("import sys; sys.path.insert(0, %r); import macboost_b200, macboost_b200._core as c;"
            "c.native_available(); print('torch' in sys.modules, 'oracle' in sys.modules)"
            % str(ROOT))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
    assert r.stdout.split() == ["False", "False"]


def test_predict_without_gpu_fails_loudly(lib_built):
    """No CPU fallback: without a usable GPU a predict raises."""
    import numpy as np
    from conftest import golden_text
    core = lib_built
    if core.device_count() > 0:
        import pytest
        pytest.skip("a GPU is visible")
    h = core.load_json(golden_text("cfg1_small"))
    try:
        core.predict(h, np.zeros((8, 100), np.float32))
    except core.MacBoostError as e:
        assert "CUDA" in str(e) or "device" in str(e)
    else:
        raise AssertionError("predict succeeded without a GPU")
