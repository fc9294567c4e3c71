"""MacBoost's own Python package binds to libmacboostc.so unchanged.

The package comes from MACBOOST_REFERENCE_ROOT (a MacBoost source tree, whose
``python/`` directory is imported) or, when that is unset, from baseline/_ref
(the reference's package installed unmodified with pip); the tests skip when
neither is present, and no other test needs the reference.  Its ctypes bridge
(python/macboost/_core.py:_configure) declares every entry point of the
reference ABI, so loading succeeds only if this library exports them all with
the names it expects; MacBoostClassifier.load_model -> predict_proba then
reaches macboost_predict on the GPU (or fails loudly without one).
"""

import os
import subprocess
import sys

import pytest

from conftest import GOLDEN, ROOT, golden_arrays

def _package_dir():
    ref = os.environ.get("MACBOOST_REFERENCE_ROOT")
    if ref:
        return os.path.join(ref, "python")
    installed = ROOT / "baseline" / "_ref"
    if (installed / "macboost" / "_core.py").exists():
        return str(installed)
    return None


PKG = _package_dir()

pytestmark = pytest.mark.skipif(PKG is None, reason="the reference Python package is not "
                                "available (MACBOOST_REFERENCE_ROOT unset, baseline/_ref empty)")

SCRIPT = r"""
import gzip, sys, tempfile
import numpy as np
sys.path.insert(0, sys.argv[1])
from macboost import _core, MacBoostClassifier
assert _core.native_available()
text = gzip.open(sys.argv[2], "rt").read()
p = tempfile.mktemp(suffix=".json")
open(p, "w").write(text)
m = MacBoostClassifier.load_model(p)
assert m.n_trees_ == 100 and m.n_features_in_ == 28
X = np.load(sys.argv[3])["X"]
try:
    proba = m.predict_proba(X)
except Exception as e:
    print("NO_GPU", type(e).__name__, e)
else:
    np.save(sys.argv[4], proba)
    print("OK")
"""


def _run(lib, tmp_path):
    out = tmp_path / "proba.npy"
    env = dict(os.environ, MACBOOST_LIB=lib.library_path())
    r = subprocess.run([sys.executable, "-c", SCRIPT, PKG,
                        str(GOLDEN / "cfg2_small.model.json.gz"),
                        str(GOLDEN / "cfg2_small.npz"), str(out)],
                       env=env, capture_output=True, text=True, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    return r, out


def _check_gpu_result(r, out):
    import numpy as np
    assert r.stdout.strip().endswith("OK"), r.stdout
    # the reference's float64 predict_proba on the margins this library
    # returned through macboost_predict, against the golden values from the
    # reference's own PyModel: the margins are bit-identical, so the
    # probabilities agree to float64 rounding
    assert np.allclose(np.load(out), golden_arrays("cfg2_small")["proba"], rtol=0, atol=1e-6)


def test_reference_package_binds(lib_built, tmp_path):
    r, out = _run(lib_built, tmp_path)
    if lib_built.device_count() > 0:
        _check_gpu_result(r, out)
    else:
        assert "NO_GPU MacBoostError" in r.stdout and "CUDA" in r.stdout, r.stdout


@pytest.mark.gpu
def test_reference_package_predicts_on_gpu(gpu, tmp_path):
    """The unmodified reference bridge predicting on the B200 through this
    library (MacBoostClassifier.load_model -> predict_proba)."""
    r, out = _run(gpu, tmp_path)
    _check_gpu_result(r, out)
