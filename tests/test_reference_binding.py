"""MacBoost's own Python package binds to libmacboostc.so unchanged.

Runs only when MACBOOST_REFERENCE_ROOT points at a MacBoost source tree (its
``python/`` directory is imported); the reference is never needed by the other
tests.  Its ctypes bridge (python/macboost/_core.py:_configure) declares every
entry point of the reference ABI, so loading succeeds only if this library
exports them all with the names it expects; predict_proba then reaches
macboost_predict on the GPU (or fails loudly without one).
"""

import os
import subprocess
import sys

import pytest

from conftest import GOLDEN, ROOT, golden_arrays

REF = os.environ.get("MACBOOST_REFERENCE_ROOT")

pytestmark = pytest.mark.skipif(not REF, reason="MACBOOST_REFERENCE_ROOT not set")

SCRIPT = r"""
import gzip, sys, tempfile
import numpy as np
sys.path.insert(0, sys.argv[1] + "/python")
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


def test_reference_package_binds(lib_built, tmp_path):
    out = tmp_path / "proba.npy"
    env = dict(os.environ, MACBOOST_LIB=lib_built.library_path())
    r = subprocess.run([sys.executable, "-c", SCRIPT, REF,
                        str(GOLDEN / "cfg2_small.model.json.gz"),
                        str(GOLDEN / "cfg2_small.npz"), str(out)],
                       env=env, capture_output=True, text=True, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    if lib_built.device_count() > 0:
        import numpy as np
        assert r.stdout.strip().endswith("OK"), r.stdout
        assert np.allclose(np.load(out), golden_arrays("cfg2_small")["proba"], rtol=0,
                           atol=1e-6)
    else:
        assert "NO_GPU MacBoostError" in r.stdout and "CUDA" in r.stdout, r.stdout
