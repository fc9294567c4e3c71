"""Shared fixtures for the macboost_b200 test suite.

Tests marked ``gpu`` need an sm_100 GPU and call the engine through its C ABI
(libmacboostc.so via macboost_b200._core); everything else runs on the CPU:
the oracle against the reference's golden vectors, the model loader and
flattening (no device needed), ABI exports and the host-side sharding logic.
"""

from __future__ import annotations

import gzip
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402  (test infrastructure)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def golden_names():
    return sorted(p.name[:-4] for p in GOLDEN.glob("*.npz"))


def golden_text(name: str) -> str:
    with gzip.open(GOLDEN / f"{name}.model.json.gz", "rt") as fh:
        return fh.read()


def golden_arrays(name: str) -> dict:
    d = np.load(GOLDEN / f"{name}.npz")
    return {k: d[k] for k in d.files}


def golden_oracle_model(name: str):
    return O.model_from_dict(json.loads(golden_text(name)))


@pytest.fixture(scope="session")
def lib_built():
    """Build libmacboostc.so in-tree if needed and return the _core module."""
    from macboost_b200 import build as B
    B.build()
    from macboost_b200 import _core
    return _core


@pytest.fixture(scope="session")
def oracle_built():
    O.build()
    return O


@pytest.fixture(scope="session")
def gpu(lib_built):
    """The _core module, on a machine with a usable sm_100 GPU."""
    if lib_built.device_count() < 1:
        pytest.fail("GPU test run on a machine without a visible CUDA device")
    return lib_built


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bitwise(a, b, what=""):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    diff = np.nonzero(bits(a).ravel() != bits(b).ravel())[0]
    if diff.size:
        i = diff[0]
        raise AssertionError(f"{what}: {diff.size} of {a.size} values differ bitwise; first at "
                             f"{i}: {a.ravel()[i]!r} vs {b.ravel()[i]!r}")


def assert_ulp(a, b, max_ulp=2, what=""):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    both_nan = np.isnan(a) & np.isnan(b)
    d = np.where(both_nan, 0, O.ulp_distance(a, b))
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{what}: {worst} ulp apart (limit {max_ulp})"
