"""Bounded device waits that run out, and the error they report.

Every mbarrier wait of the forest kernels gives up after a limit
(MACBOOST_WAIT_LIMIT_US, 2 s by default), records kErrWaitTimeout in the
status word, drains the copies its CTA or warp still has in flight and
returns; the host reports -1 with a message through the reference's error
channel (Sources/MacBoostC/CAPI.swift:77-80).  The test hook
MACBOOST_TEST_STALL_TILES=1 makes the row-tile barriers expect bytes that no
copy brings, so the waits run out with nothing in flight (no GPU fault, no
hang: each wait ends after the limit).  Each case checks the three device
entry points -- host-memory predict, device predict on the caller's stream
(then check_device), and the no-alloc entry point -- and that the next call
on the same handle, with the hook off, is bit-exact against the oracle.
"""

from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest

from conftest import O, assert_bitwise
from macboost_b200 import synth

pytestmark = pytest.mark.gpu

LIMIT_US = "3000"  # 3 ms per wait while the hook is on


def _noalloc(core, h, x, rows, cols, ld, kind, out):
    fn = core._lib.macboost_predict_device_noalloc
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p)]
    err = ctypes.c_char_p()
    if fn(h.ptr, 0, x, rows, cols, ld, 0, kind, out, None, ctypes.byref(err)) != 0:
        raise core.MacBoostError(core._take_error(err))


@pytest.mark.parametrize("cfg,trees,plan", [
    ("cfg2", None, "codes=0,bufs=1,grid=4"),     # per-warp pipeline, one buffer
    ("cfg2", None, "codes=0,bufs=2,grid=4"),     # per-warp pipeline, next chunk in flight
    ("cfg4", 300, "codes=0,bufs=2,grid=4"),      # CTA-wide tiles, streamed forest blocks
    ("cfg5", 60, "grid=4"),                      # explicit layout
    ("cfg2", None, "codes=1,grid=4"),            # binned codes
])
def test_wait_runs_out_and_recovers(gpu, oracle_built, monkeypatch, cfg, trees, plan):
    core = gpu
    from test_gpu_parity import _cudart
    monkeypatch.setenv("MACBOOST_PLAN", plan)
    text = synth.model_to_json(synth.make_model(cfg, trees=trees))
    h = core.load_json(text)
    monkeypatch.delenv("MACBOOST_PLAN")
    om = O.model_from_dict(json.loads(text))
    rows = 9_000
    X = synth.make_data(cfg, rows=rows, row_start=11, layout="feature")
    want = O.predict_raw(om, X, layout="feature")
    F = X.shape[0]
    cu = _cudart()
    dx = cu.alloc(X.nbytes)
    dout = cu.alloc(rows * want.shape[1] * 4)
    try:
        cu.h2d(dx, np.ascontiguousarray(X))
        assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW, layout="feature"), want,
                       "before")
        monkeypatch.setenv("MACBOOST_WAIT_LIMIT_US", LIMIT_US)
        monkeypatch.setenv("MACBOOST_TEST_STALL_TILES", "1")
        with pytest.raises(core.MacBoostError, match="gave up waiting"):
            core.predict_ex(h, X, kind=core.KIND_RAW, layout="feature")
        core.predict_device(h, 0, dx, rows, F, rows, dout, kind=core.KIND_RAW)
        with pytest.raises(core.MacBoostError, match="gave up waiting"):
            core.check_device(h, 0)
        with pytest.raises(core.MacBoostError, match="gave up waiting"):
            _noalloc(core, h, dx, rows, F, rows, core.KIND_RAW, dout)
        monkeypatch.delenv("MACBOOST_TEST_STALL_TILES")
        monkeypatch.delenv("MACBOOST_WAIT_LIMIT_US")
        # the context and the handle stay usable
        assert_bitwise(core.predict_ex(h, X, kind=core.KIND_RAW, layout="feature"), want,
                       "after")
        core.predict_device(h, 0, dx, rows, F, rows, dout, kind=core.KIND_RAW)
        core.check_device(h, 0)
        assert_bitwise(cu.d2h(dout, rows * want.shape[1], np.float32).reshape(want.shape),
                       want, "device entry point after")
        _noalloc(core, h, dx, rows, F, rows, core.KIND_RAW, dout)
        assert_bitwise(cu.d2h(dout, rows * want.shape[1], np.float32).reshape(want.shape),
                       want, "no-alloc entry point after")
    finally:
        cu.free(dx)
        cu.free(dout)
