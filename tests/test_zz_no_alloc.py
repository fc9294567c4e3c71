"""macboost_predict_device_noalloc: the entry point that allocates no device
memory, for hosts whose GPU memory belongs to their own pool or whose other
streams must not be stalled by a library's cudaMalloc / cudaFree.

Its results are checked against the allocating device entry point
(macboost_predict_device) on the same model and inputs, twice in a row (the
shared scratch keeps the previous call's contents, so a second call must not
depend on them), for feature-major and row-major input, with the tolerance the
rest of the suite uses (margins bit-exact, transformed outputs within 2 ulp).
Collected last so that a failure here never hides the other tests' results.
"""

import ctypes
import glob
import os

import numpy as np
import pytest

from conftest import assert_bitwise, assert_ulp, golden_text
from macboost_b200 import synth

pytestmark = pytest.mark.gpu


class _DeviceMemory:
    """Device buffers for the test (the test may allocate; the call under test may not)."""

    def __init__(self):
        cands = sorted(glob.glob("/usr/local/cuda/lib64/libcudart.so*")) + ["libcudart.so.12"]
        for c in cands:
            try:
                self.lib = ctypes.CDLL(c)
                break
            except OSError:
                continue
        self.lib.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
        self.lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_int]
        self.lib.cudaFree.argtypes = [ctypes.c_void_p]
        self.lib.cudaMemGetInfo.argtypes = [ctypes.POINTER(ctypes.c_size_t),
                                            ctypes.POINTER(ctypes.c_size_t)]
        self.ptrs = []

    def free_bytes(self):
        free, total = ctypes.c_size_t(), ctypes.c_size_t()
        assert self.lib.cudaMemGetInfo(ctypes.byref(free), ctypes.byref(total)) == 0
        return free.value

    def upload(self, a):
        p = ctypes.c_void_p()
        assert self.lib.cudaMalloc(ctypes.byref(p), max(a.nbytes, 4)) == 0
        assert self.lib.cudaMemcpy(p.value, a.ctypes.data, a.nbytes, 1) == 0
        self.ptrs.append(p.value)
        return p.value

    def empty(self, nbytes):
        return self.upload(np.zeros(max(nbytes // 4, 1), np.float32))

    def download(self, p, shape, dtype):
        out = np.empty(shape, dtype)
        assert self.lib.cudaMemcpy(out.ctypes.data, p, out.nbytes, 2) == 0
        return out

    def free(self):
        for p in self.ptrs:
            self.lib.cudaFree(p)
        self.ptrs = []


def _noalloc(core):
    fn = core._lib.macboost_predict_device_noalloc
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p)]
    return fn


def _call(core, h, x, rows, cols, ld, layout, kind, out):
    err = ctypes.c_char_p()
    rc = _noalloc(core)(h.ptr, 0, x, rows, cols, ld, layout, kind, out, None, ctypes.byref(err))
    if rc != 0:
        raise core.MacBoostError(core._take_error(err))


@pytest.mark.parametrize("kind", [1, 2])  # raw margins, predict_proba
def test_noalloc_matches_allocating_entry_point(gpu, kind):
    core = gpu
    h = core.load_json(golden_text("cfg2_small"))
    core.prepare(h, [0])                  # set-up: the one step that allocates
    rows, F = 3001, 28
    X = synth.make_data("cfg2", rows=rows, row_start=4242, layout="feature")
    ld = 3004
    Xf = np.zeros((F, ld), np.float32)
    Xf[:, :rows] = X
    ncol = core.output_cols(h, kind)
    mem = _DeviceMemory()
    try:
        dx = mem.upload(Xf)
        dxr = mem.upload(np.ascontiguousarray(X.T))   # row-major copy
        dref = mem.empty(rows * ncol * 4)
        dout = mem.empty(rows * ncol * 4)
        core.predict_device(h, 0, dx, rows, F, ld, dref, kind=kind)
        core.check_device(h, 0)
        ref = mem.download(dref, (rows, ncol), np.float32)
        # one call per layout first: the kernels' modules load (and the driver
        # reserves their memory) on first use; after that the free device
        # memory must not move while the entry point runs
        _call(core, h, dx, rows, F, ld, 0, kind, dout)
        _call(core, h, dxr, rows, F, 0, 1, kind, dout)
        free0 = mem.free_bytes()
        for layout, x, stride in [(0, dx, ld), (0, dx, ld), (1, dxr, 0), (1, dxr, 0)]:
            _call(core, h, x, rows, F, stride, layout, kind, dout)
            got = mem.download(dout, (rows, ncol), np.float32)
            if kind == 1:
                assert_bitwise(got, ref, f"no-alloc layout={layout}")
            else:
                assert_ulp(got, ref, 2, f"no-alloc layout={layout}")
        assert mem.free_bytes() == free0, "the no-alloc entry point changed free device memory"
    finally:
        mem.free()


def test_noalloc_limits_and_preconditions(gpu):
    core = gpu
    h = core.load_json(golden_text("cfg2_small"))
    mem = _DeviceMemory()
    try:
        dx = mem.empty(64 * 28 * 4)
        dout = mem.empty(64 * 4)
        with pytest.raises(core.MacBoostError, match="not resident"):
            _call(core, h, dx, 64, 28, 64, 0, 1, dout)
        core.prepare(h, [0])
        # 200,000 rows x 28 features row-major needs 22.4 MB of copy > 16 MiB
        with pytest.raises(core.MacBoostError, match="16 MiB"):
            _call(core, h, dx, 200_000, 28, 0, 1, 1, dout)
        with pytest.raises(core.MacBoostError, match="model expects 28"):
            _call(core, h, dx, 64, 27, 64, 0, 1, dout)
    finally:
        mem.free()
