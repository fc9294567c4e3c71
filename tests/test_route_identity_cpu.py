"""The routing identity behind the complete walk's no-plane records, on the CPU.

Without NaN planes a node sends its row right when `!(fmax(v, c) <= t)`, c being
either computed from the record's default-left bit (a funnel shift giving -Inf
or NaN) or, in forests with no categorical splits and no default-left threshold
below -2^127, the record's slot word itself: 0xFFC00000 | offset (a quiet NaN) for
default-right nodes and 0xFF000000 | offset (a float at or below -2^127) for
default-left ones, offset a multiple of 128 below 2^18.  Both must equal the
reference's decision (`Booster.swift:2035-2117`, `_pyinfer.py:74-84`): a NaN
goes to the node's default side, any other value goes left iff v <= t.  numpy's
fmax has CUDA's fmaxf semantics (the non-NaN operand when one is NaN).
"""

from __future__ import annotations

import numpy as np

NEG_2_127 = np.float32(-2.0 ** 127)
F32_MAX = np.finfo(np.float32).max
TINY = np.float32(1e-45)


def _bits(u):
    return np.asarray(u, dtype=np.uint32).view(np.float32)


def _values(rng):
    special = np.float32([np.nan, -np.nan, np.inf, -np.inf, 0.0, -0.0, TINY, -TINY, F32_MAX,
                          -F32_MAX, NEG_2_127, np.nextafter(NEG_2_127, np.float32(0)),
                          np.nextafter(NEG_2_127, -np.inf), -1.7e38, -1.71e38, -3e38, 1.0, -1.0])
    rand_bits = rng.integers(0, 2 ** 32, 20_000, dtype=np.uint64).astype(np.uint32)
    return np.concatenate([special, rng.standard_normal(2000).astype(np.float32),
                           _bits(rand_bits)])


def _reference(v, t, default_left):
    return np.where(np.isnan(v), not default_left, ~(v <= t))      # True = right


def test_payload_words_route_like_the_reference():
    rng = np.random.default_rng(0)
    v = _values(rng)
    thresholds = np.concatenate([
        np.float32([NEG_2_127, np.nextafter(NEG_2_127, np.float32(0)), -1.7e38, -1.0, -0.0, 0.0,
                    TINY, 1.0, 3e38, F32_MAX, np.inf]),
        rng.standard_normal(40).astype(np.float32)])
    # keep the thresholds the planner admits for default-left records (>= -2^127)
    assert np.all(thresholds >= NEG_2_127)
    offsets = np.uint32([0, 128, 4096, 0x3FF80])
    with np.errstate(invalid="ignore"):
        for off in offsets:
            c_left = _bits(np.uint32(0xFF000000) | off)
            c_right = _bits(np.uint32(0xFFC00000) | off)
            assert np.isfinite(c_left) and c_left <= NEG_2_127
            assert np.isnan(c_right)
            assert (np.uint32(0xFF000000) | off) & np.uint32(0x3FF80) == off
            for t in thresholds:
                for dl, c in ((True, c_left), (False, c_right)):
                    got = ~(np.fmax(v, c) <= t)
                    want = _reference(v, t, dl)
                    bad = np.flatnonzero(got != want)
                    assert bad.size == 0, (hex(int(off)), float(t), dl, v[bad[:4]])


def test_flag_shift_words_route_like_the_reference():
    """The route kept for the other forests: c = 0x7FC00000 << (word & 31), the word's
    low five bits being the default-left bit and zeros (offsets are multiples of 128)."""
    rng = np.random.default_rng(1)
    v = _values(rng)
    thresholds = np.float32([-np.inf, -F32_MAX, -3e38, -1.0, 0.0, 1.0, F32_MAX, np.inf])
    with np.errstate(invalid="ignore"):
        for dl in (True, False):
            word = np.uint32(4096 | (1 if dl else 0))
            c = _bits(np.uint32((0x7FC00000 << int(word & 31)) & 0xFFFFFFFF))
            for t in thresholds:
                got = ~(np.fmax(v, c) <= t)
                assert np.array_equal(got, _reference(v, t, dl)), (float(t), dl)


def test_payload_bound_is_needed():
    """Below -2^127 a default-left threshold would sit under c: a NaN (and any value
    between the threshold and c) would go right.  That is why the planner keeps the
    shift route for such forests."""
    c_left = _bits(np.uint32(0xFF000000))
    t = np.float32(-3e38)
    v = np.float32([np.nan, -np.inf, -3.1e38])
    with np.errstate(invalid="ignore"):
        got = ~(np.fmax(v, c_left) <= t)
    assert np.all(got) and not np.any(_reference(v, t, True))
