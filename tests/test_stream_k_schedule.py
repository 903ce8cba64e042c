"""The stream-K schedule of the history kernel, checked on the CPU through the
library's host view of it (``pcp_stream_k_plan`` / ``pcp_stream_k_segments``,
the same code the kernel runs): every (unit, key tile) step is covered
exactly once, each unit's segments are contiguous with slots 0..nseg-1, and
the planner's slot count bounds every unit -- also when the kernel runs
fewer key tiles than the launch was planned for (device-side lengths)."""

from __future__ import annotations

import ctypes
import random

import pytest

from aws_training_study_b200 import _capi


def _plan(units, key_tiles, sms=148, slot_cap=32):
    pairs, slots = ctypes.c_int32(), ctypes.c_int32()
    _capi.check(_capi.lib().pcp_stream_k_plan(units, key_tiles, sms, slot_cap, ctypes.byref(pairs),
                                              ctypes.byref(slots)))
    return pairs.value, slots.value


def _segments(units, key_tiles, grid_pairs, pair):
    cap = 4096
    buf = (ctypes.c_int32 * (6 * cap))()
    count = ctypes.c_int32()
    _capi.check(_capi.lib().pcp_stream_k_segments(units, key_tiles, grid_pairs, pair, buf, cap, ctypes.byref(count)))
    return [tuple(buf[6 * i : 6 * i + 6]) for i in range(count.value)]


def _check(units, planned_tiles, run_tiles, sms=148, slot_cap=32):
    pairs, slots = _plan(units, planned_tiles, sms, slot_cap)
    assert 1 <= pairs <= max(1, sms // 2) and 1 <= slots <= slot_cap
    per_unit = {}
    for g in range(pairs):
        for unit, kt0, kt1, slot, nseg, last in _segments(units, run_tiles, pairs, g):
            assert 0 <= kt0 < kt1 <= run_tiles and 0 <= slot < nseg <= slots
            per_unit.setdefault(unit, []).append((kt0, kt1, slot, nseg, last))
    if run_tiles == 0:
        assert not per_unit
        return
    assert sorted(per_unit) == list(range(units))
    for segs in per_unit.values():
        segs.sort()
        assert segs[0][0] == 0 and segs[-1][1] == run_tiles
        assert all(a[1] == b[0] for a, b in zip(segs, segs[1:]))
        assert [s[2] for s in segs] == list(range(len(segs)))
        assert all(s[3] == len(segs) for s in segs)
        assert [bool(s[4]) for s in segs] == [False] * (len(segs) - 1) + [True]


@pytest.mark.parametrize("units,tiles", [(512, 1024), (64, 896), (64, 128), (256, 16), (16, 64), (1, 1), (1, 100),
                                         (3, 7), (2, 1)])
def test_baseline_shapes(units, tiles):
    _check(units, tiles, tiles)


def test_device_lengths_shorter_than_the_plan():
    for run in (0, 1, 10, 333):
        _check(64, 896, run)


def test_random_shapes():
    rng = random.Random(0)
    for _ in range(400):
        units = rng.randint(1, 300)
        planned = rng.randint(1, 600)
        _check(units, planned, rng.randint(0, planned), sms=rng.choice([148, 132, 10, 2]),
               slot_cap=rng.randint(1, 32))


def test_bad_arguments_rejected():
    with pytest.raises(_capi.PcpError):
        _plan(0, 10)
    count = ctypes.c_int32()
    with pytest.raises(_capi.PcpError):
        _capi.check(_capi.lib().pcp_stream_k_segments(4, 4, 2, 2, None, 0, ctypes.byref(count)))
