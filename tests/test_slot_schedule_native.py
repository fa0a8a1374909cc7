"""The native slab placement (heatkv_slot_schedule, csrc/slot_schedule.cpp) against the oracle's
restatement of the reference's placement (oracle/schedule.py) on random removal masks and scale
lengths, bit for bit (CPU; no device needed). The recorded reference schedules are checked in
test_host_golden.py."""

import ctypes

import numpy as np
import pytest

from heatkv_b200 import _native
from oracle.schedule import capacity_bound, place


def _native_place(mask, starts, ends):
    S, _, H = mask.shape
    off = np.empty(S * H, np.int64)
    end = np.empty(S * H, np.int32)
    cap, bound = ctypes.c_int64(), ctypes.c_int64()
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    st = np.ascontiguousarray(starts, dtype=np.int64)
    en = np.ascontiguousarray(ends, dtype=np.int64)
    rc = _native.load().heatkv_slot_schedule(m.ctypes.data, S, H, st.ctypes.data, en.ctypes.data,
                                             off.ctypes.data, end.ctypes.data,
                                             ctypes.byref(cap), ctypes.byref(bound))
    assert rc == 0
    segs = [(s, h, s + 1, int(end[s * H + h]), int(ends[s] - starts[s]), int(off[s * H + h]))
            for s in range(S) for h in range(H) if off[s * H + h] >= 0]
    segs.sort(key=lambda x: (x[2], x[3], -x[4], x[0], x[1]))
    return segs, cap.value, bound.value


@pytest.mark.parametrize("seed", range(40))
def test_native_placement_equals_oracle(seed):
    rng = np.random.default_rng(seed)
    S = int(rng.integers(2, 14))
    H = int(rng.integers(1, 29))
    lengths = rng.integers(0, 700, size=S) * (rng.random(S) > 0.1)
    starts = np.concatenate([[0], np.cumsum(lengths)[:-1]])
    ends = starts + lengths
    # removals that persist once made (the budget policy's shape) plus random noise
    mask = np.zeros((S, S, H), np.uint8)
    for s in range(S):
        for h in range(H):
            first = int(rng.integers(s + 1, S + 2))
            mask[first:, s, h] = 1
    mask |= (rng.random((S, S, H)) < 0.05).astype(np.uint8)
    segs, cap, bound = _native_place(mask, starts, ends)
    ref_segs, ref_cap = place(mask, starts, ends)
    assert segs == ref_segs
    assert cap == ref_cap
    assert bound == capacity_bound(mask, ends - starts)


def test_invalid_arguments():
    lib = _native.load()
    z = ctypes.c_int64()
    assert lib.heatkv_slot_schedule(None, 3, 2, None, None, None, None, ctypes.byref(z),
                                    ctypes.byref(z)) == _native.HEATKV_ERR_INVALID_ARGUMENT
