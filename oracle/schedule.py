"""CPU restatement of the flat-slab slot placement (test infrastructure only).

Follows _segmented_flat_build_static_slot_schedule (enable_real_pruning_fast.py:260-370) and
_segmented_flat_cache_capacity_for_layer (:206-234) of the reference: the oracle the native
placement (libheatkv ``heatkv_slot_schedule``) is checked against, beside the schedules recorded
from the reference itself (tests/golden/schedule_*.npz). Only tests import it.
"""

from __future__ import annotations

import numpy as np


def capacity_bound(mask: np.ndarray, tokens: np.ndarray) -> int:
    """max over targets t of sum over sources s < t of (heads kept at t) x tokens of s (:206-234)."""
    num_scales, _, num_heads = mask.shape
    best = 0
    for t in range(1, num_scales):
        kept = num_heads - mask[t, :t, :].sum(axis=1).astype(np.int64)
        best = max(best, int((kept * np.maximum(tokens[:t], 0)).sum()))
    return best


def merge_free_blocks(blocks):
    """Sort by offset and coalesce overlapping or touching blocks; zero-length blocks vanish
    (:1033-1047)."""
    out = []
    for off, length in sorted((int(o), int(n)) for o, n in blocks if int(n) > 0):
        if out and off <= out[-1][0] + out[-1][1]:
            last_off, last_len = out[-1]
            out[-1] = (last_off, max(last_off + last_len, off + length) - last_off)
        else:
            out.append((off, length))
    return out


def place(mask: np.ndarray, starts: np.ndarray, ends: np.ndarray):
    """Segments ``(source, head, start_target, end_target, length, offset)`` in placement order,
    and the high-water mark, for a ``[target, source, head]`` removed mask and each scale's
    token range (:276-370)."""
    num_scales, _, num_heads = mask.shape
    intervals = []
    for s in range(num_scales):
        start_t = s + 1
        length = int(ends[s]) - int(starts[s])
        if start_t >= num_scales or length <= 0:
            continue
        for h in range(num_heads):
            hits = np.flatnonzero(mask[start_t:, s, h])
            end_t = start_t + int(hits[0]) if hits.size else num_scales
            if end_t > start_t:
                intervals.append((start_t, end_t, -length, s, h))
    free, active, placed, high_water = [], [], [], 0
    for start_t, end_t, neg_len, s, h in sorted(intervals):
        need = -neg_len
        still = []
        for a in active:
            if a[3] <= start_t:
                free.append((a[5], a[4]))
            else:
                still.append(a)
        active = still
        free = merge_free_blocks(free)
        best = None
        for i, (off, length) in enumerate(free):
            if length >= need and (best is None or (length - need, off) < (best[0], best[2])):
                best = (length - need, i, off, length)
        if best is not None:
            _, i, off, length = best
            if length == need:
                del free[i]
            else:
                free[i] = (off + need, length - need)
            offset = off
        else:
            offset = high_water
            high_water += need
        seg = (s, h, start_t, end_t, need, offset)
        placed.append(seg)
        active.append(seg)
    return placed, high_water
