"""Static flat-slab slot schedule (host side, integer, install time).

For one layer this decides, once, where every retained (source scale, head) K/V segment lives in
the layer's flat slab ``[B, capacity, D]``, and derives everything the per-scale hot path needs.
It reproduces ``_segmented_flat_build_static_slot_schedule`` (enable_real_pruning_fast.py:260-558)
bit for bit:

1. Live interval of each (source ``s``, head ``h``): ``[s+1, end)`` where ``end`` is the first
   target whose removed set holds ``h`` for ``s`` (or ``num_scales``); empty intervals are
   dropped (:276-310).
2. Intervals are placed in ``(start, end, -length, source, head)`` order (:313-322). Before each
   placement the intervals that ended by its start are freed and the free list is coalesced
   (:324-337, merge rule :1033-1047); the segment takes the best-fitting free block - least
   leftover, then lowest offset - from its front, else the high-water mark grows (:338-370).
   Steps 1-2 and the capacity bound run in native code (``heatkv_slot_schedule``,
   csrc/slot_schedule.cpp).
3. Per target ``t``: ``[H, S]`` starts/ends and ``[H]`` counts of the live segments, each head's
   segments in source-scale order (:383-412).
4. Copy descriptors, sorted by destination slot (:414-482): the activation pack of target ``t``
   reads the dense ``[B, H, T_t, D]`` cache of the ``T_t`` tokens before ``t`` (:484-510); the
   append after scale ``s`` reads that scale's ``[B, H, n_s, D]`` K/V (:512-545). Source rows use
   the flat ``head * seq_len + token`` index (:469).

The capacity bound of :206-234 (max over targets of retained tokens) is reported beside the
allocated high-water mark; like the reference default (``..._ALLOW_OVERALLOC=1``) the high-water
mark is used even when it exceeds the bound.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _native


def _placement(controller, *, layer_idx: int, num_heads: int, arrays: bool = False):
    """Placed segments (placement order), high-water mark and capacity bound of a layer, from
    libheatkv's ``heatkv_slot_schedule`` (the reference's placement and capacity bound, :206-370,
    in native code); with ``arrays`` also the raw ``(scale_start, scale_end, offset, end_target)``
    arrays."""
    mask = np.ascontiguousarray(controller.removed_mask_for_layer(layer_idx), dtype=np.uint8)
    ranges = controller.scale_ranges
    num_scales = len(controller.scale_schedule)
    if mask.shape != (num_scales, num_scales, num_heads):
        raise ValueError("removed mask must be [scales, scales, heads]")
    lo = np.array([int(ranges[s][0]) if s in ranges else 0 for s in range(num_scales)], np.int64)
    hi = np.array([int(ranges[s][1]) if s in ranges else 0 for s in range(num_scales)], np.int64)
    offset = np.empty(num_scales * num_heads, dtype=np.int64)
    end_t = np.empty(num_scales * num_heads, dtype=np.int32)
    cap, bound = ctypes.c_int64(0), ctypes.c_int64(0)
    _native.check(_native.load().heatkv_slot_schedule(
        mask.ctypes.data, num_scales, num_heads, lo.ctypes.data, hi.ctypes.data,
        offset.ctypes.data, end_t.ctypes.data, ctypes.byref(cap), ctypes.byref(bound)),
        "heatkv_slot_schedule")
    segs = []
    for s in range(num_scales):
        for h in range(num_heads):
            off = int(offset[s * num_heads + h])
            if off < 0:
                continue
            segs.append({"source_scale": s, "head": h, "start_target": s + 1,
                         "end_target": int(end_t[s * num_heads + h]), "length": int(hi[s] - lo[s]),
                         "scale_start": int(lo[s]), "scale_end": int(hi[s]), "offset": off})
    segs.sort(key=lambda it: (it["start_target"], it["end_target"], -it["length"],
                              it["source_scale"], it["head"]))
    if arrays:
        return segs, int(cap.value), int(bound.value), (lo, hi, offset, end_t)
    return segs, int(cap.value), int(bound.value)


def capacity_bound_for_layer(controller, *, layer_idx: int, num_heads: int) -> int:
    """``_segmented_flat_cache_capacity_for_layer``: max over targets of sum over earlier
    sources of (heads kept) x tokens."""
    return _placement(controller, layer_idx=layer_idx, num_heads=num_heads)[2]


def _copy_runs(items, sequence_len: int):
    """Group copy items (sorted by destination) into destination-contiguous runs."""
    runs = []
    for item in sorted(items, key=lambda it: it["dst_offset"]):
        if item["length"] <= 0:
            continue
        src = item["head"] * sequence_len + item["src_start"]
        if runs and runs[-1]["dst_end"] == item["dst_offset"]:
            run = runs[-1]
        else:
            run = {"dst_start": item["dst_offset"], "dst_end": item["dst_offset"],
                   "sequence_len": int(sequence_len), "copy_items": []}
            runs.append(run)
        run["copy_items"].append(
            {"dst_start": item["dst_offset"], "src_start": src, "length": item["length"]})
        run["dst_end"] += item["length"]
    for run in runs:
        ci = run["copy_items"]
        contiguous = all(ci[i + 1]["src_start"] == ci[i]["src_start"] + ci[i]["length"]
                         for i in range(len(ci) - 1))
        run["contiguous_src_start"] = ci[0]["src_start"] if contiguous else None
        run["contiguous_src_end"] = (ci[0]["src_start"] + run["dst_end"] - run["dst_start"]
                                     if contiguous else None)
    return runs


def copy_descriptors(runs):
    """Flatten runs into the int64 ``(dst_starts, src_starts, lengths)`` arrays the pack kernel
    takes, plus the longest item and total slots
    (``_segmented_flat_static_copy_metadata_for_runs``, enable_real_pruning_fast.py:610-671)."""
    items = [it for run in runs for it in run["copy_items"]]
    if not items:
        return None
    dst = np.array([it["dst_start"] for it in items], dtype=np.int64)
    src = np.array([it["src_start"] for it in items], dtype=np.int64)
    lengths = np.array([it["length"] for it in items], dtype=np.int64)
    return {"dst_starts": dst, "src_starts": src, "lengths": lengths,
            "max_length": int(lengths.max()), "slots": int(lengths.sum()),
            "item_count": len(items)}


def prep_append_split(schedule, scale: int, num_heads: int):
    """Split the append after ``scale`` (``append_runs_by_key[(scale, scale + 1)]``) into the heads
    whose rows the q/k/v preparation of that scale may write straight into the slab
    (``heatkv_qkv_prepare_append``) and the copy runs left for the pack after the attention.

    The reference appends after the attention of ``scale`` (enable_real_pruning_fast.py:2218-2225),
    because a new segment may take slots freed by segments that the attention of ``scale`` still
    reads (their live interval ends at ``scale + 1``). A head's rows can be written before that
    attention only when its segment shares no slot with any segment live at ``scale``; the slab
    then holds the same bytes after the attention as with the reference's order.

    Returns None when nothing is appended, else ``{"offsets": int64 [num_heads] (-1 = not written
    by the preparation), "early_slots": int, "rest_runs": runs for ``copy_descriptors``}``."""
    runs = schedule["append_runs_by_key"].get((scale, scale + 1))
    if not runs:
        return None
    reads = sorted((seg["offset"], seg["offset"] + seg["length"])
                   for seg in schedule["segments_by_target"].get(scale, []) if seg["length"] > 0)
    starts = np.array([r[0] for r in reads], dtype=np.int64)
    ends = np.array([r[1] for r in reads], dtype=np.int64)
    offsets = np.full(int(num_heads), -1, dtype=np.int64)
    early, rest = 0, []
    for run in runs:
        seq_len = run["sequence_len"]
        for it in run["copy_items"]:
            lo, hi = it["dst_start"], it["dst_start"] + it["length"]
            clash = bool(np.any((starts < hi) & (ends > lo)))
            whole = it["src_start"] % seq_len == 0 and it["length"] == seq_len
            if clash or not whole:
                rest.append({"dst_offset": lo, "head": it["src_start"] // seq_len,
                             "src_start": it["src_start"] % seq_len, "length": it["length"]})
            else:
                offsets[it["src_start"] // seq_len] = lo
                early += it["length"]
    seq_len = runs[0]["sequence_len"]
    return {"offsets": offsets, "early_slots": int(early), "rest_runs": _copy_runs(rest, seq_len)}


def build_static_slot_schedule(controller, *, layer_idx: int, num_heads: int,
                               allow_overalloc: bool = True):
    """Return the reference's schedule dict (keys ``enabled``, ``capacity``, ``capacity_bound``,
    ``allocated_capacity``, ``overalloc_slots``, ``segments``, ``segments_by_key``,
    ``segments_by_target``, ``metadata_cpu_by_target``, ``old_pack_runs_by_target``,
    ``old_pack_cache_lens_by_target``, ``append_runs_by_key``); metadata values are numpy int32.
    The placement (``heatkv_slot_schedule``), the per-target segment tables and the copy items
    (``heatkv_slot_tables``) are computed in native code; this function only shapes them into the
    reference's dict."""
    num_heads = int(num_heads)
    ranges = controller.scale_ranges
    num_scales = len(controller.scale_schedule)
    assigned, high_water, bound, placed = _placement(controller, layer_idx=layer_idx,
                                                     num_heads=num_heads, arrays=True)

    if high_water > bound and not allow_overalloc:
        return {"enabled": False, "capacity": bound, "capacity_bound": bound,
                "allocated_capacity": high_water}

    S, H = num_scales, num_heads
    lo, hi, offset, end_t = placed
    m_st = np.empty((S, H, S), dtype=np.int32)
    m_en = np.empty((S, H, S), dtype=np.int32)
    m_ct = np.empty((S, H), dtype=np.int32)
    pack_items = np.empty((S * S * H, 3), dtype=np.int64)
    pack_index = np.empty(S + 1, dtype=np.int64)
    app_items = np.empty((S * H, 3), dtype=np.int64)
    app_index = np.empty(S + 1, dtype=np.int64)
    _native.check(_native.load().heatkv_slot_tables(
        S, H, lo.ctypes.data, hi.ctypes.data, offset.ctypes.data, end_t.ctypes.data,
        m_st.ctypes.data, m_en.ctypes.data, m_ct.ctypes.data, pack_items.ctypes.data,
        pack_index.ctypes.data, app_items.ctypes.data, app_index.ctypes.data),
        "heatkv_slot_tables")

    by_key = {(seg["source_scale"], seg["head"]): seg for seg in assigned}
    by_target, metadata = {}, {}
    for t in range(1, num_scales):
        by_target[t] = [seg for seg in assigned if seg["start_target"] <= t < seg["end_target"]]
        width = int(m_ct[t].max()) if H else 0
        metadata[t] = (np.ascontiguousarray(m_st[t, :, :width]),
                       np.ascontiguousarray(m_en[t, :, :width]), m_ct[t].copy())

    old_runs, old_lens = {}, {}
    for t in by_target:
        if t not in ranges:
            continue
        old_len = int(ranges[t][0])
        old_lens[t] = old_len
        old_runs[t] = _runs_from_items(pack_items[pack_index[t]:pack_index[t + 1]], old_len)

    append_runs = {}
    for s_, (a, b) in ranges.items():
        if s_ + 1 >= num_scales or int(b) - int(a) <= 0:
            continue
        append_runs[(s_, s_ + 1)] = _runs_from_items(app_items[app_index[s_]:app_index[s_ + 1]],
                                                     int(b) - int(a))

    return {
        "enabled": True, "capacity": int(high_water), "capacity_bound": int(bound),
        "allocated_capacity": int(high_water),
        "overalloc_slots": max(0, int(high_water) - int(bound)),
        "segments": assigned, "segments_by_key": by_key, "segments_by_target": by_target,
        "metadata_cpu_by_target": metadata, "metadata_device_cache": {},
        "old_pack_runs_by_target": old_runs, "old_pack_cache_lens_by_target": old_lens,
        "append_runs_by_key": append_runs,
    }


def _runs_from_items(items: np.ndarray, sequence_len: int):
    """Destination-contiguous runs (the reference's run dicts, :414-482) of copy items
    ``(dst, src, length)`` already sorted by destination."""
    runs = []
    for dst, src, length in items.tolist():
        if length <= 0:
            continue
        if runs and runs[-1]["dst_end"] == dst:
            run = runs[-1]
        else:
            run = {"dst_start": dst, "dst_end": dst, "sequence_len": int(sequence_len),
                   "copy_items": []}
            runs.append(run)
        run["copy_items"].append({"dst_start": dst, "src_start": src, "length": length})
        run["dst_end"] += length
    for run in runs:
        ci = run["copy_items"]
        contiguous = all(ci[i + 1]["src_start"] == ci[i]["src_start"] + ci[i]["length"]
                         for i in range(len(ci) - 1))
        run["contiguous_src_start"] = ci[0]["src_start"] if contiguous else None
        run["contiguous_src_end"] = (ci[0]["src_start"] + run["dst_end"] - run["dst_start"]
                                     if contiguous else None)
    return runs
