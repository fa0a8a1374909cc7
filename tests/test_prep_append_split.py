"""``scheduler.prep_append_split`` (CPU, integer): which heads of the append after a scale
(enable_real_pruning_fast.py:2218-2225) the q/k/v preparation may write into the slab before that
scale's attention.

Properties on the 2B (5/10/50 %) and 8B (10 %) schedules of every layer and scale:
* the early heads and the remaining copy items partition the reference's append items exactly;
* no early head's segment shares a slot with a segment the attention of that scale reads, and every
  remaining item does share one (the split is maximal);
* the remaining runs are ``_copy_runs`` of the remaining items (sorted by destination).
"""

import numpy as np
import pytest

from heatkv_b200.scheduler import build_static_slot_schedule, prep_append_split

from test_host_golden import _controller


def _overlaps(lo, hi, reads):
    return any(a < hi and b > lo for a, b in reads)


@pytest.mark.parametrize("name,layers", [("2b_b05", range(0, 32, 5)), ("2b_b10", range(32)),
                                         ("2b_b50", range(0, 32, 7)), ("8b_b10", range(0, 40, 3))])
def test_split_partitions_the_append_and_avoids_live_slots(name, layers):
    _, ctrl = _controller(name)
    heads = ctrl.num_heads
    early_total = rest_total = 0
    for layer in layers:
        sched = build_static_slot_schedule(ctrl, layer_idx=layer, num_heads=heads)
        for (s, nxt), runs in sched["append_runs_by_key"].items():
            split = prep_append_split(sched, s, heads)
            items = [it for run in runs for it in run["copy_items"]]
            if not items:
                assert split is None
                continue
            reads = [(g["offset"], g["offset"] + g["length"])
                     for g in sched["segments_by_target"].get(s, [])]
            seq_len = runs[0]["sequence_len"]
            rest = [it for run in split["rest_runs"] for it in run["copy_items"]]
            early = {h: int(o) for h, o in enumerate(split["offsets"]) if o >= 0}
            # partition: every reference item is either an early head or a remaining item
            got = sorted([(o, h * seq_len, seq_len) for h, o in early.items()]
                         + [(it["dst_start"], it["src_start"], it["length"]) for it in rest])
            want = sorted((it["dst_start"], it["src_start"], it["length"]) for it in items)
            assert got == want, (layer, s)
            for h, o in early.items():
                assert not _overlaps(o, o + seq_len, reads), (layer, s, h)
            for it in rest:
                assert _overlaps(it["dst_start"], it["dst_start"] + it["length"], reads)
            dst = [it["dst_start"] for it in rest]
            assert dst == sorted(dst)
            assert split["early_slots"] == seq_len * len(early)
            early_total += split["early_slots"]
            rest_total += sum(it["length"] for it in rest)
    assert early_total > 0 and rest_total > 0


def test_split_of_a_scale_without_append_is_none():
    _, ctrl = _controller("2b_b10")
    sched = build_static_slot_schedule(ctrl, layer_idx=0, num_heads=ctrl.num_heads)
    last = len(ctrl.scale_schedule) - 1
    assert prep_append_split(sched, last, ctrl.num_heads) is None


def test_2b_b10_share_of_early_slots():
    """At the benchmark configuration 60 % of the appended slots move into the preparation."""
    _, ctrl = _controller("2b_b10")
    early = total = 0
    for layer in range(32):
        sched = build_static_slot_schedule(ctrl, layer_idx=layer, num_heads=16)
        for t in range(1, 12):
            if not ctrl.any_removed(layer, t):
                continue
            split = prep_append_split(sched, t, 16)
            if split is None:
                continue
            early += split["early_slots"]
            total += split["early_slots"] + sum(
                it["length"] for run in split["rest_runs"] for it in run["copy_items"])
    assert (early, total) == (272384, 454400)
    assert np.isclose(early / total, 0.5994, atol=1e-4)
