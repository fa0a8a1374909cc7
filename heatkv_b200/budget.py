"""Budget -> keep-mask policy of HeatKV (host side, integer, install time).

Same entry points, argument meaning, results and error messages as the reference's
``tools/utils.py``:

* ``get_scale_schedule`` (utils.py:600) - the 13-scale 1:1 1024x1024 schedule.
* ``pruned_heads_for_budget`` (utils.py:235-305) - how many (layer, head) cache slots must be
  pruned before each scale so the incoming cache stays under ``budget`` of its unpruned peak.
* ``strict_pruning_schedule_for_budget_scale_specific`` (utils.py:308-522) - which
  ``(source_scale, head, layer)`` atoms are removed after each target scale (the first ``x``
  entries of each source scale's order) and which of them must be activated early, inside the
  target scale, so every layer checkpoint stays under the token budget. Activation priority:
  last layer first, then larger source scale, then order rank (utils.py:134-136, :206-219).
* ``strict_removed_heads_by_scale_specific_for_budget`` (utils.py:525-597) - the per-target
  removed-head view: atoms finalised after the previous target plus atoms activated early.

The per-target loop of the strict schedule runs in native code (``heatkv_strict_budget``,
csrc/install_plan.cpp). The reference re-sums the whole cache after every activation; there the
cache total is kept as an integer and decremented by ``tokens[source]`` per activated atom, and
the activation candidates are walked once per target in their fixed priority order. The
arithmetic (integers compared with the double threshold) is the same, so the removed sets are
identical.
"""

from __future__ import annotations

import math

from .synthetic import SCALE_SCHEDULE_1M


def get_scale_schedule():
    """``[(1, h, w), ...]`` of the 1:1 ``1M`` template: 13 scales, 10,521 tokens."""
    return [tuple(x) for x in SCALE_SCHEDULE_1M]


def orders(start_order=3, prompts=10, model_type=2):
    """The shipped S-CAS removal orders (``orders/{2,8}b.json``) as ``9 x [[head, layer], ...]``.

    Same signature as tools/utils.py:604 so its call sites (``orders(initial_scales,
    model_type=2)``) work unchanged. The shipped orders were ranked from source scale 3 over 10
    prompts; other values are rejected as in the reference. The reference first looks for a
    locally regenerated ``outputs/scas_2b/scas_orders.json``; pass such orders to the installer
    directly instead.
    """
    import json
    import os

    if start_order != 3 or prompts != 10:
        raise AssertionError("the shipped orders were computed with start_order=3 and prompts=10")

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "orders", f"{int(model_type)}b.json")
    with open(path) as fh:
        return json.load(fh)


def _validate_removal_order(removal_order, *, num_layers, num_heads):
    total_slots = int(num_layers) * int(num_heads)
    if len(removal_order) != total_slots:
        raise ValueError(f"expected {total_slots} removal-order entries, got {len(removal_order)}")
    seen = set()
    out = []
    for idx, pair in enumerate(removal_order):
        if not isinstance(pair, (tuple, list)) or len(pair) != 2:
            raise ValueError(f"removal_order[{idx}] must be a (head, layer) tuple")
        head, layer = int(pair[0]), int(pair[1])
        if not 0 <= head < num_heads:
            raise ValueError(f"head index out of range at position {idx}: {head}")
        if not 0 <= layer < num_layers:
            raise ValueError(f"layer index out of range at position {idx}: {layer}")
        if (head, layer) in seen:
            raise ValueError(f"duplicate (head, layer) entry at position {idx}: {(head, layer)}")
        seen.add((head, layer))
        out.append((head, layer))
    return out


def _validate_scale_specific_removal_orders(orders_seq, *, num_layers, num_heads,
                                            source_scale_start=4, source_scale_end=11):
    expected = int(source_scale_end) - int(source_scale_start) + 1
    if len(orders_seq) != expected:
        raise ValueError(
            "scale_specific_removal_orders must contain exactly "
            f"{expected} orders for source scales {source_scale_start}-{source_scale_end}"
        )
    return tuple(
        tuple(_validate_removal_order(o, num_layers=num_layers, num_heads=num_heads))
        for o in orders_seq
    )


def _check_budget(budget) -> float:
    budget = float(budget)
    if not 0.0 <= budget <= 1.0:
        raise ValueError(f"budget must be in [0, 1], got {budget}")
    return budget


def pruned_heads_for_budget(budget, *, retained_tokens=51, num_layers=32, num_heads=16,
                            skip_last_scale=True, scale_schedule=None):
    """Per scale index: number of (layer, head) slots pruned so the incoming cache (tokens of all
    earlier cached scales) is at most ``budget`` x its unpruned peak, when a pruned slot keeps
    ``retained_tokens`` positions."""
    budget = _check_budget(budget)
    schedule = get_scale_schedule() if scale_schedule is None else list(scale_schedule)
    if not schedule:
        return {}
    total_slots = int(num_layers) * int(num_heads)
    if total_slots <= 0:
        raise ValueError("num_layers * num_heads must be positive")
    if retained_tokens < 0:
        raise ValueError("retained_tokens must be non-negative")

    tokens = [h * w for _, h, w in schedule]
    incoming, running = [], 0
    for idx, n in enumerate(tokens):
        incoming.append(running)
        if idx < len(tokens) - 1 or not skip_last_scale:
            running += n
    peak = max(incoming, default=0)
    if peak <= 0:
        return {idx: 0 for idx in range(len(schedule))}
    min_budget = min(retained_tokens, peak) / peak
    if budget + 1e-12 < min_budget:
        raise ValueError(f"budget {budget} is below the minimum feasible ratio {min_budget:.12f}")

    allowed = budget * peak
    counts = {}
    for idx, inc in enumerate(incoming):
        kept_here = min(retained_tokens, inc)
        if inc <= allowed:
            need = 0
        elif inc == kept_here:
            raise ValueError(f"budget {budget} is infeasible at scale index {idx}")
        else:
            need = math.ceil(total_slots * (inc - allowed) / (inc - kept_here))
        counts[idx] = max(0, min(total_slots, need))
    return counts


def _atoms_by_source_and_layer(atoms, *, num_layers, source_scale_indices):
    grouped = {s: {l: [] for l in range(num_layers)} for s in source_scale_indices}
    for s, h, l in sorted(atoms):
        grouped[s][l].append(h)
    return {s: {l: tuple(hs) for l, hs in by_layer.items()} for s, by_layer in grouped.items()}


def strict_pruning_schedule_for_budget_scale_specific(
    budget, scale_specific_removal_orders, *, num_layers=32, num_heads=16, source_scale_start=4,
    source_scale_end=11, protected_prefix_scales=4, skip_last_scale=True, scale_schedule=None,
):
    """Final removed atoms per target and the early activations inside each target (see module
    docstring). Returns the reference's dict: ``final_removed_counts``, ``final_removed_by_scale``,
    ``early_activation_by_scale``."""
    budget = _check_budget(budget)
    num_layers, num_heads = int(num_layers), int(num_heads)
    if num_layers <= 0 or num_heads <= 0:
        raise ValueError("num_layers * num_heads must be positive")
    seq = _validate_scale_specific_removal_orders(
        scale_specific_removal_orders, num_layers=num_layers, num_heads=num_heads,
        source_scale_start=source_scale_start, source_scale_end=source_scale_end)
    s0, s1 = int(source_scale_start), int(source_scale_end)
    order_of = {s0 + i: o for i, o in enumerate(seq)}
    rank_of = {s: {pair: r for r, pair in enumerate(o)} for s, o in order_of.items()}

    schedule = get_scale_schedule() if scale_schedule is None else list(scale_schedule)
    if not schedule:
        return {"final_removed_counts": {}, "final_removed_by_scale": {},
                "early_activation_by_scale": {}}
    tokens = [h * w for _, h, w in schedule]
    num_scales = len(tokens)
    budgeted = num_scales - 1 if skip_last_scale else num_scales
    sources = tuple(range(s0, min(s1, num_scales - 1) + 1))
    if budgeted <= 0:
        empty = {s: {l: tuple() for l in range(num_layers)} for s in sources}
        return {"final_removed_counts": {i: 0 for i in range(num_scales)},
                "final_removed_by_scale": {i: empty for i in range(num_scales)},
                "early_activation_by_scale": {i: {} for i in range(num_scales)}}

    peak = sum(tokens[:budgeted])
    protected_tokens = sum(tokens[:min(int(protected_prefix_scales), num_scales)])
    min_budget = protected_tokens / peak if peak > 0 else 0.0
    if budget + 1e-12 < min_budget:
        raise ValueError(f"budget {budget} is below the minimum feasible ratio {min_budget:.12f}")
    threshold = budget * num_layers * num_heads * peak
    prune_counts = pruned_heads_for_budget(
        budget, retained_tokens=protected_tokens, num_layers=num_layers, num_heads=num_heads,
        skip_last_scale=skip_last_scale, scale_schedule=schedule)

    # the per-target loop (final removals, early activations, feasibility) in native code
    import ctypes

    import numpy as np

    from . import _native
    L, H, S = num_layers, num_heads, num_scales
    n_src = s1 - s0 + 1
    orders_arr = np.ascontiguousarray(np.array(seq, dtype=np.int32).reshape(n_src, L * H, 2))
    tok = np.array(tokens, dtype=np.int64)
    counts = np.array([int(prune_counts.get(i, 0)) for i in range(S)], dtype=np.int64)
    final_mask = np.empty((S, S, L, H), dtype=np.uint8)
    cap = max(1, S * n_src * L * H)
    early_arr = np.empty((cap, 5), dtype=np.int32)
    n_early = ctypes.c_int64(0)
    err = np.zeros(3, dtype=np.int64)
    status = _native.load().heatkv_strict_budget(
        orders_arr.ctypes.data, n_src, L, H, S, tok.ctypes.data, s0, int(protected_prefix_scales),
        budgeted, ctypes.c_double(threshold), counts.ctypes.data, final_mask.ctypes.data,
        early_arr.ctypes.data, cap, ctypes.byref(n_early), err.ctypes.data)
    if status != _native.HEATKV_OK:
        kind, t_err, l_err = (int(x) for x in err)
        if kind == 1:
            raise ValueError(f"budget {budget} is infeasible at scale index {t_err}, layer {l_err}")
        if kind == 2:
            raise ValueError(f"budget {budget} is infeasible at end of scale index {t_err}")
        if kind == 3:
            raise RuntimeError("strict scale-specific schedule failed to activate "
                               f"end-of-scale removals at scale index {t_err}")
        _native.check(status, "heatkv_strict_budget")
    final_counts, final_by_scale, early_by_scale = {}, {}, {}
    for t in range(S):
        idx = np.argwhere(final_mask[t])             # (source, layer, head), sorted
        atoms = [(int(a), int(c), int(b)) for a, b, c in idx]
        final_counts[t] = len(atoms)
        final_by_scale[t] = _atoms_by_source_and_layer(
            atoms, num_layers=num_layers, source_scale_indices=sources)
        early_by_scale[t] = {}
    for t, l, src, h, layer in early_arr[:n_early.value].tolist():
        early_by_scale[t].setdefault(l, []).append((src, h, layer))
    return {"final_removed_counts": final_counts, "final_removed_by_scale": final_by_scale,
            "early_activation_by_scale": early_by_scale}


def strict_removed_heads_by_scale_specific_for_budget(
    budget, scale_specific_removal_orders, *, num_layers=32, num_heads=16, source_scale_start=4,
    source_scale_end=11, protected_prefix_scales=4, skip_last_scale=True, strict_schedule=None,
    scale_schedule=None,
):
    """Per target scale: removed heads by source scale and layer, the removed-atom count and the
    count of remaining prunable atoms (reference keys ``removed_heads_by_scale``,
    ``removed_counts_by_scale``, ``remaining_atoms_by_scale``, ``strict_schedule``)."""
    seq = _validate_scale_specific_removal_orders(
        scale_specific_removal_orders, num_layers=num_layers, num_heads=num_heads,
        source_scale_start=source_scale_start, source_scale_end=source_scale_end)
    schedule_list = get_scale_schedule() if scale_schedule is None else list(scale_schedule)
    plan = strict_schedule
    if plan is None:
        plan = strict_pruning_schedule_for_budget_scale_specific(
            budget, seq, num_layers=num_layers, num_heads=num_heads,
            source_scale_start=source_scale_start, source_scale_end=source_scale_end,
            protected_prefix_scales=protected_prefix_scales, skip_last_scale=skip_last_scale,
            scale_schedule=schedule_list)
    num_scales = len(schedule_list)
    s0, s1 = int(source_scale_start), int(source_scale_end)
    sources = tuple(range(s0, min(s1, num_scales - 1) + 1))
    removed_by_scale, counts, remaining = {}, {}, {}
    prev_final = set()
    for t in range(num_scales):
        top = min(s1, t, num_scales - 1)
        eligible = top - s0 + 1 if top >= s0 else 0
        total_atoms = eligible * int(num_layers) * int(num_heads)
        here = set(prev_final)
        for atoms in plan["early_activation_by_scale"].get(t, {}).values():
            here.update(atoms)
        removed_by_scale[t] = _atoms_by_source_and_layer(
            here, num_layers=int(num_layers), source_scale_indices=sources)
        counts[t] = len(here)
        remaining[t] = total_atoms - len(here)
        prev_final = {
            (int(s), int(h), int(l))
            for s, by_layer in plan["final_removed_by_scale"].get(t, {}).items()
            for l, heads in by_layer.items()
            for h in heads
        }
    return {"removed_heads_by_scale": removed_by_scale, "removed_counts_by_scale": counts,
            "remaining_atoms_by_scale": remaining, "strict_schedule": plan}
