"""Removal-order validation and the scale-specific pruning controller (host side).

Same names, arguments, results and error messages as the reference's ``enable_pruning.py``:
``_assign_layer_indices`` (:10-12), ``_validate_and_normalize_removal_order`` (:15-45),
``_validate_and_normalize_scale_specific_removal_orders`` (:91-112),
``_validate_and_normalize_removed_heads_by_scale_specific`` (:115-179), ``_scale_token_ranges``
(:182-189) and ``ScaleSpecificPruningController`` (:328-401).

The controller additionally keeps the removed sets as a dense ``uint8`` array
``[target, source, layer, head]`` so the slot scheduler can derive every (source, head) live
interval with array operations; ``removed_heads_by_source_for`` answers from the same data.
The controller also accepts an explicit ``scale_schedule`` (the reference always uses the 13-scale
``get_scale_schedule()``), which the 7-scale configuration needs.
"""

from __future__ import annotations

import numpy as np

from .budget import get_scale_schedule


def _assign_layer_indices(modules):
    for layer_idx, module in enumerate(modules):
        module.layer_idx = layer_idx


def _validate_and_normalize_removal_order(removal_order, modules):
    if not modules:
        raise ValueError("model does not contain any SelfAttention modules")
    num_layers = len(modules)
    expected = sum(m.num_heads for m in modules)
    if len(removal_order) != expected:
        raise ValueError(f"expected {expected} removal-order entries, got {len(removal_order)}")
    out, seen = [], set()
    for idx, pair in enumerate(removal_order):
        if not isinstance(pair, (tuple, list)) or len(pair) != 2:
            raise ValueError(f"removal_order[{idx}] must be a (head, layer) tuple")
        head, layer = int(pair[0]), int(pair[1])
        if not 0 <= layer < num_layers:
            raise ValueError(f"layer index out of range at position {idx}: {layer}")
        if not 0 <= head < modules[layer].num_heads:
            raise ValueError(f"head index out of range at position {idx}: {head}")
        if (head, layer) in seen:
            raise ValueError(f"duplicate (head, layer) entry at position {idx}: {(head, layer)}")
        seen.add((head, layer))
        out.append((head, layer))
    return out


def _validate_and_normalize_scale_specific_removal_orders(orders, modules, *, source_scale_start=4,
                                                          source_scale_end=11):
    expected = source_scale_end - source_scale_start + 1
    if len(orders) != expected:
        raise ValueError(
            "scale_specific_removal_orders must contain exactly "
            f"{expected} orders for source scales {source_scale_start}-{source_scale_end}"
        )
    return tuple(_validate_and_normalize_removal_order(o, modules) for o in orders)


def _validate_and_normalize_removed_heads_by_scale_specific(removed_heads_by_scale, modules, *,
                                                            source_scale_start=4,
                                                            source_scale_end=11):
    if not modules:
        raise ValueError("model does not contain any SelfAttention modules")
    num_layers = len(modules)
    normalized = {}
    for target, source_map in removed_heads_by_scale.items():
        target = int(target)
        if not isinstance(source_map, dict):
            raise ValueError(f"removed_heads_by_scale[{target}] must be a dict")
        norm_sources = {s: {l: set() for l in range(num_layers)}
                        for s in range(int(source_scale_start), int(source_scale_end) + 1)}
        for source, layer_map in source_map.items():
            source = int(source)
            if not int(source_scale_start) <= source <= int(source_scale_end):
                raise ValueError(
                    f"removed_heads_by_scale[{target}] source scale out of range: {source}")
            if not isinstance(layer_map, dict):
                raise ValueError(f"removed_heads_by_scale[{target}][{source}] must be a dict")
            norm_layers = {l: set() for l in range(num_layers)}
            for layer, heads in layer_map.items():
                layer = int(layer)
                if not 0 <= layer < num_layers:
                    raise ValueError(
                        f"removed_heads_by_scale[{target}][{source}] layer index out of range: {layer}")
                seen = set()
                for head in heads:
                    head = int(head)
                    if not 0 <= head < modules[layer].num_heads:
                        raise ValueError(
                            f"removed_heads_by_scale[{target}][{source}] "
                            f"head index out of range for layer {layer}: {head}")
                    if head in seen:
                        raise ValueError(
                            f"removed_heads_by_scale[{target}][{source}] "
                            f"duplicate head {head} for layer {layer}")
                    seen.add(head)
                    norm_layers[layer].add(head)
            norm_sources[source] = norm_layers
        normalized[target] = norm_sources
    return normalized


def _scale_token_ranges(scale_schedule):
    ranges, cursor = {}, 0
    for idx, (_, h, w) in enumerate(scale_schedule):
        ranges[idx] = (cursor, cursor + int(h) * int(w))
        cursor += int(h) * int(w)
    return ranges


class ScaleSpecificPruningController:
    """Static per-(layer, target scale, source scale) removed-head sets.

    Built either from ``static_removed_heads_by_scale`` (``{target: {source: {layer: heads}}}``)
    or from ``prune_counts`` + ``scale_specific_removal_orders`` (the first ``count`` entries of
    each source order are removed at that target, enable_pruning.py:346-368). Targets missing
    from the map use the nearest earlier target (enable_pruning.py:387-401).
    """

    def __init__(self, *, num_layers, num_heads, static_removed_heads_by_scale=None,
                 prune_counts=None, scale_specific_removal_orders=None, source_scale_start=4,
                 source_scale_end=11, scale_schedule=None):
        self.num_layers = int(num_layers)
        self.num_heads = int(num_heads)
        self.source_scale_start = int(source_scale_start)
        self.source_scale_end = int(source_scale_end)
        self.scale_schedule = get_scale_schedule() if scale_schedule is None else [
            tuple(x) for x in scale_schedule]
        self.scale_ranges = _scale_token_ranges(self.scale_schedule)
        num_scales = len(self.scale_schedule)
        n_src = self.source_scale_end - self.source_scale_start + 1
        self._sources = tuple(range(self.source_scale_start, self.source_scale_end + 1))
        if static_removed_heads_by_scale is not None:
            static = static_removed_heads_by_scale
        else:
            self.prune_counts = dict(prune_counts)
            static = {}
            total = self.num_layers * self.num_heads
            for t in range(num_scales):
                count = max(0, min(total, int(self.prune_counts.get(t, 0))))
                by_source = {}
                for s in range(self.source_scale_start, min(self.source_scale_end, t - 1) + 1):
                    removed = {l: set() for l in range(self.num_layers)}
                    for head, layer in scale_specific_removal_orders[s - self.source_scale_start][:count]:
                        removed[layer].add(head)
                    by_source[s] = removed
                static[t] = by_source
        self._static_removed_heads_by_scale = static
        # dense view [target, source - start, layer, head]; sources absent from a target's map
        # are flagged so removed_heads_by_source_for reproduces the map's key set.
        self._mask = np.zeros((num_scales, n_src, self.num_layers, self.num_heads), dtype=np.uint8)
        self._present = np.zeros((num_scales, n_src), dtype=bool)
        for t in range(num_scales):
            state = self._removed_heads_state(t)
            for s, by_layer in state.items():
                si = int(s) - self.source_scale_start
                if not 0 <= si < n_src:
                    continue
                self._present[t, si] = True
                for l, heads in by_layer.items():
                    for h in heads:
                        self._mask[t, si, int(l), int(h)] = 1

    def reset(self):
        return None

    def _removed_heads_state(self, target_scale_idx):
        static = self._static_removed_heads_by_scale
        if target_scale_idx in static:
            return static[target_scale_idx]
        earlier = [t for t in static if t <= target_scale_idx]
        if not earlier:
            return {s: {l: set() for l in range(self.num_layers)} for s in self._sources}
        return static[max(earlier)]

    def removed_heads_for(self, layer_idx, target_scale_idx, source_scale_idx):
        return set(self._removed_heads_state(target_scale_idx).get(source_scale_idx, {}).get(
            layer_idx, set()))

    def removed_heads_by_source_for(self, layer_idx, target_scale_idx):
        state = self._removed_heads_state(target_scale_idx)
        return {s: set(by_layer.get(layer_idx, set())) for s, by_layer in state.items()}

    def removed_mask_for_layer(self, layer_idx: int) -> np.ndarray:
        """``uint8 [num_scales(target), num_scales(source), H]``: 1 where head ``h`` of source
        scale ``s`` is removed at target ``t`` for this layer (sources outside the prunable range
        are never removed)."""
        num_scales = len(self.scale_schedule)
        out = np.zeros((num_scales, num_scales, self.num_heads), dtype=np.uint8)
        lo = self.source_scale_start
        hi = min(self.source_scale_end, num_scales - 1)
        if hi >= lo:
            out[:, lo:hi + 1, :] = self._mask[:, : hi - lo + 1, int(layer_idx), :]
        return out

    def any_removed(self, layer_idx: int, target_scale_idx: int) -> bool:
        """True when the removed-head map of (layer, target) holds at least one head (a table
        built once: the mask is fixed at construction and this runs every layer and scale)."""
        table = self.__dict__.get("_any_removed")
        if table is None:
            table = self._any_removed = self._mask.any(axis=(1, 3)).tolist()
        t = min(int(target_scale_idx), len(table) - 1)
        return table[t][int(layer_idx)]
