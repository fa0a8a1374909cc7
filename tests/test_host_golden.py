"""Host-side integer logic vs fixtures recorded from the reference (bit-exact).

Covers the budget policy (tools/utils.py:235-597), the controller (enable_pruning.py:328-401) and
the static slab schedule with its copy descriptors (enable_real_pruning_fast.py:206-671) for the
2B orders at 5/10/25/50/100 %, the 8B orders at 10 %, seeded random orders, and the 7-scale
config-1 keep-mask.
"""

import os

import numpy as np
import pytest

from heatkv_b200 import budget, synthetic
from heatkv_b200.enable_pruning import (
    ScaleSpecificPruningController,
    _validate_and_normalize_removed_heads_by_scale_specific,
)
from heatkv_b200.scheduler import build_static_slot_schedule, copy_descriptors

CONFIGS = {
    "2b_b05": ("2b", 32, 16, 0.05),
    "2b_b10": ("2b", 32, 16, 0.10),
    "2b_b25": ("2b", 32, 16, 0.25),
    "2b_b50": ("2b", 32, 16, 0.50),
    "2b_b100": ("2b", 32, 16, 1.00),
    "8b_b10": ("8b", 40, 28, 0.10),
    "rand_b05": ("rand", 32, 16, 0.05),
    "rand_b10": ("rand", 32, 16, 0.10),
    "rand_b25": ("rand", 32, 16, 0.25),
    "rand_b50": ("rand", 32, 16, 0.50),
    "rand_b100": ("rand", 32, 16, 1.00),
}


class _Mod:
    def __init__(self, h):
        self.num_heads = h


def _orders(kind, layers, heads):
    if kind == "rand":
        return synthetic.random_removal_orders(layers, heads, seed=1234)
    return budget.orders(model_type=int(kind[0]))


def _controller(name):
    kind, layers, heads, b = CONFIGS[name]
    view = budget.strict_removed_heads_by_scale_specific_for_budget(
        b, _orders(kind, layers, heads), num_layers=layers, num_heads=heads,
        source_scale_start=3, protected_prefix_scales=3)
    norm = _validate_and_normalize_removed_heads_by_scale_specific(
        view["removed_heads_by_scale"], [_Mod(heads)] * layers, source_scale_start=3)
    ctrl = ScaleSpecificPruningController(num_layers=layers, num_heads=heads,
                                          static_removed_heads_by_scale=norm, source_scale_start=3)
    return view, ctrl


@pytest.fixture(scope="module")
def controllers():
    return {}


def _get(controllers, name):
    if name not in controllers:
        controllers[name] = _controller(name)
    return controllers[name]


@pytest.mark.parametrize("name", list(CONFIGS))
def test_budget_policy_matches_reference(name, golden_dir, controllers):
    g = np.load(os.path.join(golden_dir, f"budget_{name}.npz"))
    kind, layers, heads, _ = CONFIGS[name]
    if kind == "rand":
        assert np.array_equal(np.array(_orders(kind, layers, heads), dtype=np.int16), g["orders"])
    view, _ = _get(controllers, name)
    ts = len(budget.get_scale_schedule())
    mine = np.zeros((ts, 9, layers, heads), dtype=np.uint8)
    for t, by_source in view["removed_heads_by_scale"].items():
        for s, by_layer in by_source.items():
            for l, hs in by_layer.items():
                for h in hs:
                    mine[t, s - 3, l, h] = 1
    assert np.array_equal(mine, g["removed"])
    assert [view["removed_counts_by_scale"][t] for t in range(ts)] == g["removed_counts"].tolist()
    assert [view["remaining_atoms_by_scale"][t] for t in range(ts)] == g["remaining_atoms"].tolist()


def _check_layer(g, layer, sched, heads, num_scales):
    pre = f"L{layer}_"
    caps = [sched["capacity"], sched["capacity_bound"], sched["allocated_capacity"],
            sched["overalloc_slots"]]
    assert caps == g[pre + "caps"].tolist()
    segs = np.array([[s["source_scale"], s["head"], s["start_target"], s["end_target"],
                      s["length"], s["offset"]] for s in sched["segments"]],
                    dtype=np.int32).reshape(-1, 6)
    assert np.array_equal(segs, g[pre + "segments"])
    rows = []
    for t in range(1, num_scales):
        st, en, ct = sched["metadata_cpu_by_target"][t]
        w = st.shape[1]
        for h in range(heads):
            rows.append([t, h, int(ct[h]), w] + st[h].tolist() + [-1] * (16 - w)
                        + en[h].tolist() + [-1] * (16 - w))
    assert np.array_equal(np.array(rows, dtype=np.int32), g[pre + "metadata"])
    pack = []
    for t, runs in sorted(sched["old_pack_runs_by_target"].items()):
        d = copy_descriptors(runs)
        if d is None:
            continue
        seq = sched["old_pack_cache_lens_by_target"][t]
        pack += [[t, seq, a, b, c] for a, b, c in zip(d["dst_starts"], d["src_starts"], d["lengths"])]
    assert np.array_equal(np.array(pack, dtype=np.int64).reshape(-1, 5), g[pre + "old_pack"])
    app = []
    for (cur, nxt), runs in sorted(sched["append_runs_by_key"].items()):
        d = copy_descriptors(runs)
        if d is None:
            continue
        app += [[cur, nxt, a, b, c] for a, b, c in zip(d["dst_starts"], d["src_starts"], d["lengths"])]
    assert np.array_equal(np.array(app, dtype=np.int64).reshape(-1, 5), g[pre + "append"])


@pytest.mark.parametrize("name", list(CONFIGS))
def test_static_schedule_matches_reference(name, golden_dir, controllers):
    g = np.load(os.path.join(golden_dir, f"schedule_{name}.npz"))
    _, layers, heads, _ = CONFIGS[name]
    _, ctrl = _get(controllers, name)
    layer_ids = sorted({int(k.split("_")[0][1:]) for k in g.files})
    assert layer_ids, "fixture holds no layer"
    for layer in layer_ids:
        sched = build_static_slot_schedule(ctrl, layer_idx=layer, num_heads=heads)
        _check_layer(g, layer, sched, heads, len(ctrl.scale_schedule))


class _SevenScaleRemoved:
    def __init__(self, pairs):
        self.pairs = pairs

    def __call__(self, layer, target):
        out = {}
        for s, h in self.pairs:
            if s < target:
                out.setdefault(s, set()).add(h)
        return out


def config1_controller():
    cfg = synthetic.config1()
    num_scales = len(synthetic.C1_SCALE_SCHEDULE)
    static = {}
    for t in range(num_scales):
        by_source = {s: {0: set()} for s in range(3, 12)}
        for s, h in cfg.removed_pairs:
            if s < t:
                by_source[s][0].add(h)
        static[t] = by_source
    ctrl = ScaleSpecificPruningController(num_layers=1, num_heads=cfg.num_heads,
                                          static_removed_heads_by_scale=static,
                                          source_scale_start=3,
                                          scale_schedule=synthetic.C1_SCALE_SCHEDULE)
    return cfg, ctrl


def test_config1_schedule_matches_reference(golden_dir):
    g = np.load(os.path.join(golden_dir, "schedule_c1.npz"))
    cfg, ctrl = config1_controller()
    sched = build_static_slot_schedule(ctrl, layer_idx=0, num_heads=cfg.num_heads)
    _check_layer(g, 0, sched, cfg.num_heads, len(synthetic.C1_SCALE_SCHEDULE))
    p = np.load(os.path.join(golden_dir, "pack_c1.npz"))
    assert sched["capacity"] == int(p["capacity"][0])


def test_budget_errors_match_reference_messages():
    with pytest.raises(ValueError, match=r"budget must be in \[0, 1\], got 1.5"):
        budget.pruned_heads_for_budget(1.5)
    with pytest.raises(ValueError, match="below the minimum feasible ratio"):
        budget.strict_pruning_schedule_for_budget_scale_specific(
            0.001, budget.orders(model_type=2), source_scale_start=3, protected_prefix_scales=3)
    bad = [list(o) for o in budget.orders(model_type=2)]
    bad[0][1] = list(bad[0][0])
    with pytest.raises(ValueError, match="duplicate"):
        budget.strict_removed_heads_by_scale_specific_for_budget(0.1, bad, source_scale_start=3)
    with pytest.raises(ValueError, match="must contain exactly 9 orders"):
        budget.strict_removed_heads_by_scale_specific_for_budget(0.1, bad[:3], source_scale_start=3)


def test_controller_from_prune_counts_matches_static_view():
    orders = budget.orders(model_type=2)
    counts = {t: (0 if t < 8 else 100 * (t - 7)) for t in range(13)}
    ctrl = ScaleSpecificPruningController(num_layers=32, num_heads=16, prune_counts=counts,
                                          scale_specific_removal_orders=orders,
                                          source_scale_start=3)
    for t in (8, 12):
        by_source = ctrl.removed_heads_by_source_for(5, t)
        assert set(by_source) == set(range(3, min(11, t - 1) + 1))
        for s, heads in by_source.items():
            expect = {h for h, l in orders[s - 3][:counts[t]] if l == 5}
            assert heads == expect
