"""Host-side plan of the projection-driven hot path (no GPU: tensors on the CPU, no launch runs).

Checks that every scale's K/V reach the layer's caches exactly once - the preparation's early
appends (dense cache before the first pruned target, hazard-free slab heads after it) plus the
copies left for after the attention add up to the reference's append runs
(enable_real_pruning_fast.py:969-1024) - and the launch order per (scale, layer).
"""

import numpy as np
import pytest
import torch

from heatkv_b200.hotpath import HotPath
from heatkv_b200.projected import ProjectedHotPath
from heatkv_b200.scheduler import copy_descriptors


def _controller():
    import bench
    return bench.build_controller("2b", 0.10)


def test_projected_appends_cover_the_schedule():
    ctrl, L, H = _controller()
    layers = [0, 13, 31]
    hot = HotPath(ctrl, L, H, 2, "cpu", layers=layers)
    proj = ProjectedHotPath(hot)
    want = 0
    for p in hot.plans:
        for t in range(hot.num_scales - 1):
            if t < p.first_target:
                want += H * hot.tokens[t] if t in p.dense_append else 0
            else:
                d = copy_descriptors(p.schedule["append_runs_by_key"].get((t, t + 1), []))
                want += 0 if d is None else d["slots"]
    assert proj.early_slots + proj.rest_slots == want
    assert proj.early_slots > proj.rest_slots > 0
    # the early slab heads never touch a slot the same scale's attention reads
    for (i, t), (sk, sv, rows, offs, written) in proj.prep_target.items():
        p = hot.plans[i]
        if t < p.first_target:
            assert sk is hot.dense_k[i] and rows == H * p.dense_len
            continue
        n = hot.tokens[t]
        live = p.schedule["segments_by_target"][t]
        for h, off in enumerate(offs.numpy().tolist()):
            if off < 0:
                continue
            for seg in live:
                assert off + n <= seg["offset"] or seg["offset"] + seg["length"] <= off


@pytest.mark.parametrize("fused", [True, False])
def test_projected_launch_order(fused):
    ctrl, L, H = _controller()
    layers = [0, 21]
    hot = HotPath(ctrl, L, H, 2, "cpu", layers=layers)
    proj = ProjectedHotPath(hot, fused_projection=fused)
    x = [torch.empty(2, n, H * 128, dtype=torch.bfloat16) for n in hot.tokens]
    out = [torch.empty(2, n, H * 128, dtype=torch.bfloat16) for n in hot.tokens]
    launches = proj.launches(x, out)
    kinds = [l.kind for l in launches]
    first = ("proj",) if fused else ("gemm", "prep")
    for k in first + ("attention",):
        assert kinds.count(k) == len(layers) * hot.num_scales
    # per (scale, layer): the projection (one or two launches), attention, then optional packs
    seq = [(l.kind, l.layer, l.target) for l in launches if l.kind != "pack"]
    step = len(first) + 1
    for j in range(0, len(seq), step):
        group = seq[j:j + step]
        assert tuple(g[0] for g in group) == first + ("attention",)
        assert len({(g[1], g[2]) for g in group}) == 1
    # one activation pack per scale that precedes some layer's first pruned target
    acts = {p.first_target - 1 for p in hot.plans if p.activation is not None}
    batched = [l for l in launches if l.kind == "pack" and l.layer == -1]
    assert sorted(l.target for l in batched) == sorted(acts)
    assert np.isclose(sum(l.work for l in launches if l.kind in ("gemm", "proj")),
                      sum(2.0 * 2 * n * 2048 * 6144 for n in hot.tokens) * len(layers))
