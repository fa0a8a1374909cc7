"""The whole per-image hot path on the GPU (dense-prefix scales, slab activation, per-scale appends,
fused segmented attention) against an independent formulation: for every (layer, target, head)
attention over exactly the tokens the keep-mask retains - scales 0..2 always, scale s >= 3 unless
the controller removes (s, head) at that target - computed with plain PyTorch fp32 on the GPU.
This checks the slab schedule, the pack descriptors and the kernel together at full 13-scale size.
"""

import pytest
import torch

from heatkv_b200 import _native
from heatkv_b200.hotpath import HotPath, allocate_io

from _keepmask import keep_mask_attention

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_REL = 2e-2, 1e-2


def _controller(model, budget):
    import bench
    return bench.build_controller(model, budget)


def _reference(ctrl, layer, t, inputs_layer, head_dim=128):
    return keep_mask_attention(ctrl, layer, t, inputs_layer)


@pytest.mark.parametrize("model,budget,layers", [("2b", 0.10, [0, 21]), ("2b", 0.05, [3]),
                                                 ("2b", 1.00, [7]), ("8b", 0.10, [39])])
def test_hot_path_matches_keep_mask_attention(model, budget, layers):
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller(model, budget)
    hot = HotPath(ctrl, L, H, 2, dev, torch.bfloat16, torch.bfloat16, layers=layers)
    inputs, outputs, _, _ = allocate_io(hot, seed=3)
    hot.run(hot.launches(inputs, outputs))
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    for i, layer in enumerate(layers):
        for t in range(hot.num_scales):
            ref = _reference(ctrl, layer, t, inputs[i])
            err = (outputs[i][t].float() - ref).abs().max().item()
            scale = ref.abs().max().item()
            assert err <= BF16_ATOL and err / scale <= BF16_REL, (layer, t, err, scale)


def test_hot_path_every_layer_of_configs1():
    """configs[1] at full size: all 32 layers of the 2B model at 10 %, 2 rows, every target."""
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller("2b", 0.10)
    layers = list(range(L))
    hot = HotPath(ctrl, L, H, 2, dev, torch.bfloat16, torch.bfloat16, layers=layers)
    inputs, outputs, _, _ = allocate_io(hot, seed=11)
    hot.run(hot.launches(inputs, outputs))
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    for i, layer in enumerate(layers):
        for t in range(hot.num_scales):
            ref = _reference(ctrl, layer, t, inputs[i])
            err = (outputs[i][t].float() - ref).abs().max().item()
            scale = ref.abs().max().item()
            assert err <= BF16_ATOL and err / scale <= BF16_REL, (layer, t, err, scale)


def _random_controller(budget, seed, layers=32, heads=16):
    """2B-shaped controller from seeded random per-source removal orders (the budget sweep)."""
    from heatkv_b200 import budget as bud, synthetic
    from heatkv_b200.enable_pruning import (ScaleSpecificPruningController,
                                            _validate_and_normalize_removed_heads_by_scale_specific)

    class _M:
        num_heads = heads

    orders = synthetic.random_removal_orders(layers, heads, seed=seed)
    view = bud.strict_removed_heads_by_scale_specific_for_budget(
        budget, orders, num_layers=layers, num_heads=heads, source_scale_start=3,
        protected_prefix_scales=3)
    norm = _validate_and_normalize_removed_heads_by_scale_specific(
        view["removed_heads_by_scale"], [_M()] * layers, source_scale_start=3)
    return ScaleSpecificPruningController(num_layers=layers, num_heads=heads,
                                          static_removed_heads_by_scale=norm, source_scale_start=3)


@pytest.mark.parametrize("budget,rows,layer", [(0.25, 16, 5), (0.5, 16, 30), (0.05, 16, 12),
                                               (0.10, 16, 17), (1.00, 16, 25)])
def test_hot_path_budget_sweep_batch16(budget, rows, layer):
    """Budget sweep shape (2B, 16 rows = batch 8 + CFG, seeded random orders): uneven slab
    lengths per head, several query blocks per CTA."""
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    ctrl = _random_controller(budget, seed=1234)
    hot = HotPath(ctrl, 32, 16, rows, dev, torch.bfloat16, torch.bfloat16, layers=[layer])
    inputs, outputs, _, _ = allocate_io(hot, seed=9)
    hot.run(hot.launches(inputs, outputs))
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    for t in range(hot.num_scales):
        ref = _reference(ctrl, layer, t, inputs[0])
        err = (outputs[0][t].float() - ref).abs().max().item()
        scale = ref.abs().max().item()
        assert err <= BF16_ATOL and err / scale <= BF16_REL, (layer, t, err, scale)


def test_hot_path_8b_batch8():
    """configs[2] shape: 8B (28 heads), batch 4 + CFG = 8 rows, orders/8b.json at 10 %."""
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    ctrl, L, H = _controller("8b", 0.10)
    hot = HotPath(ctrl, L, H, 8, dev, torch.bfloat16, torch.bfloat16, layers=[20])
    inputs, outputs, _, _ = allocate_io(hot, seed=4)
    hot.run(hot.launches(inputs, outputs))
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    for t in range(hot.num_scales):
        ref = _reference(ctrl, 20, t, inputs[0])
        err = (outputs[0][t].float() - ref).abs().max().item()
        scale = ref.abs().max().item()
        assert err <= BF16_ATOL and err / scale <= BF16_REL, (t, err, scale)


def test_batched_scale_packs_equal_per_layer_packs():
    """One batched compaction launch per scale leaves the same slabs and outputs, bit for bit, as
    one pack launch per layer (the orchestrator's order)."""
    ctrl, L, H = _controller("2b", 0.10)
    dev = torch.device("cuda", 0)
    layers = [0, 9, 30]
    results = []
    for batched in (False, True):
        hot = HotPath(ctrl, L, H, 2, dev, layers=layers)
        inputs, outputs, _, _ = allocate_io(hot, seed=3)
        launches = hot.launches(inputs, outputs, batch_packs=batched)
        packs = sum(1 for l in launches if l.kind == "pack")
        hot.run(launches)
        torch.cuda.synchronize()
        results.append((packs, [o.clone() for row in outputs for o in row],
                        [s.clone() for s in hot.slab_k + hot.slab_v]))
    (n0, out0, slab0), (n1, out1, slab1) = results
    assert n1 < n0
    assert all(torch.equal(a, b) for a, b in zip(out0, out1))
    assert all(torch.equal(a, b) for a, b in zip(slab0, slab1))
    assert _native.device_status(dev) == 0


def test_dense_append_first_matches_append_after():
    """Appending each dense scale to the dense cache before its attention, which then walks one
    segment of cached tokens + scale per head (HEATKV_ATTN_CURRENT_IN_SEGMENTS), against the
    reference's order (append after the attention, current scale as separate tiles): the same
    slabs bit for bit and the outputs within bf16 tolerance of each other (only the key-tile
    partition of the dense targets differs)."""
    ctrl, L, H = _controller("2b", 0.10)
    dev = torch.device("cuda", 0)
    layers = [0, 17]
    results = []
    for first in (False, True):
        hot = HotPath(ctrl, L, H, 2, dev, layers=layers, dense_append_first=first)
        inputs, outputs, _, _ = allocate_io(hot, seed=9)
        launches = hot.launches(inputs, outputs)
        pre = [l for l in launches if l.kind == "pack" and l.sources]
        assert bool(pre) == first
        hot.run(launches)
        torch.cuda.synchronize()
        results.append(([o.clone() for row in outputs for o in row],
                        [s.clone() for s in hot.slab_k + hot.slab_v]))
    (out0, slab0), (out1, slab1) = results
    assert all(torch.equal(a, b) for a, b in zip(slab0, slab1))
    for a, b in zip(out0, out1):
        err = (a.float() - b.float()).abs().max().item()
        assert err <= BF16_ATOL and err / max(b.float().abs().max().item(), 1e-6) <= BF16_REL
    assert _native.device_status(dev) == 0


def test_merged_prefix_matches_reference_layout():
    """The protected prefix scales read as one segment per head from a contiguous copy past the
    reference slab layout (HotPath(merge_prefix=True), the default) against the reference layout's
    three segments: the reference region of every slab bit for bit, outputs within bf16 tolerance
    (only the key-tile partition differs), and fewer key tiles."""
    ctrl, L, H = _controller("2b", 0.10)
    dev = torch.device("cuda", 0)
    layers = [2, 21]
    results = []
    for merge in (False, True):
        hot = HotPath(ctrl, L, H, 2, dev, layers=layers, merge_prefix=merge)
        inputs, outputs, _, _ = allocate_io(hot, seed=13)
        hot.run(hot.launches(inputs, outputs))
        torch.cuda.synchronize()
        assert _native.device_status(dev) == 0
        results.append((hot, [o.clone() for row in outputs for o in row],
                        [s.clone() for s in hot.slab_k + hot.slab_v]))
    (h0, out0, slab0), (h1, out1, slab1) = results
    for p0, p1 in zip(h0.plans, h1.plans):
        assert p1.prefix_scales == 3 and p1.capacity == p0.capacity + H * p1.prefix_len
        t = p1.first_target
        assert sum(map(len, p1.segment_lengths(t))) == sum(map(len, p0.segment_lengths(t))) - 2 * H
    for a, b in zip(slab0, slab1):
        assert torch.equal(a, b[:, :a.shape[1]])
    for a, b in zip(out0, out1):
        err = (a.float() - b.float()).abs().max().item()
        assert err <= BF16_ATOL and err / max(b.float().abs().max().item(), 1e-6) <= BF16_REL
