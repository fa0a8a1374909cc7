"""The drop-in installer end to end on a small Infinity-shaped model (GPU): after
``enable_real_pruning_scale_specific_fused_segmented`` every layer's output at every one of the 13
scales equals attention over exactly the tokens the keep-mask retains (plain PyTorch fp32 on the
GPU), through the model's own projections. bf16 model (tcgen05 kernel, 2e-2 / 1e-2), fp32
cos-attn model (exact kernel; the attention output itself, the output projection set to the
identity, at 1e-5), and fp32 cos-attn model under bf16 autocast, the real model's setting: q and
k fp32, v bf16 (tf32 tcgen05 kernel, 2e-2 / 1e-2). The scales before a layer's first pruned target
run through the segmented kernel over a preallocated dense cache by default, and through the
reference's SDPA route with ``dense_prefix="sdpa"``; both are checked."""

import contextlib

import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from heatkv_b200 import _native, synthetic
from heatkv_b200.enable_real_pruning_fast import (
    enable_real_pruning_scale_specific_fused_segmented,
    set_real_pruning_fast_phase_profile_enabled,
    snapshot_real_pruning_fast_phase_profile,
)

pytestmark = pytest.mark.gpu


def apply_rotary_emb(q, k, scale_schedule, rope2d_freqs_grid, pad_to_multiplier,
                     rope2d_normalized_by_hw, scale_ind):
    """The 2-D rotary embedding of infinity/models/basic.py:97-117, restated; the drop-in looks
    it up beside the attention class, as it does in the Infinity model."""
    qk = torch.stack((q, k), dim=0)
    with torch.autocast(device_type="cuda", enabled=False):
        seq_len = qk.shape[3]
        start = sum(a * b * c for a, b, c in scale_schedule[:scale_ind]) if scale_ind >= 1 else 0
        cache = rope2d_freqs_grid[str(tuple(scale_schedule))].to(qk.device)[:, :, :, :, start:start + seq_len]
        qk = qk.reshape(*qk.shape[:-1], -1, 2)
        qk = torch.stack([cache[0] * qk[..., 0] - cache[1] * qk[..., 1],
                          cache[1] * qk[..., 0] + cache[0] * qk[..., 1]], dim=-1)
        qk = qk.reshape(*qk.shape[:-2], -1)
        q, k = qk.unbind(dim=0)
    return q, k


class SelfAttention(nn.Module):
    """Infinity's self-attention (infinity/models/basic.py:196-316, customized_flash_attn=False)
    reduced to what the installer touches."""

    def __init__(self, embed_dim, num_heads, cos_attn):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, embed_dim // num_heads
        self.cos_attn = cos_attn
        if cos_attn:
            self.scale = 1
            self.scale_mul_1H11 = nn.Parameter(torch.full((1, num_heads, 1, 1), 4.0).log())
            self.max_scale_mul = math.log(100)
        else:
            self.scale = 1 / math.sqrt(self.head_dim)
        self.mat_qkv = nn.Linear(embed_dim, embed_dim * 3, bias=False)
        self.q_bias = nn.Parameter(torch.randn(embed_dim) * 0.02)
        self.v_bias = nn.Parameter(torch.randn(embed_dim) * 0.02)
        self.register_buffer("zero_k_bias", torch.zeros(embed_dim))
        self.proj = nn.Linear(embed_dim, embed_dim)
        self.proj_drop = nn.Identity()
        self.caching, self.cached_k, self.cached_v = False, None, None
        self.pad_to_multiplier, self.rope2d_normalized_by_hw = 1, 0

    def kv_caching(self, enable):
        self.caching, self.cached_k, self.cached_v = enable, None, None

    def qkv(self, x):
        B, L, C = x.shape
        qkv = F.linear(x, self.mat_qkv.weight, torch.cat((self.q_bias, self.zero_k_bias, self.v_bias)))
        q, k, v = qkv.view(B, L, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4).unbind(0)
        if self.cos_attn:
            mul = self.scale_mul_1H11.clamp_max(self.max_scale_mul).exp()
            q = F.normalize(q, dim=-1, eps=1e-12).mul(mul)
            k = F.normalize(k, dim=-1, eps=1e-12)
        return q.contiguous(), k.contiguous(), v.contiguous()

    def forward(self, x, attn_bias_or_two_vector, attn_fn=None, scale_schedule=None,
                rope2d_freqs_grid=None, scale_ind=0):
        B, L, C = x.shape
        q, k, v = self.qkv(x)
        if rope2d_freqs_grid is not None:
            q, k = apply_rotary_emb(q, k, scale_schedule, rope2d_freqs_grid, 1, 0, scale_ind)
        if self.caching:
            if self.cached_k is None:
                self.cached_k, self.cached_v = k, v
            else:
                k = self.cached_k = torch.cat((self.cached_k, k), dim=2)
                v = self.cached_v = torch.cat((self.cached_v, v), dim=2)
        out = F.scaled_dot_product_attention(q, k, v, scale=self.scale)
        return self.proj_drop(self.proj(out.transpose(1, 2).reshape(B, L, C)))


def _autocast(enabled):
    return torch.autocast("cuda", dtype=torch.bfloat16) if enabled else contextlib.nullcontext()


def _masked_reference(module, ctrl, layer, xs, t, autocast=False):
    """Attention of scale t's queries over the retained earlier tokens + scale t, fp32 (q, k, v
    computed as the model computes them, under autocast when the model ran under it)."""
    with torch.no_grad():
        with _autocast(autocast):
            qkv = [module.qkv(x) for x in xs[: t + 1]]
        q = qkv[t][0].float()
        k = torch.cat([z[1] for z in qkv], dim=2).float()
        v = torch.cat([z[2] for z in qkv], dim=2).float()
        mask = ctrl.removed_mask_for_layer(layer)
        ranges = ctrl.scale_ranges
        B, H, n, D = q.shape
        out = torch.empty(B, n, H, D, device=q.device)
        for h in range(H):
            idx = [torch.arange(*ranges[s]) for s in range(t) if not mask[t, s, h]]
            idx.append(torch.arange(*ranges[t]))
            idx = torch.cat(idx).to(q.device)
            att = torch.softmax((q[:, h] @ k[:, h, idx].transpose(-1, -2)) * module.scale, -1)
            out[:, :, h] = att @ v[:, h, idx]
        out = out.reshape(B, n, H * D)
        if isinstance(module.proj, nn.Linear):
            out = module.proj(out.to(module.proj.weight.dtype))
        return out.float()


@pytest.mark.parametrize("dense_prefix", ["kernel", "sdpa"])
@pytest.mark.parametrize("dtype,cos_attn,autocast,atol,rel", [
    (torch.bfloat16, False, False, 2e-2, 1e-2),
    (torch.float32, True, False, 1e-5, 1e-5),
    (torch.float32, True, True, 2e-2, 1e-2),
])
def test_installed_model_matches_keep_mask_attention(dtype, cos_attn, autocast, atol, rel,
                                                     dense_prefix):
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    L, H, C = 3, 16, 2048
    model = nn.ModuleList([SelfAttention(C, H, cos_attn) for _ in range(L)]).to(dev, dtype)
    if dtype == torch.float32 and not autocast:
        for m in model:   # compare the attention output itself at the fp32 tolerance
            m.proj = nn.Identity()
    orders = synthetic.random_removal_orders(L, H, seed=7)
    enable_real_pruning_scale_specific_fused_segmented(
        model, 0.10, orders, protected_prefix_scales=3, source_scale_start=3,
        dense_prefix=dense_prefix)
    ctrl = model[0]._real_pruning_scale_specific_controller
    for m in model:
        m.kv_caching(True)
    set_real_pruning_fast_phase_profile_enabled(True)
    schedule = synthetic.SCALE_SCHEDULE_1M
    xs = {l: [torch.randn(2, h * w, C, device=dev, dtype=dtype) for _, h, w in schedule]
          for l in range(L)}
    outs = {l: [] for l in range(L)}
    if autocast:  # the premise: cos-attn under bf16 autocast gives fp32 q, k and bf16 v
        with torch.no_grad(), _autocast(True):
            q, k, v = model[0].qkv(xs[0][1])
        assert (q.dtype, k.dtype, v.dtype) == (torch.float32, torch.float32, torch.bfloat16)
    with torch.no_grad(), _autocast(autocast):
        for t in range(len(schedule)):
            for l, m in enumerate(model):
                outs[l].append(m(xs[l][t], None, scale_ind=t))
    prof = snapshot_real_pruning_fast_phase_profile(reset=True)
    set_real_pruning_fast_phase_profile_enabled(False)
    assert prof["calls"].get("attention", 0) > 0 and prof["calls"].get("compact", 0) > 0
    assert any(m._real_pruning_segmented_cache_active is False for m in model)  # freed at the end
    assert _native.device_status(dev) == 0
    for l, m in enumerate(model):
        for t in range(len(schedule)):
            ref = _masked_reference(m, ctrl, l, xs[l], t, autocast)
            err = (outs[l][t].float() - ref).abs().max().item()
            assert err <= atol and err / ref.abs().max().item() <= rel, (l, t, err)


def test_fused_qkv_prep_matches_the_torch_chain():
    """fused_qkv_prep=True against the PyTorch chain, on cos-attention models with a 2-D rope cache
    under bf16 autocast (fp32 q, k and bf16 v: the real model's dtypes) and non-zero q/v biases,
    every layer at every one of the 13 scales. Under autocast the fused path is the QKV projection
    with the preparation in its epilogue (heatkv_qkv_project); the chain is F.linear, then
    unbind / permute / normalisation / RoPE in PyTorch."""
    dev = torch.device("cuda", 0)
    L, H, C = 2, 16, 2048
    schedule = synthetic.SCALE_SCHEDULE_1M
    n_tok = sum(a * b * c for a, b, c in schedule)
    g = torch.Generator().manual_seed(9)
    angles = torch.rand(1, 1, 1, n_tok, 64, generator=g) * 6.0
    freqs = {str(tuple(schedule)): torch.stack([torch.cos(angles), torch.sin(angles)]).to(dev)}
    orders = synthetic.random_removal_orders(L, H, seed=7)
    xs = None
    outs = []
    for fused in (False, True):
        torch.manual_seed(0)
        model = nn.ModuleList([SelfAttention(C, H, True) for _ in range(L)]).to(dev)
        with torch.no_grad():
            for m in model:
                m.q_bias.normal_(0.0, 0.1)
                m.v_bias.normal_(0.0, 0.1)
        enable_real_pruning_scale_specific_fused_segmented(
            model, 0.10, orders, protected_prefix_scales=3, source_scale_start=3,
            fused_qkv_prep=fused)
        for m in model:
            m.kv_caching(True)
        if xs is None:
            xs = [[torch.randn(2, h * w, C, device=dev) for _, h, w in schedule] for _ in range(L)]
        res = []
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            for t in range(len(schedule)):
                for l, m in enumerate(model):
                    res.append(m(xs[l][t], None, scale_schedule=schedule, rope2d_freqs_grid=freqs,
                                 scale_ind=t).float())
        outs.append(res)
    assert _native.device_status(dev) == 0
    for a, b in zip(*outs):
        err = (a - b).abs().max().item()
        assert err <= 2e-2 and err / b.abs().max().item() <= 1e-2, err


def test_prep_append_leaves_outputs_and_slabs_bit_identical():
    """With fused_qkv_prep the preparation writes the append heads whose new segment is clear of
    the scale's live segments into the slab before the attention (scheduler.prep_append_split).
    Against the same model with every append left to the pack after the attention (the
    reference's order, :2218-2225), every output and every slab segment live at the next scale is
    bit-identical, and the slot counters add up: early + packed = the reference's append slots."""
    dev = torch.device("cuda", 0)
    L, H, C = 3, 16, 2048
    schedule = synthetic.SCALE_SCHEDULE_1M
    n_tok = sum(a * b * c for a, b, c in schedule)
    g = torch.Generator().manual_seed(3)
    angles = torch.rand(1, 1, 1, n_tok, 64, generator=g) * 6.0
    freqs = {str(tuple(schedule)): torch.stack([torch.cos(angles), torch.sin(angles)]).to(dev)}
    orders = synthetic.random_removal_orders(L, H, seed=11)
    xs = [[torch.randn(2, h * w, C, device=dev) for _, h, w in schedule] for _ in range(L)]
    runs = []
    for early in (True, False):
        torch.manual_seed(0)
        model = nn.ModuleList([SelfAttention(C, H, True) for _ in range(L)]).to(dev)
        enable_real_pruning_scale_specific_fused_segmented(
            model, 0.10, orders, protected_prefix_scales=3, source_scale_start=3,
            fused_qkv_prep=True)
        for m in model:
            m.kv_caching(True)
        set_real_pruning_fast_phase_profile_enabled(True)
        snapshot_real_pruning_fast_phase_profile(reset=True)
        outs, slabs = [], []
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            for t in range(len(schedule)):
                for l, m in enumerate(model):
                    if not early:
                        m._heatkv_layer.prep_append.clear()
                    outs.append(m(xs[l][t], None, scale_schedule=schedule,
                                  rope2d_freqs_grid=freqs, scale_ind=t))
                    if getattr(m, "_real_pruning_segmented_cache_active", False):
                        for seg in m._heatkv_layer.schedule["segments_by_target"][t + 1]:
                            lo, hi = seg["offset"], seg["offset"] + seg["length"]
                            slabs.append((l, t, seg["source_scale"], seg["head"],
                                          m._heatkv_slab_k[:, lo:hi].clone(),
                                          m._heatkv_slab_v[:, lo:hi].clone()))
        stats = snapshot_real_pruning_fast_phase_profile(reset=True)["segmented_flat_stats"]
        set_real_pruning_fast_phase_profile_enabled(False)
        runs.append((outs, slabs, stats))
    assert _native.device_status(dev) == 0
    (oa, sa, ca), (ob, sb, cb) = runs
    assert ca.get("prep_append_slots", 0) > 0 and cb.get("prep_append_slots", 0) == 0
    assert ca["prep_append_slots"] + ca.get("append_copy_slots", 0) == cb["append_copy_slots"]
    assert len(oa) == len(ob) and all(torch.equal(a, b) for a, b in zip(oa, ob))
    assert len(sa) == len(sb) > 0
    for a, b in zip(sa, sb):
        assert a[:4] == b[:4]
        assert torch.equal(a[4], b[4]) and torch.equal(a[5], b[5]), a[:4]


@pytest.mark.parametrize("dtype,autocast", [(torch.bfloat16, False), (torch.float32, True)])
def test_planned_schedule_is_bit_identical(dtype, autocast):
    """The installer's per-(layer, target) launch plans (longest-first item maps of the
    column-split kernel, from the static segment tables) change only which CTA runs which query
    block: every output at every scale is bit-identical to the round-robin launch."""
    from heatkv_b200.enable_real_pruning_fast import _LayerState
    dev = torch.device("cuda", 0)
    L, H, C = 2, 16, 2048
    schedule = synthetic.SCALE_SCHEDULE_1M
    orders = synthetic.random_removal_orders(L, H, seed=5)
    xs = [[torch.randn(2, h * w, C, device=dev, dtype=dtype) for _, h, w in schedule]
          for _ in range(L)]
    runs = []
    original = _LayerState.attention_plan
    for planned in (True, False):
        if not planned:
            _LayerState.attention_plan = lambda self, *a, **k: None
        try:
            torch.manual_seed(0)
            model = nn.ModuleList([SelfAttention(C, H, True) for _ in range(L)]).to(dev, dtype)
            enable_real_pruning_scale_specific_fused_segmented(
                model, 0.10, orders, protected_prefix_scales=3, source_scale_start=3)
            for m in model:
                m.kv_caching(True)
            outs = []
            with torch.no_grad(), _autocast(autocast):
                for t in range(len(schedule)):
                    for l, m in enumerate(model):
                        outs.append(m(xs[l][t], None, scale_ind=t))
            runs.append(outs)
        finally:
            _LayerState.attention_plan = original
    assert _native.device_status(dev) == 0
    assert all(torch.equal(a, b) for a, b in zip(*runs))


@pytest.mark.parametrize("dtype,autocast,fused", [(torch.bfloat16, False, False),
                                                  (torch.float32, True, False),
                                                  (torch.float32, True, True)])
def test_dense_prefix_kernel_route_matches_sdpa_route(dtype, autocast, fused):
    """The dense-prefix scales through the segmented kernel (default) against the reference's SDPA
    route: outputs of the dense scales agree within the bf16 tolerance. Without the fused
    preparation both routes compute and cache the same K/V, so every slab segment after the
    activation and every output of the pruned scales is bit-identical; with it (the SDPA route's
    dense scales run the module's own forward, whose q/k normalisation rounds differently)
    those agree within the tolerance too."""
    dev = torch.device("cuda", 0)
    L, H, C = 2, 16, 2048
    schedule = synthetic.SCALE_SCHEDULE_1M
    n_tok = sum(a * b * c for a, b, c in schedule)
    g = torch.Generator().manual_seed(4)
    angles = torch.rand(1, 1, 1, n_tok, 64, generator=g) * 6.0
    freqs = {str(tuple(schedule)): torch.stack([torch.cos(angles), torch.sin(angles)]).to(dev)}
    if not autocast:
        freqs = None   # the fp32 rope cache would promote q/k of a bf16 model to fp32
    orders = synthetic.random_removal_orders(L, H, seed=21)
    xs = [[torch.randn(2, h * w, C, device=dev, dtype=dtype) for _, h, w in schedule]
          for _ in range(L)]
    runs = []
    for route in ("kernel", "sdpa"):
        torch.manual_seed(0)
        model = nn.ModuleList([SelfAttention(C, H, True) for _ in range(L)]).to(dev, dtype)
        enable_real_pruning_scale_specific_fused_segmented(
            model, 0.10, orders, protected_prefix_scales=3, source_scale_start=3,
            fused_qkv_prep=fused, dense_prefix=route)
        for m in model:
            m.kv_caching(True)
        outs, slabs = [], []
        with torch.no_grad(), _autocast(autocast):
            for t in range(len(schedule)):
                for l, m in enumerate(model):
                    dense = not m._real_pruning_segmented_cache_active
                    outs.append((l, t, dense, m(xs[l][t], None, scale_schedule=schedule,
                                                rope2d_freqs_grid=freqs, scale_ind=t)))
                    if m._real_pruning_segmented_cache_active and t + 1 < len(schedule):
                        for seg in m._heatkv_layer.schedule["segments_by_target"][t + 1]:
                            lo, hi = seg["offset"], seg["offset"] + seg["length"]
                            slabs.append((l, t, m._heatkv_slab_k[:, lo:hi].clone(),
                                          m._heatkv_slab_v[:, lo:hi].clone()))
        runs.append((outs, slabs))
    assert _native.device_status(dev) == 0
    (oa, sa), (ob, sb) = runs
    assert any(d for _, _, d, _ in oa) and not all(d for _, _, d, _ in oa)
    def close(a, b):
        err = (a.float() - b.float()).abs().max().item()
        return err <= 2e-2 and err <= 1e-2 * max(b.float().abs().max().item(), 1e-6)

    for (l, t, dense, a), (_, _, dense_b, b) in zip(oa, ob):
        assert dense == dense_b
        if dense or fused:
            assert close(a, b), (l, t)
        else:
            assert torch.equal(a, b), (l, t)
    assert len(sa) == len(sb) > 0
    for a, b in zip(sa, sb):
        if fused:
            assert close(a[2], b[2]) and close(a[3], b[3]), a[:2]
        else:
            assert torch.equal(a[2], b[2]) and torch.equal(a[3], b[3]), a[:2]
