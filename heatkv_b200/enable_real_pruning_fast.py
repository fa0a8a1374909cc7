"""Drop-in for the reference's ``enable_real_pruning_fast.py``: HeatKV scale-specific pruning of
an Infinity-style model, with the flat-slab KV cache run on the B200 kernels of libheatkv.

Entry points (same names, arguments and errors as the reference):

* ``enable_real_pruning_scale_specific_fused_segmented(model, budget, orders, *, ...)`` (:2381) and
  ``enable_real_pruning_scale_specific_fast`` (:2279) - install: validate the orders, derive the
  strict budget view (``budget.strict_removed_heads_by_scale_specific_for_budget``), build the
  controller and, per layer, the static slab schedule (``scheduler.build_static_slot_schedule``),
  then patch every self-attention module's ``forward`` and ``kv_caching``.
* the patched ``forward`` (:1951-2254): the scales before a layer's first target with removed
  heads are dense. By default (``dense_prefix="kernel"``) they run through the same segmented
  kernel as the pruned scales, over a dense cache ``[B, H * dense_len, D]`` allocated once per
  layer (one segment per head: the cached tokens, then the current scale) into which each scale's
  K/V are appended; ``dense_prefix="sdpa"`` keeps the reference's route (the module's own forward,
  or SDPA over ``torch.cat`` of the cache and the scale, :2073-2121). The end of the scale before
  the first pruned target packs the retained segments of the dense cache into the slab
  (activation, :2020-2037); every later scale runs the fused segmented attention over the slab
  and appends its own K/V into its slab segments (:2218-2225); the final scale frees the slab
  (:2176-2185).
* ``reset_/set_/snapshot_real_pruning_fast_phase_profile`` (:40-62) - CUDA-event phase timers for
  ``materialize``, ``attention`` and ``compact`` and the slab byte counters (:102-163).

Attention modules are found by type name ``SelfAttention`` (the reference's ``isinstance`` check,
:2294) or passed explicitly with ``attention_modules=``; they must expose ``num_heads``,
``head_dim``, ``mat_qkv``, ``q_bias``, ``v_bias``, ``zero_k_bias``, ``proj``, ``proj_drop``,
``scale``, ``cos_attn`` and ``kv_caching`` like ``infinity.models.basic.SelfAttention``. The 2-D
RoPE function is taken from the module's defining Python module (``apply_rotary_emb``).

Precision note: with cos-attn under bf16 autocast the model produces fp32 q/k and bf16 v; those
mixed calls run the tcgen05 kernel with tf32 scores (the reference's default dot mode on fp32
operands), as do all-bf16/all-fp16 calls; ``REAL_PRUNING_FUSED_QK_DOT_MODE=fp32`` selects the exact
CUDA-core kernel.

``fused_qkv_prep=True`` (installer keyword, not in the reference) replaces the q/k/v preparation
between the QKV projection and the attention (unbind, permute, cos-attention normalisation and
head scale, 2-D RoPE) by one pass of ``heatkv_qkv_prepare`` (``qkv_prep.prepare_qkv``), when the
projection is bf16/fp16, the head dim is 128 and, with cos-attention, autocast is enabled (the
kernel normalises in fp32 as F.normalize does under autocast). Its RoPE is the one of
infinity/models/basic.py:97-117 applied to the module's rope cache rows. On scales whose slab is
already active, the same pass writes the slab append of every head whose new segment shares no
slot with the segments this scale's attention reads (``scheduler.prep_append_split``); the pack
after the attention then copies only the other heads. The slab holds the same bytes afterwards.
"""

from __future__ import annotations

import os
import sys
import time
import types
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F
from torch.nn.functional import scaled_dot_product_attention as slow_attn

from . import budget as _budget
from . import qkv_prep as _qkv_prep
from .enable_pruning import (
    ScaleSpecificPruningController,
    _assign_layer_indices,
    _validate_and_normalize_removed_heads_by_scale_specific,
    _validate_and_normalize_scale_specific_removal_orders,
)
from . import _native
from .hotpath import NUM_SMS, plan_column_split
from .real_pruning_fused_attention import (
    _kernel_selector,
    _scheduled_attention,
    fused_real_pruning_flat_segmented_attention,
    pack_flat_segments_kv,
)
from .scheduler import build_static_slot_schedule, copy_descriptors, prep_append_split

# ------------------------------------------------------------------------------------------------
# phase profiler and slab counters (enable_real_pruning_fast.py:32-163)
# ------------------------------------------------------------------------------------------------
_PHASE_PROFILE_ENABLED = False
_PHASE_CPU_NS: dict = {}
_PHASE_CUDA_MS: dict = {}
_PHASE_CALLS: dict = {}
_SEGMENTED_FLAT_STATS: dict = {}
_PROFILE_PHASES = {"materialize", "attention", "compact"}


def reset_real_pruning_fast_phase_profile() -> None:
    _PHASE_CPU_NS.clear()
    _PHASE_CUDA_MS.clear()
    _PHASE_CALLS.clear()
    _SEGMENTED_FLAT_STATS.clear()


def set_real_pruning_fast_phase_profile_enabled(enabled: bool = True) -> None:
    global _PHASE_PROFILE_ENABLED
    _PHASE_PROFILE_ENABLED = bool(enabled)
    reset_real_pruning_fast_phase_profile()


def snapshot_real_pruning_fast_phase_profile(*, reset: bool = False) -> dict:
    _resolve_phase_events()
    result = {
        "cpu_ms": {k: v / 1e6 for k, v in _PHASE_CPU_NS.items()},
        "cuda_ms": dict(_PHASE_CUDA_MS),
        "calls": dict(_PHASE_CALLS),
        "segmented_flat_stats": dict(_SEGMENTED_FLAT_STATS),
    }
    if reset:
        reset_real_pruning_fast_phase_profile()
    return result


class _Phase:
    """Times one phase with CUDA events; the events are resolved lazily (no synchronisation on
    the hot path, unlike the reference's per-phase ``synchronize``)."""

    _pending: list = []

    def __init__(self, name: str):
        self.name = name
        self.active = _PHASE_PROFILE_ENABLED and name in _PROFILE_PHASES

    def __enter__(self):
        if self.active:
            self.t0 = time.perf_counter_ns()
            self.e0 = torch.cuda.Event(enable_timing=True) if torch.cuda.is_available() else None
            if self.e0 is not None:
                self.e0.record()
        return self

    def __exit__(self, *exc):
        if not self.active:
            return
        _PHASE_CPU_NS[self.name] = _PHASE_CPU_NS.get(self.name, 0) + time.perf_counter_ns() - self.t0
        _PHASE_CALLS[self.name] = _PHASE_CALLS.get(self.name, 0) + 1
        if self.e0 is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            _Phase._pending.append((self.name, self.e0, e1))
            if len(_Phase._pending) > 4096:
                _resolve_phase_events()


def _resolve_phase_events() -> None:
    for name, e0, e1 in _Phase._pending:
        e1.synchronize()
        _PHASE_CUDA_MS[name] = _PHASE_CUDA_MS.get(name, 0.0) + e0.elapsed_time(e1)
    _Phase._pending.clear()


def _stat_add(name: str, value=1) -> None:
    if _PHASE_PROFILE_ENABLED:
        _SEGMENTED_FLAT_STATS[name] = _SEGMENTED_FLAT_STATS.get(name, 0) + value


def _record_kv_copy(prefix: str, slots: int, k: torch.Tensor, v: torch.Tensor) -> None:
    if not _PHASE_PROFILE_ENABLED or slots <= 0:
        return
    _stat_add(f"{prefix}_slots", int(slots))
    _stat_add(f"{prefix}_bytes", int(slots) * int(k.shape[0]) * int(k.shape[-1])
              * (k.element_size() + v.element_size()))


def _fused_softmax_mode() -> str:
    mode = os.environ.get("REAL_PRUNING_FUSED_SOFTMAX_MODE", "exp")
    return mode if mode in {"exp", "exp2"} else "exp"


def _validate_merge_mode(merge_mode: str) -> str:
    if merge_mode != "exact":
        raise ValueError("real pruning fast v1 only supports merge_mode='exact'")
    return merge_mode


# ------------------------------------------------------------------------------------------------
# per-layer device state
# ------------------------------------------------------------------------------------------------


class _LayerState:
    """Static schedule of one layer and its device-resident metadata / copy descriptors."""

    def __init__(self, controller, layer_idx: int, num_heads: int):
        self.schedule = build_static_slot_schedule(controller, layer_idx=layer_idx,
                                                   num_heads=num_heads)
        self.capacity = int(self.schedule["capacity"])
        self.num_heads = int(num_heads)
        ranges = controller.scale_ranges
        num_scales = len(controller.scale_schedule)
        # dense prefix: scales before the layer's first target with removed heads; their K/V
        # live in a preallocated cache [B, H * dense_len, D] (head h at rows h * dense_len + ...)
        # that holds every token before that target (or before the last scale)
        self.first_target = next((t for t in range(1, num_scales)
                                  if controller.any_removed(layer_idx, t)), num_scales)
        self.dense_len = int(ranges[min(self.first_target, num_scales - 1)][0])
        self.device = None
        self.meta = {}
        self.old_pack = {}
        self.append = {}
        self.prep_append = {}
        self.plans = {}
        self.dense_meta = {}

    def dense_segments(self, old_len: int, device):
        """``[H, 1]`` starts/ends and ``[H]`` counts of the dense-prefix attention after
        ``old_len`` cached tokens: head h reads rows ``[h * dense_len, h * dense_len + old_len)``
        of the dense cache (no segment when nothing is cached yet)."""
        key = (int(old_len), device)
        if key not in self.dense_meta:
            H, ld = self.num_heads, max(self.dense_len, 1)
            st = (torch.arange(H, dtype=torch.int32) * ld).reshape(H, 1)
            ct = torch.full((H,), 1 if old_len > 0 else 0, dtype=torch.int32)
            self.dense_meta[key] = (st.to(device), (st + int(old_len)).to(device), ct.to(device))
        return self.dense_meta[key]

    def dense_offsets(self, old_len: int, device):
        """int64 ``[H]`` dense-cache rows where a scale starting after ``old_len`` cached tokens
        begins for each head (``h * dense_len + old_len``), built once per scale."""
        key = ("offs", int(old_len), device)
        if key not in self.dense_meta:
            ld = max(self.dense_len, 1)
            self.dense_meta[key] = (torch.arange(self.num_heads, dtype=torch.int64) * ld
                                    + int(old_len)).to(device)
        return self.dense_meta[key]

    def dense_plan(self, old_len: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """``attention_plan`` of a dense-prefix call over ``old_len`` cached tokens per head."""
        key = ("dense", old_len, q.shape[0], q.shape[2], q.dtype, k.dtype, v.dtype, q.device)
        if key not in self.plans:
            lens = [[int(old_len)] if old_len > 0 else [] for _ in range(self.num_heads)]
            self.plans[key] = self._plan_for(lens, q, k, v)
        return self.plans[key]

    def _plan_for(self, lens, q, k, v):
        dt = _native.DTYPE_CODES
        run = _native.load().heatkv_attention_kernel_for(
            dt[q.dtype], dt[k.dtype], dt[v.dtype], q.shape[0], q.shape[1], q.shape[2],
            _kernel_selector(), 1, 0, 0)
        if run not in (_native.RUN_TCGEN05_CS, _native.RUN_TCGEN05_TF32, _native.RUN_TCGEN05_CS64):
            return None
        cs64 = run == _native.RUN_TCGEN05_CS64
        order, _, _, item_map, grid = plan_column_split(
            lens, q.shape[2], q.shape[0], splits=1, sms=(2 if cs64 else 1) * NUM_SMS,
            key_tile=64 if cs64 else 128)
        return (torch.from_numpy(order).to(q.device), torch.from_numpy(item_map).to(q.device),
                grid)

    def attention_plan(self, target: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """Launch schedule of this layer's fused attention at ``target`` for these tensors, planned
        once per (target, batch, dtypes) from the static segment tables: ``(head_order, item_map,
        grid)`` when the call runs the column-split kernel, else None."""
        key = (target, q.shape[0], q.dtype, k.dtype, v.dtype, q.device)
        if key not in self.plans:
            st, en, ct = self.schedule["metadata_cpu_by_target"][target]
            lens = [[int(en[h, i]) - int(st[h, i]) for i in range(int(ct[h]))]
                    for h in range(self.num_heads)]
            self.plans[key] = self._plan_for(lens, q, k, v)
        return self.plans[key]

    def to(self, device: torch.device) -> None:
        if self.device == device:
            return
        sched = self.schedule
        self.meta = {t: tuple(torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in m)
                     for t, m in sched["metadata_cpu_by_target"].items()}

        def desc(runs):
            d = copy_descriptors(runs)
            if d is None:
                return None
            return (torch.from_numpy(d["dst_starts"]).to(device),
                    torch.from_numpy(d["src_starts"]).to(device),
                    torch.from_numpy(d["lengths"]).to(device), d["max_length"], d["slots"])

        self.old_pack = {t: desc(r) for t, r in sched["old_pack_runs_by_target"].items()}
        self.append = {k: desc(r) for k, r in sched["append_runs_by_key"].items()}
        # per scale: heads the q/k/v preparation may append before the attention, and the rest
        self.prep_append = {}
        for s, _ in sched["append_runs_by_key"]:
            split = prep_append_split(sched, s, self.num_heads)
            if split is None or split["early_slots"] == 0:
                continue
            self.prep_append[s] = (torch.from_numpy(split["offsets"]).to(device),
                                   desc(split["rest_runs"]), split["early_slots"])
        self.device = device


def _pack(desc, dst_k, dst_v, src_k, src_v, prefix: str) -> None:
    """Copy descriptor items from a ``[B, H, S, D]`` source into the slab ``[B, cap, D]``."""
    if desc is None:
        return
    dst, src, ln, max_len, slots = desc
    B, H, S, D = src_k.shape
    pack_flat_segments_kv(dst_k=dst_k, dst_v=dst_v,
                          src_k=src_k.reshape(B, H * S, D), src_v=src_v.reshape(B, H * S, D),
                          dst_starts=dst, src_starts=src, lengths=ln, max_length=max_len)
    _stat_add(f"{prefix}_calls")
    _record_kv_copy(prefix, slots, dst_k, dst_v)


def _items_desc(items, seq_len: int, device):
    """Copy descriptors for ad-hoc ``(dst_offset, head, src_start, length)`` items."""
    items = [it for it in items if it[3] > 0]
    if not items:
        return None
    items.sort()
    dst = torch.tensor([it[0] for it in items], dtype=torch.int64, device=device)
    src = torch.tensor([it[1] * seq_len + it[2] for it in items], dtype=torch.int64, device=device)
    ln = torch.tensor([it[3] for it in items], dtype=torch.int64, device=device)
    return dst, src, ln, max(it[3] for it in items), sum(it[3] for it in items)


def _derived(module, name, params, make):
    """``make()`` computed once per module and reused while ``params`` (tensors it is derived
    from) keep their data pointer and version: inference calls need not rebuild the QKV bias
    (torch.cat of three parameters) or the cos-attention head scale (clamp_max + exp) every
    scale and layer, while an update of a parameter still takes effect. With autograd enabled the
    value is rebuilt every call, so gradients still reach the parameters."""
    if torch.is_grad_enabled():
        return make()
    key = tuple((p.data_ptr(), p._version, p.device, p.dtype) for p in params)
    cache = module.__dict__.setdefault("_heatkv_derived", {})
    hit = cache.get(name)
    if hit is not None and hit[0] == key:
        return hit[1]
    value = make()
    cache[name] = (key, value)
    return value


def _qkv_bias(module) -> torch.Tensor:
    """``cat(q_bias, zero_k_bias, v_bias)`` (enable_real_pruning_fast.py:2043)."""
    ps = (module.q_bias, module.zero_k_bias, module.v_bias)
    return _derived(module, "qkv_bias", ps, lambda: torch.cat(ps))


def _head_scale(module) -> torch.Tensor:
    """The cos-attention head scale ``scale_mul_1H11.clamp_max(max_scale_mul).exp()``
    (:2051-2055) as ``[1, H, 1, 1]``."""
    p = module.scale_mul_1H11
    return _derived(module, "scale_mul", (p,), lambda: p.reshape(
        1, module.num_heads, 1, 1).clamp_max(module.max_scale_mul).exp())


def _fused_project_dtype(module, x):
    """The 16-bit dtype in which ``heatkv_qkv_project`` can stand for this call's QKV linear and
    preparation (None when it cannot): inference (no autograd) on CUDA with the one-pass
    preparation enabled, head_dim 128, an even head count, a width that is a multiple of 64, and
    the linear computed in bf16/f16 - autocast's dtype, or x's own when x and the weight share it."""
    if (not getattr(module, "_heatkv_fused_qkv_prep", False) or not x.is_cuda
            or torch.is_grad_enabled() or module.head_dim != 128 or module.num_heads % 2
            or x.ndim != 3 or x.shape[-1] % 64):
        return None
    w = module.mat_qkv.weight
    if tuple(w.shape) != (3 * module.num_heads * 128, x.shape[-1]):
        return None
    if torch.is_autocast_enabled():
        dt = torch.get_autocast_dtype("cuda")
    else:
        if module.cos_attn:
            return None  # the preparation's fp32 norm reproduces autocast only (as prepare_qkv)
        dt = x.dtype if x.dtype == w.dtype else None
    return dt if dt in (torch.bfloat16, torch.float16) else None


def _project_weights(module, dt):
    """The QKV weight and bias as F.linear uses them in ``dt``: the weight cast to ``dt``, the
    bias ``cat(q_bias, zero_k_bias, v_bias)`` cast to ``dt`` and held in fp32."""
    w = module.mat_qkv.weight
    wd = _derived(module, ("qkv_weight", dt), (w,), lambda: w.detach().to(dt).contiguous())
    ps = (module.q_bias, module.zero_k_bias, module.v_bias)
    bd = _derived(module, ("qkv_bias32", dt), ps,
                  lambda: torch.cat(ps).detach().to(dt).float().contiguous())
    return wd, bd


def _fused_prep_applies(module, qkv) -> bool:
    """The one-pass q/k/v preparation reproduces the PyTorch chain's dtypes here."""
    return (bool(getattr(module, "_heatkv_fused_qkv_prep", False)) and qkv.is_cuda
            and qkv.dtype in (torch.bfloat16, torch.float16) and module.head_dim == 128
            and (not module.cos_attn or torch.is_autocast_enabled()))


def _rope_fn(module):
    mod = sys.modules.get(type(module).__module__)
    fn = getattr(mod, "apply_rotary_emb", None) if mod is not None else None
    if fn is None:
        raise RuntimeError("rope2d_freqs_grid given but apply_rotary_emb was not found beside "
                           f"{type(module).__name__}")
    return fn


def _ensure_slab(self, batch: int, head_dim: int, device, k_dtype, v_dtype) -> None:
    cap = max(int(self._heatkv_layer.capacity), 0)
    shape = (batch, cap, head_dim)
    ck, cv = getattr(self, "_heatkv_slab_k", None), getattr(self, "_heatkv_slab_v", None)
    if (ck is None or tuple(ck.shape) != shape or ck.device != device or ck.dtype != k_dtype
            or cv.dtype != v_dtype):
        self._heatkv_slab_k = torch.empty(shape, device=device, dtype=k_dtype)
        self._heatkv_slab_v = torch.empty(shape, device=device, dtype=v_dtype)
        _stat_add("storage_allocations")
        _stat_add("storage_capacity_slots", cap)
    self._heatkv_layer.to(device)


def _reset_state(self) -> None:
    self._real_pruning_segmented_cache_active = False
    self._real_pruning_logical_len = 0
    self._heatkv_slab_k = None
    self._heatkv_slab_v = None
    self._heatkv_dense_live = False


def _activate_from_dense(self, dense_k, dense_v, target: int) -> None:
    """Pack the retained segments of the dense ``[B, H, T, D]`` cache (T = tokens before
    ``target``) into the slab (enable_real_pruning_fast.py:1639-1671 with the static runs)."""
    B, H, T, D = dense_k.shape
    _ensure_slab(self, B, D, dense_k.device, dense_k.dtype, dense_v.dtype)
    layer = self._heatkv_layer
    if layer.schedule["old_pack_cache_lens_by_target"].get(target) == T:
        desc = layer.old_pack.get(target)
    else:
        items = []
        for seg in layer.schedule["segments_by_target"].get(target, []):
            hi = min(seg["scale_end"], T)
            if seg["scale_start"] < hi:
                items.append((seg["offset"], seg["head"], seg["scale_start"], hi - seg["scale_start"]))
        desc = _items_desc(items, T, dense_k.device)
    _pack(desc, self._heatkv_slab_k, self._heatkv_slab_v, dense_k.contiguous(),
          dense_v.contiguous(), "activation_copy")
    self._real_pruning_segmented_cache_active = True


def _activate_from_dense_and_current(self, dense_k, dense_v, cur_k, cur_v, current_scale: int,
                                     old_len: int, target: int) -> None:
    """Activation that also packs the current scale (enable_real_pruning_fast.py:1673-1789)."""
    B, H, L, D = cur_k.shape
    _ensure_slab(self, B, D, cur_k.device, cur_k.dtype, cur_v.dtype)
    old_items, cur_items = [], []
    for seg in self._heatkv_layer.schedule["segments_by_target"].get(target, []):
        if seg["source_scale"] == current_scale:
            s0 = max(seg["scale_start"], old_len) - old_len
            s1 = min(seg["scale_end"], old_len + L) - old_len
            if s0 < s1:
                cur_items.append((seg["offset"], seg["head"], s0, s1 - s0))
        elif dense_k is not None:
            hi = min(seg["scale_end"], old_len)
            if seg["scale_start"] < hi:
                old_items.append((seg["offset"], seg["head"], seg["scale_start"], hi - seg["scale_start"]))
    if old_items and dense_k is not None:
        _pack(_items_desc(old_items, old_len, cur_k.device), self._heatkv_slab_k,
              self._heatkv_slab_v, dense_k.contiguous(), dense_v.contiguous(), "activation_copy")
    _pack(_items_desc(cur_items, L, cur_k.device), self._heatkv_slab_k, self._heatkv_slab_v,
          cur_k, cur_v, "activation_copy")
    self._real_pruning_segmented_cache_active = True


# ------------------------------------------------------------------------------------------------
# patched forward / kv_caching
# ------------------------------------------------------------------------------------------------


def _dense_prefix_mode(module) -> str:
    """``"kernel"``: scales before a layer's first pruned target run the segmented kernel over a
    preallocated dense cache (one segment per head); ``"sdpa"``: the reference's route (the
    module's own forward, or SDPA over a concatenated cache). Installer keyword ``dense_prefix``;
    ``HEATKV_DENSE_PREFIX`` overrides it."""
    env = os.environ.get("HEATKV_DENSE_PREFIX")
    if env in ("kernel", "sdpa"):
        return env
    return getattr(module, "_heatkv_dense_prefix", "kernel")


def _ensure_dense(self, batch: int, head_dim: int, device, k_dtype, v_dtype):
    """The layer's dense-prefix cache ``[B, H * dense_len, D]`` (kept across images)."""
    ld = max(int(self._heatkv_layer.dense_len), 1)
    shape = (batch, self.num_heads * ld, head_dim)
    dk, dv = getattr(self, "_heatkv_dense_k", None), getattr(self, "_heatkv_dense_v", None)
    if (dk is None or tuple(dk.shape) != shape or dk.device != device or dk.dtype != k_dtype
            or dv.dtype != v_dtype):
        dk = self._heatkv_dense_k = torch.empty(shape, device=device, dtype=k_dtype)
        dv = self._heatkv_dense_v = torch.empty(shape, device=device, dtype=v_dtype)
        _stat_add("dense_cache_allocations")
    return dk, dv


def _dense_append_desc(layer, old_len: int, n: int, device):
    """Copy items of a scale's ``[B, H, n, D]`` K/V into the dense cache after ``old_len`` cached
    tokens: head h's rows to ``h * dense_len + old_len``."""
    ld = max(layer.dense_len, 1)
    return _items_desc([(h * ld + old_len, h, 0, n) for h in range(layer.num_heads)], n, device)


def _segmented_attention(module, q, slab_k, slab_v, meta, k, v, plan):
    """The fused segmented attention of the installer's forward: straight to the planned launch
    when the layer has a plan and q/k/v are contiguous (the slabs and segment tables are the
    installer's own, checked here against q/k/v for what the library cannot see: the batch and
    the slab dtypes), else through the validating public wrapper."""
    if (plan is not None and q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
            and slab_k.dtype == k.dtype and slab_v.dtype == v.dtype
            and slab_k.shape == slab_v.shape and slab_k.shape[0] == q.shape[0]):
        return _scheduled_attention(q, slab_k, slab_v, *meta, k, v, module.scale, plan)
    starts, ends, counts = meta
    return fused_real_pruning_flat_segmented_attention(
        q=q, persisted_k=slab_k, persisted_v=slab_v, segment_starts=starts, segment_ends=ends,
        segment_counts=counts, current_k=k, current_v=v, softmax_scale=module.scale,
        softmax_mode=_fused_softmax_mode(), _schedule=plan)


def _real_pruning_scale_specific_fast_forward(self, x, attn_bias_or_two_vector=None, attn_fn=None,
                                               scale_schedule=None, rope2d_freqs_grid=None,
                                               scale_ind=0):
    if not self.caching:
        raise NotImplementedError("real pruning fused segmented only supports kv-cached inference")
    if attn_bias_or_two_vector is not None:
        raise NotImplementedError("real pruning fused segmented does not support training attention masks")
    if attn_fn is not None:
        raise NotImplementedError("real pruning fused segmented does not support custom attention functions")
    ctrl = self._real_pruning_scale_specific_controller
    layer = self.layer_idx
    state = self._heatkv_layer
    batch_size, seq_len, channels = x.shape
    final_scale = self._num_scales == scale_ind + 1
    old_len = int(getattr(self, "_real_pruning_logical_len", 0))
    logical_len = old_len + seq_len
    active = bool(getattr(self, "_real_pruning_segmented_cache_active", False))
    removed_now = ctrl.any_removed(layer, scale_ind)
    dense_kernel = (_dense_prefix_mode(self) == "kernel" and x.is_cuda and
                    self.head_dim == 128 and not active and not removed_now)

    if (not active and not removed_now and not dense_kernel and _baseline_prefix_enabled()):
        # dense scale: the module's own forward (SDPA over its cat cache)
        output = self._pre_real_prune_scale_specific_fast_forward(
            x, attn_bias_or_two_vector, attn_fn=attn_fn, scale_schedule=scale_schedule,
            rope2d_freqs_grid=rope2d_freqs_grid, scale_ind=scale_ind)
        self._real_pruning_logical_len = logical_len
        if final_scale:
            _reset_state(self)
            self.cached_k = self.cached_v = None
            return output
        if ctrl.any_removed(layer, scale_ind + 1):
            with _Phase("compact"):
                _activate_from_dense(self, self.cached_k, self.cached_v, scale_ind + 1)
            self.cached_k = self.cached_v = None
        return output

    # the QKV linear and the preparation in one tensor-core kernel when it can stand for them
    pdt = _fused_project_dtype(self, x)
    qkv = None
    if pdt is None:
        qkv = F.linear(input=x, weight=self.mat_qkv.weight,
                       bias=_qkv_bias(self)).view(
            batch_size, seq_len, 3, self.num_heads, self.head_dim)
    if rope2d_freqs_grid is not None and scale_schedule is None:
        raise ValueError("scale_schedule is required when rope2d_freqs_grid is provided")
    # the dense cache receives this scale (all heads) unless it is the last one or does not fit
    dense_append = (dense_kernel and not final_scale
                    and logical_len <= max(state.dense_len, 0))
    early_dense = False
    if pdt is not None or _fused_prep_applies(self, qkv):
        in_dtype = pdt if pdt is not None else qkv.dtype
        scale_mul = None
        if self.cos_attn:
            scale_mul = _head_scale(self)
        rope = None
        if rope2d_freqs_grid is not None:
            if pdt is not None:
                cg, sg = _qkv_prep.rope_groups(rope2d_freqs_grid, scale_schedule, x.device)
                rope = (cg, sg, _qkv_prep.schedule_info(scale_schedule)[1][scale_ind])
            else:
                rope = _qkv_prep.rope_rows(rope2d_freqs_grid, scale_schedule, scale_ind,
                                           seq_len, qkv.device)
        dts = _qkv_prep.prepared_dtypes(in_dtype, cos_attention=scale_mul is not None,
                                        rope=rope is not None)
        early, append = None, None
        if active and not final_scale:
            early = self._heatkv_layer.prep_append.get(scale_ind)
            if early is not None and (self._heatkv_slab_k.dtype, self._heatkv_slab_v.dtype) != dts:
                early = None
            if early is not None:
                append = (self._heatkv_slab_k, self._heatkv_slab_v, early[0])
        elif dense_append:
            # the preparation writes the scale straight into the dense cache (rows past the
            # segments this scale's attention reads)
            dk, dv = _ensure_dense(self, batch_size, self.head_dim, x.device, *dts)
            offs = state.dense_offsets(old_len, x.device)
            append = (dk, dv, offs)
            early_dense = True
        if pdt is not None:
            wd, bd = _project_weights(self, pdt)
            q, k, v = _qkv_prep.project_qkv(x.to(pdt), wd, bd, self.num_heads,
                                            scale_mul=scale_mul, rope=rope, qk_dtype=dts[0],
                                            append=append)
            _stat_add("qkv_project_calls")
        else:
            q, k, v = _qkv_prep.prepare_qkv(qkv, scale_mul=scale_mul, rope=rope, append=append)
        if early is not None:
            _stat_add("prep_append_calls")
            _record_kv_copy("prep_append", early[2], self._heatkv_slab_k, self._heatkv_slab_v)
        if early_dense:
            _stat_add("prep_dense_append_calls")
            _record_kv_copy("prep_dense_append", self.num_heads * seq_len, dk, dv)
        del qkv
    else:
        early = None
        q, k, v = qkv.unbind(dim=2)
        q = q.permute(0, 2, 1, 3).contiguous()
        k = k.permute(0, 2, 1, 3).contiguous()
        v = v.permute(0, 2, 1, 3).contiguous()
        del qkv
        if self.cos_attn:
            scale_mul = _head_scale(self)
            q = F.normalize(q, dim=-1, eps=1e-12).mul(scale_mul).contiguous()
            k = F.normalize(k, dim=-1, eps=1e-12).contiguous()
            v = v.contiguous()
        if rope2d_freqs_grid is not None:
            q, k = _rope_fn(self)(q, k, scale_schedule, rope2d_freqs_grid, self.pad_to_multiplier,
                                  self.rope2d_normalized_by_hw, scale_ind)

    dense_candidate = None
    if dense_kernel:
        # dense-prefix scale through the segmented kernel: one segment per head over the cached
        # tokens of the preallocated dense cache, then the current scale (the keys of the
        # reference's SDPA over cat(cache, scale), in the same order)
        with _Phase("materialize"):
            dk, dv = _ensure_dense(self, batch_size, self.head_dim, k.device, k.dtype, v.dtype)
            starts, ends, counts = state.dense_segments(old_len, k.device)
        with _Phase("attention"):
            output = _segmented_attention(self, q, dk, dv, (starts, ends, counts), k, v,
                                          state.dense_plan(old_len, q, k, v))
    elif old_len == 0:
        with _Phase("attention"):
            output = slow_attn(query=q, key=k, value=v, scale=self.scale, dropout_p=0.0).transpose(
                1, 2).reshape(batch_size, seq_len, channels)
    elif not active and not removed_now:
        with _Phase("materialize"):
            attn_k = torch.cat((self.cached_k, k), dim=2)
            attn_v = torch.cat((self.cached_v, v), dim=2)
            dense_candidate = (attn_k, attn_v)
        with _Phase("attention"):
            output = slow_attn(query=q, key=attn_k, value=attn_v, scale=self.scale,
                               dropout_p=0.0).transpose(1, 2).reshape(batch_size, seq_len, channels)
    else:
        with _Phase("materialize"):
            if not active:
                if getattr(self, "_heatkv_dense_live", False):
                    B_, _, D_ = self._heatkv_dense_k.shape
                    ld = max(state.dense_len, 1)
                    _activate_from_dense(
                        self, self._heatkv_dense_k.view(B_, self.num_heads, ld, D_)[:, :, :old_len],
                        self._heatkv_dense_v.view(B_, self.num_heads, ld, D_)[:, :, :old_len],
                        scale_ind)
                    self._heatkv_dense_live = False
                else:
                    _activate_from_dense(self, self.cached_k, self.cached_v, scale_ind)
                self.cached_k = self.cached_v = None
                active = True
            self._heatkv_layer.to(k.device)
            starts, ends, counts = self._heatkv_layer.meta[scale_ind]
        with _Phase("attention"):
            output = _segmented_attention(self, q, self._heatkv_slab_k, self._heatkv_slab_v,
                                          (starts, ends, counts), k, v,
                                          self._heatkv_layer.attention_plan(scale_ind, q, k, v))
    del q
    output = self.proj_drop(self.proj(output))

    with _Phase("compact"):
        if final_scale:
            _reset_state(self)
            self.cached_k = self.cached_v = None
        elif dense_kernel:
            dk, dv = self._heatkv_dense_k, self._heatkv_dense_v
            if dense_append and not early_dense:
                _pack(_dense_append_desc(state, old_len, seq_len, k.device), dk, dv, k, v,
                      "dense_append_copy")
            # plain attributes written straight into the instance dict, as nn.Module's
            # __setattr__ ends up doing for them, without its checks: this runs every call
            self.__dict__["_heatkv_dense_live"] = True
            if ctrl.any_removed(layer, scale_ind + 1):
                # activation: the dense cache holds exactly the tokens before the next scale
                ld = max(state.dense_len, 1)
                B_, _, D_ = dk.shape
                _activate_from_dense(self, dk.view(B_, self.num_heads, ld, D_)[:, :, :logical_len],
                                     dv.view(B_, self.num_heads, ld, D_)[:, :, :logical_len],
                                     scale_ind + 1)
                self.__dict__["_heatkv_dense_live"] = False
            self.__dict__["_real_pruning_logical_len"] = logical_len
        else:
            removed_next = ctrl.any_removed(layer, scale_ind + 1)
            if not active and not removed_next:
                if dense_candidate is not None:
                    self.cached_k, self.cached_v = dense_candidate
                elif self.cached_k is None:
                    self.cached_k, self.cached_v = k, v
                else:
                    self.cached_k = torch.cat((self.cached_k, k), dim=2)
                    self.cached_v = torch.cat((self.cached_v, v), dim=2)
            elif active:
                # heads already appended by the q/k/v preparation leave only the rest here
                desc = (early[1] if early is not None
                        else self._heatkv_layer.append.get((scale_ind, scale_ind + 1)))
                _pack(desc, self._heatkv_slab_k, self._heatkv_slab_v, k, v, "append_copy")
            else:
                _activate_from_dense_and_current(self, self.cached_k, self.cached_v, k, v,
                                                 scale_ind, old_len, scale_ind + 1)
                self.cached_k = self.cached_v = None
            self.__dict__["_real_pruning_logical_len"] = logical_len
    return output


def _baseline_prefix_enabled() -> bool:
    return os.environ.get("REAL_PRUNING_FUSED_SEGMENTED_BASELINE_PREFIX", "1") not in {
        "0", "false", "False", "no", "NO"}


def _real_pruning_scale_specific_fast_kv_caching(self, enable: bool):
    self._pre_real_prune_scale_specific_fast_kv_caching(enable)
    self._real_pruning_scale_specific_controller.reset()
    _reset_state(self)
    if enable:
        try:
            device = next(self.parameters()).device
        except StopIteration:
            device = torch.device("cpu")
        if device.type == "cuda":
            self._heatkv_layer.to(device)


def _attention_modules(model):
    return [m for m in model.modules() if type(m).__name__ == "SelfAttention"]


def enable_real_pruning_scale_specific_fast(model, budget, scale_specific_removal_orders, *,
                                            protected_prefix_scales=4, source_scale_start=None,
                                            skip_last_scale=True, merge_mode="exact",
                                            attention_impl="fused_segmented",
                                            requested_generation_batch_size=None,
                                            attention_modules=None, scale_schedule=None,
                                            fused_qkv_prep=False, dense_prefix="kernel"):
    """Install HeatKV scale-specific pruning (enable_real_pruning_fast.py:2279-2378).
    ``dense_prefix``: ``"kernel"`` (default) runs the scales before each layer's first pruned
    target through the segmented kernel over a preallocated dense cache; ``"sdpa"`` keeps the
    reference's route for them (the module's own forward, or SDPA over a concatenated cache)."""
    merge_mode = _validate_merge_mode(merge_mode)
    if dense_prefix not in ("kernel", "sdpa"):
        raise ValueError("dense_prefix must be 'kernel' or 'sdpa'")
    if attention_impl != "fused_segmented":
        raise ValueError(f"unsupported real pruning fast attention_impl: {attention_impl!r}")
    modules = list(attention_modules) if attention_modules is not None else _attention_modules(model)
    if not modules:
        return model
    _assign_layer_indices(modules)
    num_heads = modules[0].num_heads
    if any(m.num_heads != num_heads for m in modules):
        raise ValueError("real pruning fast requires all SelfAttention modules to use the same num_heads")
    protected_prefix_scales = int(protected_prefix_scales)
    if protected_prefix_scales < 0:
        raise ValueError("protected_prefix_scales must be non-negative")
    if source_scale_start is None:
        source_scale_start = protected_prefix_scales
    source_scale_start = int(source_scale_start)
    schedule = _budget.get_scale_schedule() if scale_schedule is None else list(scale_schedule)
    if len(schedule) <= protected_prefix_scales:
        raise ValueError("scale-specific real pruning fast requires at least one scale after the protected prefix")
    normalized_orders = _validate_and_normalize_scale_specific_removal_orders(
        scale_specific_removal_orders, modules, source_scale_start=source_scale_start)
    view = _budget.strict_removed_heads_by_scale_specific_for_budget(
        budget, normalized_orders, num_layers=len(modules), num_heads=num_heads,
        source_scale_start=source_scale_start, protected_prefix_scales=protected_prefix_scales,
        skip_last_scale=skip_last_scale, scale_schedule=schedule)
    normalized_removed = _validate_and_normalize_removed_heads_by_scale_specific(
        view["removed_heads_by_scale"], modules, source_scale_start=source_scale_start)
    controller = ScaleSpecificPruningController(
        num_layers=len(modules), num_heads=num_heads,
        static_removed_heads_by_scale=normalized_removed, source_scale_start=source_scale_start,
        scale_schedule=schedule)
    for module in modules:
        module._num_scales = len(schedule)
        module._real_pruning_scale_specific_controller = controller
        module._real_prune_scale_specific_budget = float(budget)
        module._real_prune_merge_mode = merge_mode
        module._real_pruning_requested_generation_batch_size = (
            None if requested_generation_batch_size is None else int(requested_generation_batch_size))
        module._heatkv_layer = _LayerState(controller, module.layer_idx, num_heads)
        module._heatkv_fused_qkv_prep = bool(fused_qkv_prep)
        module._heatkv_dense_prefix = dense_prefix
        module._real_pruning_segmented_static_schedule = module._heatkv_layer.schedule
        try:
            device = next(module.parameters()).device
        except StopIteration:
            device = torch.device("cpu")
        if device.type == "cuda":
            module._heatkv_layer.to(device)
        _reset_state(module)
        module._real_pruning_fast_attention_impl = attention_impl
        if not hasattr(module, "_pre_real_prune_scale_specific_fast_forward"):
            module._pre_real_prune_scale_specific_fast_forward = module.forward
        module.forward = types.MethodType(_real_pruning_scale_specific_fast_forward, module)
        if not hasattr(module, "_pre_real_prune_scale_specific_fast_kv_caching"):
            module._pre_real_prune_scale_specific_fast_kv_caching = module.kv_caching
        module.kv_caching = types.MethodType(_real_pruning_scale_specific_fast_kv_caching, module)
    return model


def enable_real_pruning_scale_specific_fused_segmented(model, budget, scale_specific_removal_orders,
                                                       *, protected_prefix_scales=4,
                                                       source_scale_start=None,
                                                       skip_last_scale=True, merge_mode="exact",
                                                       requested_generation_batch_size=None,
                                                       attention_modules=None,
                                                       scale_schedule=None, fused_qkv_prep=False,
                                                       dense_prefix="kernel"):
    """Alias of the installer with ``attention_impl='fused_segmented'`` (:2381-2402)."""
    return enable_real_pruning_scale_specific_fast(
        model, budget, scale_specific_removal_orders,
        protected_prefix_scales=protected_prefix_scales, source_scale_start=source_scale_start,
        skip_last_scale=skip_last_scale, merge_mode=merge_mode, attention_impl="fused_segmented",
        requested_generation_batch_size=requested_generation_batch_size,
        attention_modules=attention_modules, scale_schedule=scale_schedule,
        fused_qkv_prep=fused_qkv_prep, dense_prefix=dense_prefix)
