"""Drop-in for the reference's ``real_pruning_fused_attention.py`` on B200.

Same entry points, keyword-only signatures, validation order, exception types and messages as
the reference (real_pruning_fused_attention.py:365-591):

* ``pack_flat_segments_kv`` - copy K/V token runs into the flat slab, in place.
* ``fused_real_pruning_flat_segmented_attention`` - attention of the current scale over the head's
  slab segments plus the current K/V, output ``[B, Lq, H*D]`` in q's dtype.

Both call libheatkv.so (hand-written sm_100a CUDA, include/heatkv.h) on the current CUDA stream
with no host synchronisation. There is no Triton and no CPU fallback: CPU tensors raise
``RuntimeError`` even with ``allow_cpu_fallback=True``, and a missing library raises
``RuntimeError``.

Environment knobs of the reference: ``REAL_PRUNING_FUSED_QK_DOT_MODE`` /
``REAL_PRUNING_FUSED_VALUE_DOT_MODE`` are validated the same way. The default ``bf16`` modes (and
``tf32`` for QK) select a tcgen05 tensor-core kernel with the reference's precision: all-bf16 or
all-fp16 inputs, or fp32 q/k with bf16/fp16 v (the real model's cos-attention dtypes), where the
scores are tf32 products as ``tl.dot`` makes them on fp32 operands and P is rounded to v's dtype;
``fp32``/``ieee`` in either knob, and every other dtype combination, select the exact CUDA-core
kernel (fp32 products). ``REAL_PRUNING_FUSED_BLOCK_M/_N/_NUM_WARPS/_NUM_STAGES`` tune the Triton
kernel and have no meaning here. ``HEATKV_ATTENTION_KERNEL`` = ``auto|exact|tcgen05`` (or a named
tcgen05 variant: ``tcgen05_cs``, ``tcgen05_cs64``) forces a kernel.
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from . import _native

__all__ = ["fused_real_pruning_flat_segmented_attention", "pack_flat_segments_kv"]


def _fused_value_dot_mode_id() -> int:
    mode = os.environ.get("REAL_PRUNING_FUSED_VALUE_DOT_MODE", "bf16").strip().lower()
    if mode in {"bf16", "flash"}:
        return 0
    if mode in {"fp32", "ieee", "mixed", "fp32_probs"}:
        return 2
    raise ValueError("REAL_PRUNING_FUSED_VALUE_DOT_MODE must be one of: bf16, fp32")


def _fused_qk_dot_mode_id() -> int:
    mode = os.environ.get("REAL_PRUNING_FUSED_QK_DOT_MODE", "bf16").strip().lower()
    if mode in {"bf16", "tensorcore"}:
        return 0
    if mode in {"tf32", "fp32_tf32"}:
        return 1
    if mode in {"fp32", "ieee"}:
        return 2
    raise ValueError("REAL_PRUNING_FUSED_QK_DOT_MODE must be one of: bf16, tf32, fp32")


_KERNEL_NAMES = {"auto": _native.ATTN_AUTO, "exact": _native.ATTN_EXACT,
                 "tcgen05": _native.ATTN_TCGEN05,
                 "tcgen05_cs": _native.ATTN_TCGEN05_CS, "tcgen05_cs64": _native.ATTN_TCGEN05_CS64}


def _kernel_selector() -> int:
    forced = os.environ.get("HEATKV_ATTENTION_KERNEL")
    if forced:
        try:
            return _KERNEL_NAMES[forced.strip().lower()]
        except KeyError:
            raise ValueError("HEATKV_ATTENTION_KERNEL must be one of: auto, exact, tcgen05, "
                             "tcgen05_cs, tcgen05_cs64") from None
    if _fused_qk_dot_mode_id() == 2 or _fused_value_dot_mode_id() == 2:
        return _native.ATTN_EXACT
    return _native.ATTN_AUTO


def pack_flat_segments_kv(
    *,
    dst_k: torch.Tensor,
    dst_v: torch.Tensor,
    src_k: torch.Tensor,
    src_v: torch.Tensor,
    dst_starts: torch.Tensor,
    src_starts: torch.Tensor,
    lengths: torch.Tensor,
    max_length: Optional[int] = None,
    block_t: int = 32,
):
    """Copy matching flat K/V segments: ``dst[b, dst_starts[i]+t] = src[b, src_starts[i]+t]``.

    ``src_*`` are ``[B, S_src, D]`` (the flat view of ``[B, H, S, D]``), ``dst_*`` are the slab
    ``[B, capacity, D]``; the descriptors are int64 device tensors. ``block_t`` is accepted for
    signature compatibility (it sized the Triton grid)."""
    del block_t
    for name, tensor in (("dst_k", dst_k), ("dst_v", dst_v), ("src_k", src_k), ("src_v", src_v)):
        if tensor.ndim != 3:
            raise ValueError(f"pack_flat_segments_kv expects {name} shaped [B, S, D]")
    if dst_k.shape != dst_v.shape:
        raise ValueError("pack_flat_segments_kv requires matching K/V destination shapes")
    if src_k.shape != src_v.shape:
        raise ValueError("pack_flat_segments_kv requires matching K/V source shapes")
    if dst_k.shape[0] != src_k.shape[0] or dst_k.shape[2] != src_k.shape[2]:
        raise ValueError("pack_flat_segments_kv requires matching batch and head_dim")
    if not (dst_k.is_cuda and dst_v.is_cuda and src_k.is_cuda and src_v.is_cuda):
        raise RuntimeError("pack_flat_segments_kv requires CUDA tensors")
    lib = _native.load()
    if dst_starts.numel() == 0:
        return dst_k, dst_v
    dev = dst_k.device
    if dst_starts.device != dev or src_starts.device != dev or lengths.device != dev:
        raise ValueError("pack segment metadata tensors must be on the destination device")
    n = dst_starts.numel()
    if src_starts.numel() != n or lengths.numel() != n:
        raise ValueError("pack segment metadata tensors must have matching lengths")
    if not dst_k.is_contiguous() or not dst_v.is_contiguous():
        raise ValueError("pack_flat_segments_kv requires contiguous destination tensors")
    # the Triton kernel stored through the destination's element type; the byte copy needs equal
    # element types, so a mismatched source is converted first (rare; the hot path never does it)
    if src_k.dtype != dst_k.dtype:
        src_k = src_k.to(dst_k.dtype)
    if src_v.dtype != dst_v.dtype:
        src_v = src_v.to(dst_v.dtype)
    if not src_k.is_contiguous():
        src_k = src_k.contiguous()
    if not src_v.is_contiguous():
        src_v = src_v.contiguous()
    head_dim = int(dst_k.shape[2])
    if head_dim > 128:
        raise RuntimeError("pack_flat_segments_kv currently supports head_dim <= 128")
    if dst_k.dtype not in _native.DTYPE_CODES or dst_v.dtype not in _native.DTYPE_CODES:
        raise RuntimeError("pack_flat_segments_kv supports float32, float16 and bfloat16 tensors")
    if dst_starts.dtype != torch.int64:
        dst_starts = dst_starts.to(torch.int64)
    if src_starts.dtype != torch.int64:
        src_starts = src_starts.to(torch.int64)
    if lengths.dtype != torch.int64:
        lengths = lengths.to(torch.int64)
    max_len = int(max_length) if max_length is not None else int(lengths.max().item())
    if max_len <= 0:
        return dst_k, dst_v
    status = lib.heatkv_pack_kv(
        _native.ptr(dst_k), _native.ptr(dst_v), _native.ptr(src_k), _native.ptr(src_v),
        _native.DTYPE_CODES[dst_k.dtype], _native.DTYPE_CODES[dst_v.dtype],
        int(dst_k.shape[0]), int(src_k.shape[1]), int(dst_k.shape[1]), head_dim,
        _native.ptr(dst_starts.contiguous()), _native.ptr(src_starts.contiguous()),
        _native.ptr(lengths.contiguous()), int(n), max_len, _native.stream_handle(dev))
    _native.check(status, "pack_flat_segments_kv")
    return dst_k, dst_v


_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32)
_WORKSPACES: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device scratch of the split-KV scheduler, zero-filled when (re)allocated; every call
    leaves it zeroed again, so it is reused across calls on the device's streams in order."""
    ws = _WORKSPACES.get(device)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WORKSPACES[device] = ws
    return ws


def fused_real_pruning_flat_segmented_attention(
    *,
    q: torch.Tensor,
    persisted_k: Optional[torch.Tensor],
    persisted_v: Optional[torch.Tensor],
    segment_starts: torch.Tensor,
    segment_ends: torch.Tensor,
    segment_counts: torch.Tensor,
    current_k: torch.Tensor,
    current_v: torch.Tensor,
    softmax_scale: float,
    allow_cpu_fallback: bool = False,
    softmax_mode: str = "exp",
    _schedule: Optional[tuple] = None,
) -> torch.Tensor:
    """Attention over a flat K/V segment slab without compacting old K/V.

    ``persisted_k/v`` are ``[B, capacity_slots, D]`` (or None for an empty slab). Segment
    starts/ends are flat slot offsets into that slab, ``[H, S]`` per head, with ``[H]`` counts;
    entries with ``start >= end`` are skipped. Returns ``[B, Lq, H*D]`` in q's dtype.

    ``_schedule`` (not in the reference; used by the installer, which knows the static segment
    tables): ``(head_order, item_map, grid)`` device tensors of a column-split launch planned by
    ``hotpath.plan_column_split`` - the same result, with the heads' query blocks assigned to
    the CTAs longest first instead of in a fixed round robin."""
    if q.ndim != 4 or current_k.ndim != 4 or current_v.ndim != 4:
        raise ValueError("q, current_k, and current_v must have shape [B, H, L, D]")
    if q.shape != current_k.shape or q.shape != current_v.shape:
        raise ValueError("q, current_k, and current_v must have identical [B, H, L, D] shapes")
    if q.device != current_k.device or q.device != current_v.device:
        raise ValueError("q, current_k, and current_v must be on the same device")
    empty_slab = persisted_k is None or persisted_v is None
    if empty_slab:
        persisted_k = current_k.new_empty((current_k.shape[0], 0, current_k.shape[3]))
        persisted_v = current_v.new_empty((current_v.shape[0], 0, current_v.shape[3]))
    if persisted_k.ndim != 3 or persisted_v.ndim != 3:
        raise ValueError("persisted_k and persisted_v must have shape [B, S, D]")
    if persisted_k.shape != persisted_v.shape:
        raise ValueError("persisted_k and persisted_v must have identical shapes")
    if persisted_k.shape[0] != q.shape[0]:
        raise ValueError("persisted K/V batch dimension must match q")
    if persisted_k.shape[2] != q.shape[3]:
        raise ValueError("persisted K/V head_dim must match q")
    if persisted_k.device != q.device or persisted_v.device != q.device:
        raise ValueError("persisted K/V must be on the same device as q")
    if persisted_k.dtype != current_k.dtype:
        raise ValueError("persisted_k dtype must match current_k")
    if persisted_v.dtype != current_v.dtype:
        raise ValueError("persisted_v dtype must match current_v")
    batch_size, num_heads, current_len, head_dim = q.shape
    if segment_starts.shape != segment_ends.shape:
        raise ValueError("segment_starts and segment_ends must have identical shapes")
    if segment_starts.ndim != 2 or segment_starts.shape[0] != num_heads:
        raise ValueError("segment_starts must have shape [H, S]")
    if tuple(segment_counts.shape) != (num_heads,):
        raise ValueError("segment_counts must have shape [H]")
    if (segment_starts.device != q.device or segment_ends.device != q.device
            or segment_counts.device != q.device):
        raise ValueError("segment metadata must be on the same device as q")
    if softmax_mode not in {"exp", "exp2"}:
        raise ValueError(f"unsupported softmax_mode {softmax_mode!r}")
    if q.device.type != "cuda":
        if allow_cpu_fallback:
            raise RuntimeError("real_scale_fused_segmented requires CUDA tensors "
                               "(this implementation has no CPU fallback)")
        raise RuntimeError("real_scale_fused_segmented requires CUDA tensors")
    lib = _native.load()
    if head_dim != 128:
        raise RuntimeError("real_scale_fused_segmented v1 only supports head_dim=128")
    if current_len <= 0:
        raise RuntimeError("real_scale_fused_segmented requires current_len > 0")
    if q.dtype not in _SUPPORTED:
        raise RuntimeError(
            "real_scale_fused_segmented supports only float16, bfloat16, or float32 q tensors")
    if current_k.dtype not in _SUPPORTED:
        raise RuntimeError(
            "real_scale_fused_segmented supports only float16, bfloat16, or float32 k tensors")
    if current_v.dtype not in _SUPPORTED:
        raise RuntimeError(
            "real_scale_fused_segmented supports only float16, bfloat16, or float32 v tensors")
    kernel = _kernel_selector()

    q = q.contiguous()
    persisted_k = persisted_k.contiguous()
    persisted_v = persisted_v.contiguous()
    if segment_starts.dtype != torch.int32:
        segment_starts = segment_starts.to(torch.int32)
    if segment_ends.dtype != torch.int32:
        segment_ends = segment_ends.to(torch.int32)
    if segment_counts.dtype != torch.int32:
        segment_counts = segment_counts.to(torch.int32)
    segment_starts = segment_starts.contiguous()
    segment_ends = segment_ends.contiguous()
    segment_counts = segment_counts.contiguous()
    current_k = current_k.contiguous()
    current_v = current_v.contiguous()
    capacity = int(persisted_k.shape[1])
    if _schedule is not None:
        return _scheduled_attention(q, persisted_k, persisted_v, segment_starts, segment_ends,
                                    segment_counts, current_k, current_v, softmax_scale,
                                    _schedule, kernel)
    output = q.new_empty((batch_size, current_len, num_heads * head_dim))
    splits = int(os.environ.get("HEATKV_KV_SPLITS", "1"))
    need = int(lib.heatkv_attention_workspace_bytes(batch_size, num_heads, current_len, splits))
    ws = _workspace(q.device, need) if need > 0 else None
    status = lib.heatkv_segmented_attention_ws(
        _native.ptr(q), _native.ptr(persisted_k) if capacity else None,
        _native.ptr(persisted_v) if capacity else None, _native.ptr(segment_starts),
        _native.ptr(segment_ends), _native.ptr(segment_counts), _native.ptr(current_k),
        _native.ptr(current_v), _native.ptr(output), _native.DTYPE_CODES[q.dtype],
        _native.DTYPE_CODES[current_k.dtype], _native.DTYPE_CODES[current_v.dtype],
        int(batch_size), int(num_heads), int(current_len), capacity, int(head_dim),
        int(segment_starts.shape[1]), float(softmax_scale), int(softmax_mode == "exp2"), kernel,
        None, splits, _native.ptr(ws), 0 if ws is None else ws.numel(),
        _native.stream_handle(q.device))
    _native.check(status, "fused_real_pruning_flat_segmented_attention")
    return output


def _scheduled_attention(q, persisted_k, persisted_v, segment_starts, segment_ends, segment_counts,
                         current_k, current_v, softmax_scale, schedule, kernel=None):
    """The launch of ``fused_real_pruning_flat_segmented_attention(..., _schedule=schedule)``
    without the Python-side validation: for the installer's forward, whose tensors are its own
    (contiguous CUDA tensors, int32 segment tables, ``[B, capacity, 128]`` slabs). The library
    still checks sizes, dtypes and head_dim with the reference's messages. ``kernel``: the
    selector, read from the environment knobs when None."""
    if kernel is None:
        kernel = _kernel_selector()
    lib = _native.load()
    batch_size, num_heads, current_len, head_dim = q.shape
    capacity = int(persisted_k.shape[1])
    order, item_map, grid = schedule
    output = q.new_empty((batch_size, current_len, num_heads * head_dim))
    status = lib.heatkv_segmented_attention_mapped(
        q.data_ptr(), persisted_k.data_ptr() if capacity else None,
        persisted_v.data_ptr() if capacity else None, segment_starts.data_ptr(),
        segment_ends.data_ptr(), segment_counts.data_ptr(), current_k.data_ptr(),
        current_v.data_ptr(), output.data_ptr(), _native.DTYPE_CODES[q.dtype],
        _native.DTYPE_CODES[current_k.dtype], _native.DTYPE_CODES[current_v.dtype],
        batch_size, num_heads, current_len, capacity, head_dim, int(segment_starts.shape[1]),
        float(softmax_scale), kernel, order.data_ptr(), 1, 0, item_map.data_ptr(),
        item_map.numel(), int(grid), None, 0, _native.stream_handle(q.device))
    _native.check(status, "fused_real_pruning_flat_segmented_attention")
    return output
