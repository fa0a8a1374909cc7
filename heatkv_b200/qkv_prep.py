"""One-pass q/k/v preparation between the QKV projection and the segmented attention.

The reference's patched attention forward (enable_real_pruning_fast.py:2040-2072) turns the
projection output ``qkv`` ``[B, L, 3, H, D]`` into contiguous ``q, k, v`` ``[B, H, L, D]`` with a
chain of PyTorch ops: ``unbind`` + ``permute`` + ``contiguous``; with cos-attention
``q = F.normalize(q) * scale_mul`` and ``k = F.normalize(k)``; then ``apply_rotary_emb``
(infinity/models/basic.py:97-117), which computes in fp32 with autocast off.
``prepare_qkv`` does the same in one HBM pass (``heatkv_qkv_prepare``, csrc/qkv_prep.cu). With
``append=`` the same pass also writes the scale's K/V rows of the given heads into the layer's slab
(``heatkv_qkv_prepare_append``), the part of the reference's post-attention append
(enable_real_pruning_fast.py:2218-2225) that ``scheduler.prep_append_split`` shows may run first.

Result dtypes follow the PyTorch chain: q and k are fp32 when the rotary embedding is applied
(its fp32 cache promotes them) or when cos-attention normalises under autocast, else the input
dtype; v keeps the input dtype.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _native

__all__ = ["prepare_qkv", "prepared_dtypes", "rope_rows"]


def prepared_dtypes(qkv_dtype: torch.dtype, *, cos_attention: bool, rope: bool):
    """(q/k dtype, v dtype) that ``prepare_qkv`` returns by default, as the PyTorch chain gives
    them: fp32 q/k when the rotary embedding runs or cos-attention normalises under autocast."""
    fp32 = rope or (cos_attention and torch.is_autocast_enabled())
    return (torch.float32 if fp32 else qkv_dtype), qkv_dtype


def rope_rows(rope2d_freqs_grid, scale_schedule, scale_ind: int, seq_len: int,
              device) -> Tuple[torch.Tensor, torch.Tensor]:
    """The (cos, sin) rows ``[seq_len, D/2]`` that ``apply_rotary_emb`` slices for a scale
    (infinity/models/basic.py:104-109): the rope cache of the schedule, rows ``start ..
    start + seq_len`` with ``start`` the tokens of the earlier scales."""
    key, starts = schedule_info(scale_schedule)
    grid = rope2d_freqs_grid[key]
    if grid.device != torch.device(device):
        grid = rope2d_freqs_grid[key] = grid.to(device)
    start = starts[scale_ind] if scale_ind >= 1 else 0
    if start + seq_len > grid.shape[4]:
        raise ValueError("rope cache shorter than the scale's tokens")
    rows = grid[:, 0, 0, 0, start:start + seq_len]  # [2, seq_len, half_dim]
    return rows[0], rows[1]


def rope_pair_groups(table: torch.Tensor) -> torch.Tensor:
    """A token-major rope table ``[T, 64]`` (cos or sin of the 64 rotary pairs of each token) in
    the pair-group-major order ``heatkv_qkv_project`` reads, ``[16, T, 4]``: pairs ``4g .. 4g+3``
    of token ``l`` at ``[g, l]``, so the consecutive tokens of a warp's rows are contiguous. The
    scale starting at token ``s`` passes ``table[:, s:]`` (the pointer ``s * 4`` floats in) and
    ``rope_group_stride = 4 * T``."""
    if table.ndim != 2 or table.shape[1] != 64:
        raise ValueError("rope_pair_groups expects a [T, 64] table")
    T = table.shape[0]
    return table.float().reshape(T, 16, 4).permute(1, 0, 2).contiguous()


def prepare_qkv(qkv: torch.Tensor, *, scale_mul: Optional[torch.Tensor] = None,
                eps: float = 1e-12, rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                qk_dtype: Optional[torch.dtype] = None,
                append: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None):
    """``qkv`` ``[B, L, 3, H, 128]`` (bf16/f16) -> ``q, k, v`` ``[B, H, L, 128]``.

    ``scale_mul``: the cos-attention head scales (any shape with H elements, e.g. the
    ``scale_mul_1H11.clamp_max(max).exp()`` tensor), or None for no normalisation. ``rope``:
    ``(cos, sin)`` rows ``[L, 64]`` fp32 (``rope_rows``), or None. ``qk_dtype``: defaults to fp32
    when ``rope`` is given or autocast is enabled with ``scale_mul``, else ``qkv.dtype``.
    ``append``: ``(slab_k, slab_v, offsets)`` - the layer's slab ``[B, capacity, 128]`` (K in the
    q/k dtype, V in ``qkv.dtype``) and an int64 ``[H]`` device tensor of slab offsets (-1 = head
    not written); head h's rows then also land in ``slab[:, offsets[h] + l]``."""
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError("prepare_qkv expects qkv shaped [B, L, 3, H, D]")
    B, L, _, H, D = qkv.shape
    if D != 128:
        raise RuntimeError("prepare_qkv only supports head_dim=128")
    if qkv.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("prepare_qkv expects a bfloat16 or float16 qkv")
    if not qkv.is_cuda:
        raise RuntimeError("prepare_qkv requires CUDA tensors")
    lib = _native.load()
    dev = qkv.device
    qkv = qkv.contiguous()
    if qk_dtype is None:
        qk_dtype = prepared_dtypes(qkv.dtype, cos_attention=scale_mul is not None,
                                   rope=rope is not None)[0]
    q = torch.empty(B, H, L, D, dtype=qk_dtype, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(B, H, L, D, dtype=qkv.dtype, device=dev)
    sm = None
    if scale_mul is not None:
        if scale_mul.numel() != H:
            raise ValueError("scale_mul must have one value per head")
        sm = scale_mul.detach().reshape(H).to(device=dev, dtype=torch.float32).contiguous()
    cos = sin = None
    stride = 0
    if rope is not None:
        cos, sin = rope
        if (cos.shape != (L, D // 2) or sin.shape != (L, D // 2) or cos.dtype != torch.float32
                or sin.dtype != torch.float32 or cos.stride(1) != 1 or sin.stride(1) != 1
                or cos.stride(0) != sin.stride(0)):
            raise ValueError("rope rows must be fp32 [L, 64] with unit inner stride")
        if cos.device != dev or sin.device != dev:
            raise ValueError("rope rows must be on the qkv device")
        stride = int(cos.stride(0))
    args = (_native.ptr(qkv), _native.ptr(q), _native.ptr(k), _native.ptr(v),
            _native.DTYPE_CODES[qkv.dtype], _native.DTYPE_CODES[qk_dtype], B, L, H, D,
            _native.ptr(sm), float(eps), _native.ptr(cos), _native.ptr(sin), stride)
    if append is None:
        _native.check(lib.heatkv_qkv_prepare(*args, _native.stream_handle(dev)), "prepare_qkv")
        return q, k, v
    slab_k, slab_v, offsets = append
    if (slab_k.ndim != 3 or slab_k.shape != slab_v.shape or slab_k.shape[0] != B
            or slab_k.shape[2] != D):
        raise ValueError("append slabs must be [B, capacity, 128] and alike")
    if slab_k.dtype != qk_dtype or slab_v.dtype != qkv.dtype:
        raise ValueError("append slab dtypes must be the prepared k and v dtypes")
    if not (slab_k.is_contiguous() and slab_v.is_contiguous()):
        raise ValueError("append slabs must be contiguous")
    if (offsets.dtype != torch.int64 or offsets.numel() != H or not offsets.is_contiguous()
            or offsets.device != dev or slab_k.device != dev or slab_v.device != dev):
        raise ValueError("append offsets must be a contiguous int64 [H] tensor on the qkv device")
    _native.check(lib.heatkv_qkv_prepare_append(
        *args, _native.ptr(slab_k), _native.ptr(slab_v), int(slab_k.shape[1]),
        _native.ptr(offsets), _native.stream_handle(dev)), "prepare_qkv")
    return q, k, v


_ROPE_GROUPS = {}
_SCHEDULES = {}


def schedule_info(scale_schedule):
    """``(str(tuple(scale_schedule)), first token of every scale)`` - the rope cache's key and the
    scales' offsets - memoised on the schedule's contents (every layer and scale asks)."""
    try:
        snap = tuple(scale_schedule)
        hit = _SCHEDULES.get(snap)
    except TypeError:  # unhashable entries (lists): no memo
        snap, hit = None, None
    if hit is None:
        starts, total = [], 0
        for a, b, c in scale_schedule:
            starts.append(total)
            total += int(a) * int(b) * int(c)
        hit = (str(tuple(scale_schedule)), starts)
        if snap is not None:
            if len(_SCHEDULES) > 16:
                _SCHEDULES.clear()
            _SCHEDULES[snap] = hit
    return hit


def rope_groups(rope2d_freqs_grid, scale_schedule, device):
    """The schedule's whole rope cache (cos, sin) in pair-group-major order ``[16, T, 4]``
    (``rope_pair_groups``), built once per cache tensor and device; a scale starting at token
    ``s`` is read from token offset ``s``."""
    key = schedule_info(scale_schedule)[0]
    grid = rope2d_freqs_grid[key]
    ck = (key, grid.data_ptr(), grid._version, str(device))
    hit = _ROPE_GROUPS.get(ck)
    if hit is None:
        rows = grid.to(device)[:, 0, 0, 0]  # [2, T, 64]
        hit = (rope_pair_groups(rows[0]), rope_pair_groups(rows[1]))
        if len(_ROPE_GROUPS) > 8:
            _ROPE_GROUPS.clear()
        _ROPE_GROUPS[ck] = hit
    return hit


def project_qkv(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], heads: int,
                *, scale_mul: Optional[torch.Tensor] = None, eps: float = 1e-12,
                rope: Optional[Tuple[torch.Tensor, torch.Tensor, int]] = None,
                qk_dtype: Optional[torch.dtype] = None,
                append: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None):
    """``F.linear(x, weight, bias)`` followed by ``prepare_qkv`` in one tensor-core kernel
    (``heatkv_qkv_project``). ``x`` ``[B, L, C]`` and ``weight`` ``[3 * heads * 128, C]`` in one
    16-bit dtype (the casts autocast would make are the caller's); ``bias``: fp32 ``[3 * heads *
    128]`` holding the values F.linear adds (e.g. the bf16 bias widened), or None. ``rope``:
    ``(cos_groups, sin_groups, start)`` - ``rope_groups`` tables and the scale's first token.
    ``qk_dtype`` defaults as in ``prepare_qkv``; ``append`` as in ``prepare_qkv`` (K slab in the q/k
    dtype). Returns ``q, k, v`` ``[B, H, L, 128]``."""
    if x.ndim != 3:
        raise ValueError("project_qkv expects x shaped [B, L, C]")
    B, L, C = x.shape
    H, D = int(heads), 128
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        raise RuntimeError("project_qkv expects x and weight in one 16-bit dtype")
    if tuple(weight.shape) != (3 * H * D, C):
        raise ValueError("project_qkv weight must be [3 * heads * 128, C]")
    if not (x.is_cuda and weight.is_cuda):
        raise RuntimeError("project_qkv requires CUDA tensors")
    lib = _native.load()
    dev = x.device
    x2 = x.reshape(B * L, C).contiguous()
    w = weight.contiguous()
    if qk_dtype is None:
        qk_dtype = prepared_dtypes(x.dtype, cos_attention=scale_mul is not None,
                                   rope=rope is not None)[0]
    q = torch.empty(B, H, L, D, dtype=qk_dtype, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(B, H, L, D, dtype=x.dtype, device=dev)
    b32 = None
    if bias is not None:
        if bias.numel() != 3 * H * D or bias.dtype != torch.float32 or bias.device != dev:
            raise ValueError("project_qkv bias must be fp32 [3 * heads * 128] on x's device")
        b32 = bias.contiguous()
    sm = None
    if scale_mul is not None:
        if scale_mul.numel() != H:
            raise ValueError("scale_mul must have one value per head")
        if (scale_mul.dtype == torch.float32 and scale_mul.device == dev
                and scale_mul.is_contiguous()):
            sm = scale_mul  # read as H contiguous fp32 values, whatever its shape
        else:
            sm = scale_mul.detach().reshape(H).to(device=dev, dtype=torch.float32).contiguous()
    cos = sin = None
    gstride = 0
    if rope is not None:
        cg, sg, start = rope
        if cg.ndim != 3 or cg.shape[0] != 16 or cg.shape[2] != 4 or cg.shape != sg.shape:
            raise ValueError("rope tables must be [16, T, 4] pair groups (rope_groups)")
        if start < 0 or start + L > cg.shape[1]:
            raise ValueError("rope table shorter than the scale's tokens")
        cos = ctypes.c_void_p(cg.data_ptr() + start * 16)
        sin = ctypes.c_void_p(sg.data_ptr() + start * 16)
        gstride = 4 * int(cg.shape[1])
    ck = cv = offs = None
    rows = 0
    if append is not None:
        ck, cv, offs = append
        if (ck.ndim != 3 or ck.shape[0] != B or ck.shape[2] != D or cv.shape != ck.shape
                or ck.dtype != qk_dtype or cv.dtype != x.dtype or not ck.is_contiguous()
                or not cv.is_contiguous()):
            raise ValueError("append caches must be contiguous [B, rows, 128] in the k and v dtypes")
        if offs.dtype != torch.int64 or offs.numel() != H or offs.device != dev:
            raise ValueError("append offsets must be an int64 [H] tensor on x's device")
        rows = int(ck.shape[1])
    _native.check(lib.heatkv_qkv_project(
        _native.ptr(x2), _native.ptr(w), _native.ptr(b32), _native.ptr(q), _native.ptr(k),
        _native.ptr(v), _native.DTYPE_CODES[x.dtype], _native.DTYPE_CODES[qk_dtype], B, L, H, C,
        _native.ptr(sm), ctypes.c_float(eps), cos, sin, gstride, _native.ptr(ck), _native.ptr(cv),
        rows, _native.ptr(offs), _native.stream_handle(dev)), "project_qkv")
    return q, k, v
