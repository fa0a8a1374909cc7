"""Segmented flat-slab attention on the CPU (test oracle).

Restates ``_flat_segmented_attention_reference`` (real_pruning_fused_attention.py:312-361):
for every batch row ``b`` and head ``h`` the keys/values are the concatenation of the slab rows
``persisted[b, start:end]`` of the head's first ``counts[h]`` segments, skipping entries with
``start >= end`` (:341-348), followed by the head's current-scale K/V (:349-350); the output is
``softmax(q k^T * scale) v`` laid out as ``[B, Lq, H*D]`` (:353-361). There is no mask inside the
current scale (block-causal attention sees the whole current scale).
"""

from __future__ import annotations

import numpy as np


def _as_numpy(x):
    if x is None:
        return None
    try:  # torch tensors (any dtype) -> float32 numpy, without importing torch here
        import torch

        if isinstance(x, torch.Tensor):
            if x.dtype in (torch.bfloat16, torch.float16):
                x = x.float()
            return x.detach().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x)


def head_keys(persisted, starts, ends, counts, b: int, h: int, capacity: int):
    """Slab rows attended by (b, h), in segment order; ``(start, end)`` is clipped to the slab
    like Python slicing does in the reference oracle (:347)."""
    parts = []
    for i in range(int(counts[h])):
        s, e = int(starts[h, i]), int(ends[h, i])
        if s >= e:
            continue
        s, e = max(0, s), min(capacity, e)
        if s < e:
            parts.append(persisted[b, s:e, :])
    return parts


def segmented_attention(*, q, persisted_k, persisted_v, segment_starts, segment_ends,
                        segment_counts, current_k, current_v, softmax_scale,
                        compute_dtype=np.float64):
    """Return ``[B, Lq, H*D]`` in ``compute_dtype``."""
    q = _as_numpy(q).astype(compute_dtype, copy=False)
    ck = _as_numpy(current_k).astype(compute_dtype, copy=False)
    cv = _as_numpy(current_v).astype(compute_dtype, copy=False)
    B, H, L, D = q.shape
    if persisted_k is None or persisted_v is None:
        pk = np.zeros((B, 0, D), dtype=compute_dtype)
        pv = np.zeros((B, 0, D), dtype=compute_dtype)
    else:
        pk = _as_numpy(persisted_k).astype(compute_dtype, copy=False)
        pv = _as_numpy(persisted_v).astype(compute_dtype, copy=False)
    starts = _as_numpy(segment_starts).astype(np.int64)
    ends = _as_numpy(segment_ends).astype(np.int64)
    counts = _as_numpy(segment_counts).astype(np.int64)
    capacity = pk.shape[1]
    out = np.empty((B, L, H, D), dtype=compute_dtype)
    scale = compute_dtype(softmax_scale) if isinstance(compute_dtype, type) else softmax_scale
    for b in range(B):
        for h in range(H):
            kparts = head_keys(pk, starts, ends, counts, b, h, capacity) + [ck[b, h]]
            vparts = head_keys(pv, starts, ends, counts, b, h, capacity) + [cv[b, h]]
            keys = np.concatenate(kparts, axis=0)
            vals = np.concatenate(vparts, axis=0)
            s = (q[b, h] @ keys.T) * scale
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(axis=1, keepdims=True)
            out[b, :, h, :] = p @ vals
    return out.reshape(B, L, H * D)


def attention_flops(*, batch: int, q_len: int, head_dim: int, segment_starts, segment_ends,
                    segment_counts, capacity: int) -> int:
    """Algorithmic FLOPs of one call: sum over (b, h) of 4 * Lq * (S_h + Lq) * D, with S_h the
    head's attended slab slots (QK^T and PV; softmax not counted)."""
    starts = _as_numpy(segment_starts).astype(np.int64)
    ends = _as_numpy(segment_ends).astype(np.int64)
    counts = _as_numpy(segment_counts).astype(np.int64)
    total = 0
    for h in range(counts.shape[0]):
        slots = 0
        for i in range(int(counts[h])):
            s, e = max(0, int(starts[h, i])), min(capacity, int(ends[h, i]))
            slots += max(0, e - s)
        total += 4 * q_len * (slots + q_len) * head_dim
    return int(total * batch)
