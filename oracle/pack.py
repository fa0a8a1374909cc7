"""Slab compaction on the CPU (test oracle).

Restates the copy of ``_pack_flat_segments_kv_kernel`` (real_pruning_fused_attention.py:33-73):
for every item ``i`` and batch row ``b``, rows ``src[b, src_starts[i] : src_starts[i]+lengths[i]]``
are copied to ``dst[b, dst_starts[i] : ...]``, for K and for V. Source rows are addressed in the
flat ``[B, H*S, D]`` view of a ``[B, H, S, D]`` tensor, i.e. ``src_start = head*S + token``
(enable_real_pruning_fast.py:469, :703-705). The copy is byte-exact: no dtype conversion.
"""

from __future__ import annotations

import numpy as np


def pack_flat_segments(dst_k: np.ndarray, dst_v: np.ndarray, src_k: np.ndarray,
                       src_v: np.ndarray, dst_starts, src_starts, lengths) -> None:
    """In-place copy on numpy arrays shaped [B, rows, D] (any dtype, K and V may differ)."""
    for d0, s0, n in zip(np.asarray(dst_starts).tolist(), np.asarray(src_starts).tolist(),
                         np.asarray(lengths).tolist()):
        if n <= 0:
            continue
        dst_k[:, d0:d0 + n, :] = src_k[:, s0:s0 + n, :]
        dst_v[:, d0:d0 + n, :] = src_v[:, s0:s0 + n, :]


def copy_bytes(n_slots: int, batch: int, head_dim: int, k_itemsize: int, v_itemsize: int) -> int:
    """Algorithmic HBM bytes of a pack: every slot is read once and written once, for K and V
    (the byte counter of enable_real_pruning_fast.py:115-130 counts one direction)."""
    return 2 * int(n_slots) * int(batch) * int(head_dim) * (int(k_itemsize) + int(v_itemsize))
