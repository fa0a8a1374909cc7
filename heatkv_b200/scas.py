"""S-CAS accumulation (tools/compute_scas.py:93-152) with the attention mass computed on the GPU in
one pass (``heatkv_scas_mass``, csrc/scas.cu) instead of from materialised probabilities.

``ScasAccumulator`` keeps the reference's interface: ``accum`` ``[layers, heads, scales]`` float64,
``update(layer_idx=, scale_ind=, probs=)`` from probabilities as the reference does it,
``update_from_qk(layer_idx=, scale_ind=, q=, k=, scale=)`` from the queries of the scale and every
key so far (the form the GPU kernel takes; the reference's capture forward computes exactly these
probabilities, :217-218), ``scores(num_prompts)`` and ``orders_from_scores(scores)``. Only batch
row 0 contributes, as in the reference (``probs[:1]``).
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import torch

from . import _native

__all__ = ["ScasAccumulator", "scale_token_bounds"]


def scale_token_bounds(scale_schedule: Sequence[Tuple[int, int, int]]) -> List[Tuple[int, int]]:
    """[start, end) token range of every scale (tools/compute_scas.py:57-64)."""
    bounds, cursor = [], 0
    for t, h, w in scale_schedule:
        n = int(t) * int(h) * int(w)
        bounds.append((cursor, cursor + n))
        cursor += n
    return bounds


class ScasAccumulator:
    """Per-(layer, head, source scale) attention mass of every later scale's queries."""

    def __init__(self, *, num_layers: int, num_heads: int, scale_schedule, sink_scales: int,
                 device):
        self.num_layers = int(num_layers)
        self.num_heads = int(num_heads)
        self.scale_schedule = scale_schedule
        self.sink_scales = int(sink_scales)
        self.num_scales = len(scale_schedule)
        self.bounds = scale_token_bounds(scale_schedule)
        self.accum = torch.zeros((self.num_layers, self.num_heads, self.num_scales),
                                 dtype=torch.float64, device=device)
        self._bounds_dev = {}

    def _sources(self, scale_ind: int, key_len: int) -> List[int]:
        """Source scales of a scale's update whose tokens are all present among key_len keys."""
        if scale_ind <= self.sink_scales or scale_ind >= self.num_scales:
            return []
        end = min(scale_ind, self.num_scales - 1)
        return [s for s in range(self.sink_scales, end) if self.bounds[s][1] <= key_len]

    def update(self, *, layer_idx: int, scale_ind: int, probs: torch.Tensor) -> None:
        """From probabilities ``[B, H, L, K]`` (the reference's form; batch row 0 only)."""
        sources = self._sources(int(scale_ind), probs.shape[-1])
        if not sources:
            return
        probs = probs[:1].float()
        for s in sources:
            start, end = self.bounds[s]
            mass = probs[..., start:end].sum(dim=-1).mean(dim=(0, 2))
            self.accum[int(layer_idx), :, s] += mass.to(dtype=torch.float64)

    def update_from_qk(self, *, layer_idx: int, scale_ind: int, q: torch.Tensor, k: torch.Tensor,
                       scale: float) -> None:
        """From the scale's queries ``q [B, H, L, 128]`` and every key so far ``k [B, H, K, 128]``
        (the cached scales, then the current one): probs = softmax(q k^T * scale) in fp32,
        computed and reduced on the GPU without being stored. q and k are widened to fp32 as the
        reference does (``q.float() @ k.float()^T``, tools/compute_scas.py:217), which runs the
        tensor-core kernel (three tf32 products a score)."""
        if q.ndim != 4 or k.ndim != 4 or q.shape[:2] != k.shape[:2] or q.shape[3] != k.shape[3]:
            raise ValueError("update_from_qk expects q [B, H, L, D] and k [B, H, K, D]")
        if not (q.is_cuda and k.is_cuda):
            raise RuntimeError("update_from_qk requires CUDA tensors")
        sources = self._sources(int(scale_ind), k.shape[2])
        if not sources:
            return
        lib = _native.load()
        dtype = torch.float32
        q0 = q[0].float().contiguous()
        k0 = k[0].float().contiguous()
        key = (sources[0], len(sources), q.device)
        b = self._bounds_dev.get(key)
        if b is None:
            offs = [self.bounds[s][0] for s in sources] + [self.bounds[sources[-1]][1]]
            b = self._bounds_dev[key] = torch.tensor(offs, dtype=torch.int32, device=q.device)
        out = self.accum[int(layer_idx), :, sources[0]:]
        _native.check(lib.heatkv_scas_mass(
            _native.ptr(q0), _native.ptr(k0), _native.DTYPE_CODES[dtype], q0.shape[0], q0.shape[1],
            k0.shape[1], q0.shape[2], float(scale), _native.ptr(b), len(sources), _native.ptr(out),
            self.accum.stride(1), _native.stream_handle(q.device)), "heatkv_scas_mass")

    def scores(self, num_prompts: int) -> torch.Tensor:
        """Mean mass per prompt and per later scale (tools/compute_scas.py:130-139)."""
        out = torch.full_like(self.accum, float("nan"))
        for s in range(self.sink_scales, self.num_scales - 1):
            future = self.num_scales - s - 1
            if future <= 0:
                continue
            out[:, :, s] = self.accum[:, :, s] / (float(num_prompts) * float(future))
        return out

    def orders_from_scores(self, scores: torch.Tensor) -> List[List[Tuple[int, int]]]:
        """Per source scale, the (head, layer) pairs by increasing score, ties by head then layer
        (tools/compute_scas.py:141-152): the removal orders the budget policy consumes."""
        cpu = scores.detach().cpu()
        orders = []
        for s in range(self.sink_scales, self.num_scales - 1):
            entries = sorted((float(cpu[l, h, s]), h, l) for l in range(self.num_layers)
                             for h in range(self.num_heads))
            orders.append([(h, l) for _, h, l in entries])
        return orders
