"""CPU sample of the benchmark workload - BENCHMARK AND TEST INFRASTRUCTURE ONLY.

The timed CPU baseline of ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm
run this same function on the same sample). It restates, with PyTorch CPU ops in fp32, the
reference's per-call CPU path of the patched attention forward for one layer and scale:

* projection ``F.linear(x, mat_qkv.weight)`` (enable_real_pruning_fast.py:2040-2043; the q/v biases
  are zero at initialisation);
* cos-attention ``F.normalize(q) * scale_mul``, ``F.normalize(k)`` (infinity/models/basic.py:282-287)
  and the 2-D rotary embedding (basic.py:97-117), in fp32;
* the flat-slab segmented attention of ``_flat_segmented_attention_reference``
  (real_pruning_fused_attention.py:312-361): per (row, head), SDPA over the head's slab segments
  followed by the current scale;
* the append of the scale into its slab segments (the ``index_select`` / ``copy_`` route of
  ``_segmented_flat_static_copy_precomputed_runs``, enable_real_pruning_fast.py:763-869).

The slab schedule is the one RECORDED FROM THE REFERENCE by ``tests/golden/make_golden.py``
(``schedule_<model>_b<budget>.npz``: per-target ``[H, S]`` segment tables, activation and append
copy items) and the first pruned target of each layer comes from the recorded keep-mask
(``budget_<model>_b<budget>.npz``), so this module loads no code of ``heatkv_b200`` and no native
library.
"""

from __future__ import annotations

import math
import os
import time

import numpy as np
import torch
import torch.nn.functional as F

SIDES_1M = (1, 2, 4, 6, 8, 12, 16, 20, 24, 32, 40, 48, 64)
GOLDEN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests",
                      "golden")


def scale_ranges(sides=SIDES_1M):
    out, cur = [], 0
    for s in sides:
        out.append((cur, cur + s * s))
        cur += s * s
    return out


class RecordedLayer:
    """One layer of the reference's recorded static slab schedule."""

    def __init__(self, sched: dict, removed: np.ndarray, layer: int, num_heads: int):
        ranges = scale_ranges()
        T = len(ranges)
        pre = f"L{layer}_"
        self.capacity = int(sched[pre + "caps"][0])
        # first target with a removal (removed: [target, source - 3, layer, head])
        hits = [t for t in range(1, T) if removed[t, :, layer, :].any()]
        self.first_target = hits[0] if hits else T
        self.dense_len = ranges[min(self.first_target, T - 1)][0]
        self.metadata = {}
        md = sched[pre + "metadata"]
        for t in range(1, T):
            rows = md[md[:, 0] == t]
            rows = rows[np.argsort(rows[:, 1])]
            width = int(rows[0, 3]) if len(rows) else 0
            starts = rows[:, 4:4 + width].astype(np.int64)
            ends = rows[:, 20:20 + width].astype(np.int64)
            self.metadata[t] = (starts, ends, rows[:, 2].astype(np.int64))
        op = sched[pre + "old_pack"]
        self.activation = op[op[:, 0] == self.first_target][:, 2:5]
        ap = sched[pre + "append"]
        self.append = {t: ap[ap[:, 0] == t][:, 2:5] for t in range(T - 1)}


def load_recorded(model: str = "2b", budget: float = 0.10, golden_dir: str = GOLDEN):
    tag = f"{model}_b{int(round(budget * 100)):02d}"
    sched = np.load(os.path.join(golden_dir, f"schedule_{tag}.npz"))
    removed = np.load(os.path.join(golden_dir, f"budget_{tag}.npz"))["removed"]
    return sched, removed


def rope_rows(head_dim: int = 128, max_side: int = 128, base: float = 10000.0):
    """(cos, sin) ``[tokens, head_dim / 2]`` of the square 1M schedule, mode 2 of
    ``precompute_rope2d_freqs_grid`` (basic.py:39-94): height angles then width angles of each
    token's position mapped onto the last scale's grid."""
    half = head_dim // 2
    inv = 1.0 / (base ** (torch.arange(0, half, 2, dtype=torch.int64).float() / half))
    pos = torch.arange(max_side, dtype=torch.float32)
    f = torch.outer(pos, inv)
    last = SIDES_1M[-1]
    cos, sin = [], []
    for s in SIDES_1M:
        i = (torch.arange(s) * (last / s)).round().long()
        ang = torch.cat([f[i][:, None, :].expand(s, s, -1), f[i][None, :, :].expand(s, s, -1)],
                        dim=-1).reshape(s * s, half)
        cos.append(torch.cos(ang))
        sin.append(torch.sin(ang))
    return torch.cat(cos), torch.cat(sin)


def _rope(x, c, s):
    a = x.reshape(*x.shape[:-1], -1, 2)
    return torch.stack([c * a[..., 0] - s * a[..., 1], s * a[..., 0] + c * a[..., 1]],
                       dim=-1).reshape(x.shape)


def prepare(x, w, cos, sin, *, heads: int = 16, scale_mul: float = 4.0):
    """Projection and q/k/v preparation of one scale: ``[B, n, C]`` -> q, k, v ``[B, H, n, D]``."""
    B, n, C = x.shape
    qkv = F.linear(x, w).view(B, n, 3, heads, C // heads)
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    q = F.normalize(q, dim=-1, eps=1e-12) * scale_mul
    k = F.normalize(k, dim=-1, eps=1e-12)
    return _rope(q, cos, sin), _rope(k, cos, sin), v.contiguous()


def layer_step(q, k, v, layer: RecordedLayer, t, slab_k, slab_v, *, softmax_scale: float):
    """Segmented attention of one (layer, fused target ``t``) over the slab, then the append of
    the scale into its slab segments. Returns the output ``[B, n, H * D]``."""
    B, heads, n, D = q.shape
    C = heads * D
    starts, ends, counts = layer.metadata[t]
    out = torch.empty(B, n, heads, D)
    for b in range(B):
        for h in range(heads):
            idx = [torch.arange(int(starts[h, i]), int(ends[h, i]))
                   for i in range(int(counts[h])) if starts[h, i] < ends[h, i]]
            if idx:
                sel = torch.cat(idx)
                keys = torch.cat([slab_k[b].index_select(0, sel), k[b, h]])
                vals = torch.cat([slab_v[b].index_select(0, sel), v[b, h]])
            else:
                keys, vals = k[b, h], v[b, h]
            out[b, :, h] = F.scaled_dot_product_attention(q[b, h][None], keys[None], vals[None],
                                                          scale=softmax_scale)[0]
    items = layer.append.get(t)
    if items is not None and len(items):
        fk, fv = k.reshape(B, heads * n, D), v.reshape(B, heads * n, D)
        for dst, src, ln in items.tolist():
            slab_k[:, dst:dst + ln] = fk[:, src:src + ln]
            slab_v[:, dst:dst + ln] = fv[:, src:src + ln]
    return out.reshape(B, n, C)


def cpu_sample(*, layers=(0, 1), n_targets: int = 5, rows: int = 2, heads: int = 16,
               model: str = "2b", budget: float = 0.10, seed: int = 0, project: bool = True,
               golden_dir: str = GOLDEN):
    """Time the reference's CPU path over the first ``n_targets`` fused targets of each of
    ``layers`` for ``rows`` batch rows. With ``project`` each call starts from the layer input
    (projection with N(0, 0.02) weights, cos-attention with scale_mul 4 and softmax scale 1, RoPE);
    without, from N(0, 1) q/k/v (softmax scale 1/sqrt(128)). The slab is filled by the recorded
    activation copy from a random dense cache and the inputs and weights are drawn before the
    clock starts. Returns ``(seconds, attention FLOPs, description)``; FLOPs = sum over
    (row, head) of 4 * n * (S_h + n) * D."""
    sched, removed = load_recorded(model, budget, golden_dir)
    ranges = scale_ranges()
    D = 128
    C = heads * D
    cos_all, sin_all = rope_rows(D)
    gen = torch.Generator().manual_seed(seed)
    seconds, flops, done = 0.0, 0, []
    for li in layers:
        layer = RecordedLayer(sched, removed, li, heads)
        t0 = layer.first_target
        targets = list(range(t0, len(ranges)))[:n_targets]
        cap = max(layer.capacity, 1)
        slab_k = torch.zeros(rows, cap, D)
        slab_v = torch.zeros(rows, cap, D)
        ld = layer.dense_len
        dense_k = torch.randn(rows, heads * max(ld, 1), D, generator=gen)
        dense_v = torch.randn(rows, heads * max(ld, 1), D, generator=gen)
        for dst, src, ln in layer.activation.tolist():
            slab_k[:, dst:dst + ln] = dense_k[:, src:src + ln]
            slab_v[:, dst:dst + ln] = dense_v[:, src:src + ln]
        w = torch.empty(3 * C, C).normal_(0.0, 0.02, generator=gen) if project else None
        for t in targets:
            lo, hi = ranges[t]
            n = hi - lo
            if project:
                x = torch.randn(rows, n, C, generator=gen)
                c, s = cos_all[lo:hi], sin_all[lo:hi]
                t1 = time.perf_counter()
                q, k, v = prepare(x, w, c, s, heads=heads)
                layer_step(q, k, v, layer, t, slab_k, slab_v, softmax_scale=1.0)
            else:
                q, k, v = (torch.randn(rows, heads, n, D, generator=gen) for _ in range(3))
                t1 = time.perf_counter()
                layer_step(q, k, v, layer, t, slab_k, slab_v, softmax_scale=D ** -0.5)
            seconds += time.perf_counter() - t1
            st, en, ct = layer.metadata[t]
            for h in range(heads):
                slots = sum(max(0, int(en[h, i]) - int(st[h, i])) for i in range(int(ct[h])))
                flops += 4 * n * (slots + n) * D * rows
        done.append(f"{li}:{targets[0]}..{targets[-1]}" if targets else f"{li}:-")
    what = ("projection + cos-norm + RoPE + segmented attention + append" if project
            else "segmented attention + append")
    desc = (f"{model.upper()} {int(round(budget * 100))}% layers/targets {','.join(done)}, "
            f"{rows} rows: {what}, torch "
            f"CPU fp32 on the reference's recorded slab schedule, {torch.get_num_threads()} "
            f"threads, {flops / 1e12:.3f} TFLOP in {seconds:.1f} s")
    return seconds, flops, desc


def cpu_threads() -> int:
    return int(torch.get_num_threads())


if __name__ == "__main__":  # pragma: no cover
    sec, fl, desc = cpu_sample()
    print(f"{fl / sec / 1e12:.4f} TFLOP/s", desc, f"({math.floor(sec)} s)")


def image_attention_flops(*, rows: int = 2, heads: int = 16, model: str = "2b",
                          budget: float = 0.10, golden_dir: str = GOLDEN) -> float:
    """Attention FLOPs of one step over every layer and scale for ``rows`` rows, from the
    recorded per-target segment tables (target 0 attends only its own token):
    sum over (layer, target, row, head) of 4 * n_t * (S_h + n_t) * 128."""
    sched, _ = load_recorded(model, budget, golden_dir)
    ranges = scale_ranges()
    n_layers = len([k for k in sched.files if k.endswith("_caps")])
    total = 4.0 * 1 * 1 * 128 * heads * rows * n_layers          # target 0
    for li in range(n_layers):
        md = sched[f"L{li}_metadata"]
        for row in md:
            t, count = int(row[0]), int(row[2])
            n = ranges[t][1] - ranges[t][0]
            slots = sum(max(0, int(row[20 + i]) - int(row[4 + i])) for i in range(count))
            total += 4.0 * n * (slots + n) * 128 * rows
    return total
