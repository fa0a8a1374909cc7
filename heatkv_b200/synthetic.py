"""Seeded synthetic inputs with the shapes of the reference's Infinity workloads.

No weights, captions or images exist on the benchmark machines, so every tensor that drives the
hot path is generated here from a seed with ``torch.Generator`` on the CPU (bit-identical on any
host for the same torch version). The same recipes feed the golden-fixture generator, the parity
tests and ``bench.py``.

Shapes follow the reference: head_dim 128, 1024x1024 = 13-scale schedule with patch sides
1,2,4,6,8,12,16,20,24,32,40,48,64 (infinity/utils/dynamic_resolution.py:6-45), the 7-scale
``0.06M`` prefix of it, Infinity-2B = 32 layers x 16 heads, Infinity-8B = 40 layers x 28 heads.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Callable

import numpy as np
import torch

HEAD_DIM = 128
SIDES_1M = (1, 2, 4, 6, 8, 12, 16, 20, 24, 32, 40, 48, 64)
SCALE_SCHEDULE_1M = tuple((1, s, s) for s in SIDES_1M)
C1_SCALE_SCHEDULE = SCALE_SCHEDULE_1M[:7]


def scale_token_ranges(schedule) -> dict[int, tuple[int, int]]:
    """Half-open token range of every scale in the flattened sequence."""
    ranges, cursor = {}, 0
    for idx, (_, h, w) in enumerate(schedule):
        ranges[idx] = (cursor, cursor + int(h) * int(w))
        cursor += int(h) * int(w)
    return ranges


def random_removal_orders(num_layers: int, num_heads: int, *, seed: int, num_orders: int = 9):
    """Seeded stand-in for an S-CAS order file: one random permutation of all (head, layer)
    pairs per prunable source scale, in the ``[[head, layer], ...]`` format of orders/*.json."""
    rng = np.random.default_rng(seed)
    pairs = [(h, l) for l in range(num_layers) for h in range(num_heads)]
    orders = []
    for _ in range(num_orders):
        perm = rng.permutation(len(pairs))
        orders.append([[int(pairs[i][0]), int(pairs[i][1])] for i in perm])
    return orders


def first_pruned_target(removed_fn: Callable, num_scales: int, layer_idx: int = 0) -> int:
    """First target scale whose removed-head map for ``layer_idx`` is non-empty."""
    for t in range(1, num_scales):
        if any(bool(h) for h in removed_fn(layer_idx, t).values()):
            return t
    return num_scales


def output_checksums(out: np.ndarray) -> np.ndarray:
    """Order-insensitive float64 fingerprints of an attention output: sum, L1, L2^2 and a dot
    product with fixed pseudo-random weights (seed 99)."""
    x = np.asarray(out, dtype=np.float64).reshape(-1)
    w = np.random.default_rng(99).standard_normal(x.size)
    return np.array([x.sum(), np.abs(x).sum(), (x * x).sum(), (x * w).sum()], dtype=np.float64)


# ------------------------------------------------------------------------------------------------
# Config 1: 7 scales, one layer, batch 2 (1 image + CFG), 16 heads, fp32.
# ------------------------------------------------------------------------------------------------


@dataclasses.dataclass(frozen=True)
class Config1:
    batch: int
    num_heads: int
    head_dim: int
    softmax_scale: float
    removed_pairs: frozenset  # {(source_scale, head)} removed for every later target


def config1(seed: int = 0, keep_fraction: float = 0.10) -> Config1:
    """Keep-mask of config 1: scales 0-2 always kept; the prunable (source, head) pairs are the
    sources 3..5 (scale 6 is the last one and is never cached) and the top ``keep_fraction`` of
    them by a seeded U(0,1) score are kept, the rest removed for every later target."""
    num_heads = 16
    sources = (3, 4, 5)
    gen = torch.Generator().manual_seed(seed)
    scores = torch.rand((len(sources), num_heads), generator=gen, dtype=torch.float64)
    pairs = [(sources[i], h) for i in range(len(sources)) for h in range(num_heads)]
    flat = scores.reshape(-1).tolist()
    n_keep = max(1, int(round(keep_fraction * len(pairs))))
    ranked = sorted(range(len(pairs)), key=lambda i: (-flat[i], i))
    kept = {pairs[i] for i in ranked[:n_keep]}
    removed = frozenset(p for p in pairs if p not in kept)
    return Config1(batch=2, num_heads=num_heads, head_dim=HEAD_DIM,
                   softmax_scale=1.0 / math.sqrt(HEAD_DIM), removed_pairs=removed)


def config1_qkv(cfg: Config1, seed: int = 0, dtype=torch.float32):
    """Per scale s: (q, k, v) each [B, H, tokens_s, D] ~ N(0, 1)."""
    gen = torch.Generator().manual_seed(seed + 1)
    out = []
    for _, h, w in C1_SCALE_SCHEDULE:
        n = h * w
        q, k, v = (torch.randn((cfg.batch, cfg.num_heads, n, cfg.head_dim), generator=gen)
                   for _ in range(3))
        out.append((q.to(dtype), k.to(dtype), v.to(dtype)))
    return out


# ------------------------------------------------------------------------------------------------
# Small direct attention cases (edge cases of the flat-slab layout)
# ------------------------------------------------------------------------------------------------


@dataclasses.dataclass(frozen=True)
class AttentionCase:
    name: str
    dtype: str          # "f32" | "bf16" | "f16"
    batch: int
    heads: int
    q_len: int
    capacity: int       # slab slots; 0 with ``empty_slab`` means persisted K/V = None
    max_segments: int
    seed: int
    empty_slab: bool = False
    zero_count_head: bool = False
    long_segments: bool = False


ATTENTION_CASES = (
    AttentionCase("f32_basic", "f32", 2, 4, 24, 300, 5, 11),
    AttentionCase("f32_zero_count", "f32", 2, 3, 17, 200, 4, 12, zero_count_head=True),
    AttentionCase("f32_empty_slab", "f32", 2, 2, 9, 0, 0, 13, empty_slab=True),
    AttentionCase("f32_long", "f32", 1, 2, 130, 700, 6, 14, long_segments=True),
    AttentionCase("bf16_basic", "bf16", 2, 4, 24, 300, 5, 15),
    AttentionCase("bf16_long", "bf16", 1, 2, 130, 700, 6, 16, long_segments=True),
    AttentionCase("f16_basic", "f16", 2, 3, 33, 260, 4, 17),
)

_TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def random_segments(heads: int, max_segments: int, capacity: int, rng: np.random.Generator,
                    *, long_segments: bool = False, zero_count_head: bool = False):
    """Per-head half-open slot ranges inside [0, capacity), including empty (start >= end)
    entries and heads that use fewer than ``max_segments`` entries. Unused entries stay 0."""
    starts = np.zeros((heads, max_segments), dtype=np.int32)
    ends = np.zeros((heads, max_segments), dtype=np.int32)
    counts = np.zeros((heads,), dtype=np.int32)
    for h in range(heads):
        count = 0 if (zero_count_head and h == 0) else int(rng.integers(1, max_segments + 1))
        counts[h] = count
        for i in range(count):
            kind = rng.integers(0, 8)
            hi = 260 if long_segments else 70
            length = int(rng.integers(1, hi))
            start = int(rng.integers(0, max(1, capacity - length)))
            end = min(capacity, start + length)
            if kind == 0:       # empty entry, skipped by the kernel
                end = start
            elif kind == 1:     # inverted entry, also skipped
                start, end = end, start
            starts[h, i], ends[h, i] = start, end
    return starts, ends, counts


def attention_case_inputs(case: AttentionCase) -> dict:
    rng = np.random.default_rng(case.seed)
    gen = torch.Generator().manual_seed(case.seed)
    dt = _TORCH_DTYPES[case.dtype]
    shape = (case.batch, case.heads, case.q_len, HEAD_DIM)
    q, k, v = (torch.randn(shape, generator=gen).to(dt) for _ in range(3))
    if case.empty_slab:
        pk = pv = None
        starts = np.zeros((case.heads, 0), dtype=np.int32)
        ends = np.zeros((case.heads, 0), dtype=np.int32)
        counts = np.zeros((case.heads,), dtype=np.int32)
    else:
        pk = torch.randn((case.batch, case.capacity, HEAD_DIM), generator=gen).to(dt)
        pv = torch.randn((case.batch, case.capacity, HEAD_DIM), generator=gen).to(dt)
        starts, ends, counts = random_segments(
            case.heads, case.max_segments, case.capacity, rng,
            long_segments=case.long_segments, zero_count_head=case.zero_count_head)
    return {
        "q": q, "persisted_k": pk, "persisted_v": pv,
        "segment_starts": torch.from_numpy(starts), "segment_ends": torch.from_numpy(ends),
        "segment_counts": torch.from_numpy(counts), "current_k": k, "current_v": v,
        "softmax_scale": 1.0 / math.sqrt(HEAD_DIM),
    }


# ------------------------------------------------------------------------------------------------
# Config 5: Q/K/V generated by random-init Infinity-2B QKV projections.
# ------------------------------------------------------------------------------------------------


def rope2d_rows(schedule=SCALE_SCHEDULE_1M, *, head_dim: int = HEAD_DIM,
                normalized_by_hw: int = 2, max_side: int = 2048 // 16, base: float = 10000.0,
                pad_to_multiplier: int = 128):
    """``(cos, sin)`` fp32 ``[padded_tokens, head_dim / 2]``: the 2-D rotary table Infinity builds
    for a square schedule (``precompute_rope2d_freqs_grid``, infinity/models/basic.py:39-94, with
    the inference defaults ``rope2d_normalized_by_hw=2`` and ``pad_to_multiplier=128`` of
    tools/run_infinity.py:248, :469). Row ``i`` of a scale ``(1, ph, pw)`` holds the height angles
    ``y * theta_j`` then the width angles ``x * theta_j`` (``theta_j = base^(-2j / (head_dim /
    2))``), where ``(y, x)`` is the token's grid position mapped onto the last scale's grid
    (``round(i * last / ph)``, mode 2) or taken as is (mode 0)."""
    half = head_dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, 2, dtype=torch.int64).float() / half))
    pos = torch.arange(max_side, dtype=torch.int64).type_as(inv_freq)
    f_h = torch.outer(pos, inv_freq)
    f_w = torch.outer(pos, inv_freq)
    grid = torch.cat([f_h[:, None, :].expand(-1, max_side, -1),
                      f_w[None, :, :].expand(max_side, -1, -1)], dim=-1)
    grid = torch.stack([torch.cos(grid), torch.sin(grid)], dim=0)    # [2, side, side, half]
    _, last_h, last_w = schedule[-1]
    parts = []
    for _, ph, pw in schedule:
        if normalized_by_hw == 2:
            idx = torch.stack([
                (torch.arange(ph) * (last_h / ph)).reshape(ph, 1).expand(ph, pw),
                (torch.arange(pw) * (last_w / pw)).reshape(1, pw).expand(ph, pw)],
                dim=-1).round().int().reshape(-1, 2)
            part = grid[:, idx[:, 0], idx[:, 1], :]
        elif normalized_by_hw == 0:
            part = grid[:, :ph, :pw, :].reshape(2, ph * pw, half)
        else:
            raise ValueError("normalized_by_hw must be 0 or 2")
        parts.append(part.reshape(2, ph * pw, half))
    table = torch.cat(parts, dim=1)
    if pad_to_multiplier > 1 and table.shape[1] % pad_to_multiplier:
        pad = pad_to_multiplier - table.shape[1] % pad_to_multiplier
        table = torch.cat([table, torch.zeros(2, pad, half)], dim=1)
    return table[0].contiguous(), table[1].contiguous()


def qkv_weight(layer: int, embed_dim: int, *, seed: int = 0, std: float = 0.02,
               dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    """Random-init ``mat_qkv.weight`` ``[3 * embed_dim, embed_dim]`` ~ N(0, std) of one layer (the
    ``nn.Linear`` layout: the projection is ``x @ W^T``), drawn from ``seed`` and the layer index on
    ``device``'s generator."""
    gen = torch.Generator(device=device).manual_seed(seed * 1000003 + layer)
    w = torch.empty(3 * embed_dim, embed_dim, dtype=torch.float32, device=device)
    w.normal_(0.0, std, generator=gen)
    return w.to(dtype)


COS_ATTN_SCALE_MUL = 4.0   # exp(log(4)): the init value of scale_mul_1H11 (basic.py:216-221)


def scas_inputs(prompt: int, layer: int, schedule, *, heads: int = 16):
    """Seeded cos-attention-like q, k of every scale for one (prompt, layer) of an S-CAS capture:
    q = normalize(x) * 4, k = normalize(y), each ``[2, heads, n_s, 128]`` fp32 (row 1 plays the CFG
    row; the accumulator reads row 0 only), from the CPU generator."""
    gen = torch.Generator().manual_seed(10007 * prompt + 101 * layer + 5)
    out = []
    for _, h, w in schedule:
        q = torch.nn.functional.normalize(torch.randn(2, heads, h * w, HEAD_DIM, generator=gen),
                                          dim=-1) * 4.0
        k = torch.nn.functional.normalize(torch.randn(2, heads, h * w, HEAD_DIM, generator=gen),
                                          dim=-1)
        out.append((q, k))
    return out
