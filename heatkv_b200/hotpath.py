"""Device-resident execution plan of the HeatKV hot path for a whole model.

For every layer this turns the static slab schedule (``scheduler.build_static_slot_schedule``) into
device tensors once, and emits the per-image launch sequence of the reference orchestrator
(enable_real_pruning_fast.py:1951-2254 with its defaults: static schedule, Triton static copy,
baseline-prefix activation) as prepared C-ABI calls:

* target ``t`` before the layer's first pruned target ``t0``: attention over the layer's dense
  cache (the reference's SDPA + ``torch.cat`` path, :2073-2121), here run by the same kernel with
  the dense cache ``[B, H, Ld, D]`` viewed as a flat slab and one segment per head. The current
  scale's K/V are appended into the preallocated dense cache (no concatenation copy) before the
  attention, so the head's one segment already ends with them (``HEATKV_ATTN_CURRENT_IN_SEGMENTS``:
  the same keys in the same order, in fewer 128-key tiles - one instead of two at targets 1-4);
  ``dense_append_first=False`` keeps the reference's order (append after the attention);
* end of scale ``t0 - 1``: activation pack of the retained (source, head) segments from the dense
  cache into the slab (``old_pack_runs_by_target[t0]``, :1999-2037 -> :871-967);
* targets ``t >= t0``: fused segmented attention over the slab (:2123-2155), then the append of the
  current scale into its slab segments (``append_runs_by_key[(t, t+1)]``, :2218-2225 -> :969-1024).

Calls go straight to libheatkv.so with pre-bound pointers (the validated Python wrappers are the
public per-call API; this engine is the pre-planned path used by the model installer, the benchmark
and CUDA-graph capture). Layers are visited scale by scale, like the model's forward.
"""

from __future__ import annotations

import ctypes
import dataclasses
import heapq
from typing import Callable, Optional

import numpy as np
import torch

from . import _native
from .scheduler import build_static_slot_schedule, copy_descriptors


NUM_SMS = 148
BLOCK_ROWS = 128   # query rows per block of the tcgen05 kernels
KEY_TILE = 128


def _makespan(costs: np.ndarray, sms: int) -> float:
    """Largest per-CTA sum when item i goes to CTA i % grid, grid = min(items, sms)."""
    grid = min(len(costs), sms)
    pad = (-len(costs)) % grid
    return float(np.pad(costs, (0, pad)).reshape(-1, grid).sum(axis=0).max())


def _head_tiles(slots_per_segment, q_len: int, current_in_segments: bool = False,
                key_tile: int = KEY_TILE) -> np.ndarray:
    """Key tiles of every head: its segments' tiles, then the current scale's (unless the current
    keys already end a non-empty head's segments)."""
    cur = (q_len + key_tile - 1) // key_tile
    out = []
    for segs in slots_per_segment:
        seg = sum((int(n) + key_tile - 1) // key_tile for n in segs if n > 0)
        out.append(seg + (0 if current_in_segments and seg > 0 else cur))
    return np.array(out, dtype=np.int64)


def plan_attention(slots_per_segment, q_len: int, batch: int, *, sms: int = NUM_SMS,
                   block_rows: int = BLOCK_ROWS, item_cost: float = 1.5,
                   merge_cost: Optional[float] = None, min_gain: float = 0.03,
                   current_in_segments: bool = False):
    """Length-aware schedule of one attention launch: heads longest first, and how many query
    blocks at the tail of the schedule to split in two key ranges so that the kernel's round-robin
    assignment of items to at most ``sms`` persistent CTAs fills its last wave.

    ``slots_per_segment[h]`` lists the head's segment lengths; ``block_rows`` is the kernel's query
    block (128 rows, one Q tile). Cost model, in units of one 128 x 128 query-tile x key-tile step:
    key tiles of the item, plus ``item_cost`` per item (Q load, pipeline fill, epilogue) and
    ``merge_cost`` (default 4) per half of a split block: each half writes an fp32 partial of its
    rows (64 KB) and the block's last CTA reads them back, several tile steps of time, so only
    tails that leave CTAs idle gain. The blocks are
    enumerated in the kernel's order (head rank, batch row, query block); a split of the last ``m``
    blocks is taken when it lowers the makespan by ``min_gain`` or more. Returns ``(head_order,
    splits, unsplit_blocks)``, the blocks counted in ``block_rows`` units."""
    if block_rows != KEY_TILE:
        raise ValueError("block_rows must be 128")
    if merge_cost is None:
        merge_cost = 4.0
    tiles = _head_tiles(slots_per_segment, q_len, current_in_segments)
    order = np.argsort(-tiles, kind="stable").astype(np.int32)
    nblk = (q_len + block_rows - 1) // block_rows
    per = block_rows // KEY_TILE
    nq = np.full(nblk, per, dtype=np.int64)
    nq[-1] = (q_len - (nblk - 1) * block_rows + KEY_TILE - 1) // KEY_TILE
    n_head = tiles[order]                                                   # [H]
    # block costs in kernel order; halves of a split block (the kernel's j0/n rounding)
    t_blk = np.broadcast_to(n_head[:, None, None], (len(order), batch, nblk)).reshape(-1)
    q_blk = np.broadcast_to(nq[None, None, :], (len(order), batch, nblk)).reshape(-1)
    whole = (t_blk * q_blk).astype(np.float64) + item_cost
    first = ((t_blk // 2) * q_blk).astype(np.float64) + item_cost + merge_cost
    second = ((t_blk - t_blk // 2) * q_blk).astype(np.float64) + item_cost + merge_cost
    blocks = len(whole)
    best = (_makespan(whole, sms), blocks)
    step = max(1, min(blocks, 2 * sms) // 64)
    for m in range(step, min(blocks, 2 * sms) + 1, step):
        u = blocks - m
        halves = np.stack([first[u:], second[u:]], axis=1).reshape(-1)
        span = _makespan(np.concatenate([whole[:u], halves]), sms)
        if span < best[0] * (1.0 - min_gain):
            best = (span, u)
    unsplit = best[1]
    return order, (2 if unsplit < blocks else 1), unsplit


def _greedy_map(costs: np.ndarray, sms: int):
    """Items longest first (ties: lower item first), each to the least-loaded CTA (ties: lower
    CTA); returns the slot map ``[rounds * grid]`` (CTA c's k-th item at ``c + k * grid``, -1 =
    empty), the grid and the makespan."""
    n = len(costs)
    grid = max(1, min(n, sms))
    heap = [(0.0, c) for c in range(grid)]
    per_cta = [[] for _ in range(grid)]
    for item in np.argsort(-costs, kind="stable"):
        load, c = heapq.heappop(heap)
        per_cta[c].append(int(item))
        heapq.heappush(heap, (load + float(costs[item]), c))
    rounds = max(len(x) for x in per_cta)
    item_map = np.full(rounds * grid, -1, dtype=np.int32)
    for c, items in enumerate(per_cta):
        for k, item in enumerate(items):
            item_map[c + k * grid] = item
    return item_map, grid, max(load for load, _ in heap)


def plan_column_split(slots_per_segment, q_len: int, batch: int, *, sms: int = NUM_SMS,
                      splits: Optional[int] = None, item_cost: float = 1.5,
                      merge_cost: float = 4.0, min_gain: float = 0.03,
                      current_in_segments: bool = False, key_tile: int = KEY_TILE):
    """Schedule of one column-split launch (128-row blocks): head order, key-range splits, and the
    item map that assigns the launch's items to its CTAs.

    Heads are ordered shortest first, so the split tail of the block order holds the longest
    blocks. Cost model as ``plan_attention`` (key tiles + ``item_cost`` per item, + ``merge_cost``
    per split item). With ``splits=None`` the longest ``k`` blocks are split in two for the ``k``
    (from a fixed candidate set, 0 included) whose greedy assignment has the lowest makespan, a
    split taken only when it gains ``min_gain``; a given ``splits`` splits every block that many
    ways (1 = none). Items then go longest first to the least-loaded CTA.
    ``key_tile`` = 64 plans the 64-key kernel (costs in its tile steps, ``sms`` = its CTAs).
    Returns ``(head_order, splits, unsplit_blocks, item_map, grid)``."""
    tiles = _head_tiles(slots_per_segment, q_len, current_in_segments, key_tile)
    order = np.argsort(tiles, kind="stable").astype(np.int32)
    nblk = (q_len + KEY_TILE - 1) // KEY_TILE                  # 128-row query blocks
    t_blk = np.repeat(tiles[order], batch * nblk)             # blocks in kernel order
    blocks = len(t_blk)

    def items(unsplit: int, nsplit: int) -> np.ndarray:
        whole = t_blk[:unsplit].astype(np.float64) + item_cost
        if nsplit <= 1 or unsplit == blocks:
            return whole
        t = t_blk[unsplit:, None]
        j = np.arange(nsplit)[None, :]
        n = (t * (j + 1)) // nsplit - (t * j) // nsplit
        return np.concatenate([whole, (n + item_cost + merge_cost).reshape(-1)])

    if splits is not None:
        nsplit = max(1, min(int(splits), 4))
        unsplit = blocks if nsplit == 1 else 0
    else:
        nsplit, unsplit = 1, blocks
        best = _greedy_map(items(blocks, 1), sms)[2]
        limit = best * (1.0 - min_gain)
        for k in sorted({1, 2, 4, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256, blocks}):
            if k > blocks:
                continue
            span = _greedy_map(items(blocks - k, 2), sms)[2]
            if span < limit and span < best:
                best, nsplit, unsplit = span, 2, blocks - k
    item_map, grid, _ = _greedy_map(items(unsplit, nsplit), sms)
    return order, nsplit, unsplit, item_map, grid


# heatkv_pack_job of include/heatkv.h
_JOB_DTYPE = np.dtype([("dst_k", "<u8"), ("dst_v", "<u8"), ("src_k", "<u8"), ("src_v", "<u8"),
                       ("src_rows", "<i8"), ("dst_rows", "<i8")])


@dataclasses.dataclass
class Launch:
    kind: str            # "attention" | "pack" | "proj" | "prep" | "gemm" | exchange kinds
    layer: int
    target: int
    fn: Callable
    args: tuple          # ctypes arguments without the trailing stream
    work: float          # algorithmic FLOPs (attention, proj, gemm) or HBM bytes (pack, prep)
    keep: object = None  # device arrays the arguments point into
    sources: tuple = ()  # (plan index, target) of the step inputs a pack reads
    # an attention launch flagged HEATKV_ATTN_CURRENT_IN_SEGMENTS: the (starts, ends, counts)
    # pointers of the same keys without the current scale inside the segments, for callers that
    # re-issue it through an entry point without a kernel selector (the scatter)
    unflagged_meta: Optional[tuple] = None
    nbytes: float = 0.0  # algorithmic HBM bytes of a launch whose work counts FLOPs (proj)

    def __call__(self, stream: ctypes.c_void_p) -> None:
        status = self.fn(*self.args, stream)
        if status != _native.HEATKV_OK:
            _native.check(status, f"{self.kind} launch (layer {self.layer}, target {self.target})")


def _dev(x: np.ndarray, device, dtype=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device)


class LayerPlan:
    """Slab schedule of one layer, resident on ``device``.

    ``merge_prefix``: the leading source scales that every head keeps at every fused target (the
    protected prefix, scales 0-2 = 21 tokens at 1024^2) sit in the reference's slab layout as one
    short segment each - three 64-key tiles for 21 keys. With the flag, the activation also copies
    each head's prefix tokens into an extra region past the reference layout (rows ``capacity_ref
    + h * prefix_len``), and the segment tables of the fused targets name that contiguous copy as
    one segment instead: the same keys in the same order, in one tile. The reference-layout region
    of the slab keeps its bytes."""

    def __init__(self, controller, layer_idx: int, num_heads: int, device, schedule=None,
                 merge_prefix: bool = False):
        self.layer = int(layer_idx)
        self.num_heads = int(num_heads)
        self.ranges = controller.scale_ranges
        self.num_scales = len(controller.scale_schedule)
        self.tokens = [self.ranges[s][1] - self.ranges[s][0] for s in range(self.num_scales)]
        sched = schedule if schedule is not None else build_static_slot_schedule(
            controller, layer_idx=layer_idx, num_heads=num_heads)
        self.schedule = sched
        self.capacity = int(sched["capacity"])
        self.first_target = next(
            (t for t in range(1, self.num_scales) if controller.any_removed(layer_idx, t)),
            self.num_scales)
        t0 = self.first_target
        # dense cache length per head: tokens before t0 (or before the last scale)
        self.dense_len = int(self.ranges[min(t0, self.num_scales - 1)][0])
        H, Ld = self.num_heads, self.dense_len
        # dense-prefix attention metadata: head h reads flat rows [h*Ld, h*Ld + T_t)
        self.dense_meta = {}
        for t in range(min(t0, self.num_scales)):
            old = int(self.ranges[t][0])
            st = (np.arange(H, dtype=np.int32) * Ld).reshape(H, 1)
            meta = (st, st + old, np.ones(H, dtype=np.int32) * (1 if old > 0 else 0))
            self.dense_meta[t] = tuple(_dev(m, device) for m in meta) + (meta,)
        # dense appends: scale t's tokens of head h -> flat row h*Ld + start_t
        self.dense_append = {}
        for t in range(min(t0, self.num_scales - 1)):
            n = self.tokens[t]
            dst = np.arange(H, dtype=np.int64) * Ld + int(self.ranges[t][0])
            src = np.arange(H, dtype=np.int64) * n
            ln = np.full(H, n, dtype=np.int64)
            self.dense_append[t] = (_dev(dst, device), _dev(src, device), _dev(ln, device), H, n,
                                    H * n)
        # dense targets whose scale is appended before its attention: one segment per head holds
        # the cached tokens and the scale, [h*Ld, h*Ld + T_t + n_t) (HEATKV_ATTN_CURRENT_IN_SEGMENTS)
        self.dense_meta_cur = {}
        for t in self.dense_append:
            end = int(self.ranges[t][1])
            st = (np.arange(H, dtype=np.int32) * Ld).reshape(H, 1)
            meta = (st, st + end, np.ones(H, dtype=np.int32))
            self.dense_meta_cur[t] = tuple(_dev(m, device) for m in meta) + (meta,)
        # activation: retained segments live at t0, read from the dense cache layout
        self.activation = None
        if t0 < self.num_scales:
            items = [(seg["offset"], seg["head"] * Ld + seg["scale_start"], seg["length"])
                     for seg in sched["segments_by_target"][t0]]
            if items:
                items.sort()
                arr = np.array(items, dtype=np.int64)
                self.activation = (_dev(arr[:, 0], device), _dev(arr[:, 1], device),
                                   _dev(arr[:, 2], device), len(items), int(arr[:, 2].max()),
                                   int(arr[:, 2].sum()))
        # fused targets: slab metadata and appends
        self.capacity_ref = self.capacity
        self.prefix_scales, self.prefix_len = 0, 0
        metas = {t: sched["metadata_cpu_by_target"][t] for t in range(t0, self.num_scales)}
        if merge_prefix and t0 < self.num_scales:
            metas = self._merge_prefix(metas, device,
                                       int(getattr(controller, "source_scale_start", 0) or 0))
        self.slab_meta = {}
        for t, (st, en, ct) in metas.items():
            self.slab_meta[t] = (_dev(st, device), _dev(en, device), _dev(ct, device), (st, en, ct))
        self.slab_append = {}
        for t in range(t0, self.num_scales - 1):
            d = copy_descriptors(sched["append_runs_by_key"].get((t, t + 1), []))
            if d is None:
                continue
            self.slab_append[t] = (_dev(d["dst_starts"], device), _dev(d["src_starts"], device),
                                   _dev(d["lengths"], device), d["item_count"], d["max_length"],
                                   d["slots"])

    def _merge_prefix(self, metas, device, protected: int):
        """The protected prefix scales (``protected`` = the controller's first source scale: the
        scales before it are never removed), merged into one segment per head over a contiguous
        copy past the reference layout (see the class doc). Only the protected prefix, not every
        scale a particular set of heads happens to keep, so that a layer's tiles - and results -
        do not depend on which heads a plan holds (a head-sharded rank computes the same bits as
        one GPU)."""
        H, Ld, t0 = self.num_heads, self.dense_len, self.first_target
        sched = self.schedule
        live = [{(seg["source_scale"], seg["head"]): seg["offset"]
                 for seg in sched["segments_by_target"][t]} for t in range(t0, self.num_scales)]
        P = 0
        while P < min(protected, t0) and all((P, h) in lv for lv in live for h in range(H)):
            P += 1
        if P < 2:
            return metas
        plen = int(self.ranges[P][0])
        # the first P segments of every head, in source order, must be exactly those scales
        for (st, en, ct), lv in zip(metas.values(), live):
            for h in range(H):
                if int(ct[h]) < P:
                    return metas
                for s in range(P):
                    if int(st[h, s]) != lv[(s, h)] or int(en[h, s] - st[h, s]) != self.tokens[s]:
                        return metas
        base = self.capacity_ref
        out = {}
        for t, (st, en, ct) in metas.items():
            S = st.shape[1]
            st2 = np.zeros((H, max(S - P + 1, 1)), dtype=st.dtype)
            en2 = np.zeros_like(st2)
            st2[:, 0] = base + np.arange(H) * plen
            en2[:, 0] = st2[:, 0] + plen
            st2[:, 1:] = st[:, P:]
            en2[:, 1:] = en[:, P:]
            out[t] = (st2, en2, (ct - P + 1).astype(ct.dtype))
        # the activation also writes the contiguous prefix copy (dense rows h*Ld .. h*Ld + plen)
        items = [(base + h * plen, h * Ld, plen) for h in range(H)]
        if self.activation is not None:
            d, s_, l_ = (x.cpu().numpy() for x in self.activation[:3])
            items += list(zip(d.tolist(), s_.tolist(), l_.tolist()))
        items.sort()
        arr = np.array(items, dtype=np.int64)
        self.activation = (_dev(arr[:, 0], device), _dev(arr[:, 1], device),
                           _dev(arr[:, 2], device), len(items), int(arr[:, 2].max()),
                           int(arr[:, 2].sum()))
        self.capacity = base + H * plen
        self.prefix_scales, self.prefix_len = P, plen
        return out

    def kernel_segment_lengths(self, t: int, current_in_cache: bool):
        """Per head, the segment lengths the kernel walks at target t, and whether the current
        scale's keys are inside them (a dense target appended before its attention)."""
        if current_in_cache and t in self.dense_meta_cur:
            end = int(self.ranges[t][1])
            return [[end] for _ in range(self.num_heads)], True
        return self.segment_lengths(t), False

    def segment_lengths(self, t: int):
        """Per head, the lengths of the slab segments attended at target t."""
        meta = self.dense_meta[t][3] if t < self.first_target else self.slab_meta[t][3]
        st, en, ct = meta
        return [[max(0, int(en[h, i]) - int(st[h, i])) for i in range(int(ct[h]))]
                for h in range(self.num_heads)]

    def attention_slots(self, t: int) -> np.ndarray:
        """Attended slab slots per head at target t (for FLOP accounting)."""
        meta = self.dense_meta[t][3] if t < self.first_target else self.slab_meta[t][3]
        st, en, ct = meta
        slots = np.zeros(self.num_heads, dtype=np.int64)
        for h in range(self.num_heads):
            for i in range(int(ct[h])):
                slots[h] += max(0, int(en[h, i]) - int(st[h, i]))
        return slots


class HotPath:
    """All layers of one model for a fixed batch: slabs, dense caches and launch plans."""

    def __init__(self, controller, num_layers: int, num_heads: int, batch: int, device,
                 k_dtype=torch.bfloat16, v_dtype=torch.bfloat16, head_dim: int = 128,
                 layers: Optional[list] = None, plan_splits=None,
                 dense_append_first: Optional[bool] = None, merge_prefix: bool = True):
        import os
        self.device = torch.device(device)
        # dense targets: append the scale to the dense cache before its attention, which then
        # walks one segment [cached tokens + scale] per head (default: HEATKV_DENSE_APPEND_FIRST,
        # else on)
        if dense_append_first is None:
            dense_append_first = os.environ.get("HEATKV_DENSE_APPEND_FIRST", "1") != "0"
        self.dense_append_first = bool(dense_append_first)
        self.num_layers = int(num_layers)
        self.num_heads = int(num_heads)
        self.batch = int(batch)
        self.head_dim = int(head_dim)
        self.k_dtype, self.v_dtype = k_dtype, v_dtype
        # the protected prefix scales as one segment per head at the fused targets (LayerPlan)
        self.merge_prefix = bool(merge_prefix)
        self.plans = [LayerPlan(controller, l, num_heads, self.device,
                                merge_prefix=self.merge_prefix) for l in
                      (layers if layers is not None else range(num_layers))]
        self.num_scales = self.plans[0].num_scales
        self.tokens = self.plans[0].tokens
        B, H, D = self.batch, self.num_heads, self.head_dim
        self.slab_k, self.slab_v, self.dense_k, self.dense_v = [], [], [], []
        for p in self.plans:
            cap = max(p.capacity, 1)
            self.slab_k.append(torch.zeros(B, cap, D, dtype=k_dtype, device=self.device))
            self.slab_v.append(torch.zeros(B, cap, D, dtype=v_dtype, device=self.device))
            ld = max(p.dense_len, 1)
            self.dense_k.append(torch.zeros(B, H * ld, D, dtype=k_dtype, device=self.device))
            self.dense_v.append(torch.zeros(B, H * ld, D, dtype=v_dtype, device=self.device))
        self.lib = _native.load()
        # length-aware schedule of every attention launch (host planner, device head orders)
        self.schedule = {}
        ws_bytes = 0
        # plan_splits (default: HEATKV_PLAN_SPLITS, else 1): "auto" = splits of the longest
        # blocks chosen by the planner for the kernel each launch runs, or a fixed number of
        # key-range splits for every block (1 = never split). Column-split and 64-key launches
        # always get an item map (greedy, longest first). On the 2B image the planner's splits
        # lost to none with both kernels (64-key: 659.6 against 702.5 TFLOP/s: a split block's
        # partial writes and merge cost more than the idle CTAs they fill), so the default is 1.
        # A split block sums its keys in a different order, so outputs are bit-reproducible
        # across launch shapes (e.g. head shards) only unsplit.
        if plan_splits is None:
            plan_splits = os.environ.get("HEATKV_PLAN_SPLITS", "1")
        forced = 0 if str(plan_splits) == "auto" else int(plan_splits)
        natural = os.environ.get("HEATKV_PLAN_ORDER", "lpt") == "natural"
        dt = _native.DTYPE_CODES
        for i, p in enumerate(self.plans):
            for t in range(self.num_scales):
                # the planner counts blocks of the kernel the launch will run
                run = self.lib.heatkv_attention_kernel_for(
                    dt[k_dtype], dt[k_dtype], dt[v_dtype], self.batch, self.num_heads,
                    self.tokens[t], _native.ATTN_AUTO, 1, 1, 0)
                imap = None
                lens, cis = p.kernel_segment_lengths(t, self.dense_append_first)
                if run == _native.RUN_TCGEN05_CS and not natural:
                    # column-split kernel: greedy item map (and tail splits of the longest blocks)
                    order, splits, unsplit, imap, grid = plan_column_split(
                        lens, self.tokens[t], self.batch, splits=forced if forced > 0 else None,
                        current_in_segments=cis)
                    imap = (torch.from_numpy(imap).to(self.device), grid)
                elif run == _native.RUN_TCGEN05_CS64 and not natural:
                    # 64-key kernel: two CTAs per SM; costs in its 64-key tile steps (an item's
                    # fill and drain ~3 of them, a split half's partial write and merge ~4)
                    order, splits, unsplit, imap, grid = plan_column_split(
                        lens, self.tokens[t], self.batch, splits=forced if forced > 0 else None,
                        sms=2 * NUM_SMS, item_cost=3.0, merge_cost=4.0, current_in_segments=cis,
                        key_tile=KEY_TILE // 2)
                    imap = (torch.from_numpy(imap).to(self.device), grid)
                else:
                    order, splits, unsplit = plan_attention(lens, self.tokens[t], self.batch,
                                                            block_rows=KEY_TILE,
                                                            current_in_segments=cis)
                    if run != _native.RUN_TCGEN05_CS:
                        splits, unsplit = 1, 0  # tf32 and exact launches run unsplit
                    if forced > 0:
                        splits, unsplit = forced, 0
                    if natural:
                        order = np.arange(self.num_heads, dtype=np.int32)
                self.schedule[(i, t)] = (torch.from_numpy(order).to(self.device), splits, unsplit,
                                         imap)
                ws_bytes = max(ws_bytes, int(self.lib.heatkv_attention_workspace_bytes(
                    self.batch, self.num_heads, self.tokens[t], splits)))
        self.workspace = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=self.device)

    def slab_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.slab_k + self.slab_v)

    # ------------------------------------------------------------------ launch plans
    def launches(self, inputs, outputs, *, kernel: int = _native.ATTN_AUTO,
                 softmax_scale: Optional[float] = None, batch_packs: bool = True) -> list:
        """Launch list of one image. ``inputs[i][t] = (q, k, v)`` ([B, H, n_t, D]) and
        ``outputs[i][t]`` ([B, n_t, H*D]) for plan index i; the tensors must stay alive.

        With ``batch_packs`` the compactions of every layer of a scale are issued as one batched
        launch after the scale's last attention (then the slab activations, which read the dense
        caches those appends complete): scale t's K/V are only read again at scale t + 1. With
        ``dense_append_first`` the dense-cache appends of a scale go before its attentions
        instead (one batched launch), and those attentions walk one segment per head that already
        ends with the scale (``HEATKV_ATTN_CURRENT_IN_SEGMENTS``)."""
        B, H, D = self.batch, self.num_heads, self.head_dim
        scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
        out = []
        for t in range(self.num_scales):
            n = self.tokens[t]
            first, appends, activations = [], [], []
            attn = []
            for i, p in enumerate(self.plans):
                q, k, v = inputs[i][t]
                o = outputs[i][t]
                dense = t < p.first_target
                cur_in = dense and self.dense_append_first and t in p.dense_meta_cur
                launch = self.attention_launch(i, t, q, k, v, o, kernel=kernel,
                                               softmax_scale=scale)
                row_k = D * k.element_size()
                row_v = D * v.element_size()
                jobs = []
                if dense and t in p.dense_append:
                    dst, src, ln, items, mx, slots = p.dense_append[t]
                    job = (self.dense_k[i], self.dense_v[i], k, v, H * n, H * max(p.dense_len, 1),
                           dst, src, ln, items, mx, slots)
                    if cur_in:
                        if batch_packs:
                            first.append((job, i))
                        else:
                            pre = self._pack(p.layer, t, *job, row_k, row_v)
                            pre.sources = ((i, t),)
                            attn.append(pre)
                    else:
                        jobs.append((appends, job))
                attn.append(launch)
                if dense and t + 1 == p.first_target and p.activation is not None:
                    dst, src, ln, items, mx, slots = p.activation
                    jobs.append((activations, (self.slab_k[i], self.slab_v[i], self.dense_k[i],
                                               self.dense_v[i], H * max(p.dense_len, 1),
                                               max(p.capacity, 1), dst, src, ln, items, mx,
                                               slots)))
                if not dense and t in p.slab_append:
                    dst, src, ln, items, mx, slots = p.slab_append[t]
                    jobs.append((appends, (self.slab_k[i], self.slab_v[i], k, v, H * n,
                                           max(p.capacity, 1), dst, src, ln, items, mx, slots)))
                for group, job in jobs:
                    if batch_packs:
                        group.append(job)
                    else:
                        attn.append(self._pack(p.layer, t, *job, row_k, row_v))
            if first:
                pre = self._pack_batched(t, [job for job, _ in first])
                pre.sources = tuple((i, t) for _, i in first)
                out.append(pre)
            out.extend(attn)
            for group in (appends, activations):
                if group:
                    out.append(self._pack_batched(t, group))
        return out

    def attention_launch(self, i: int, t: int, q, k, v, o, *, kernel: int = _native.ATTN_AUTO,
                         softmax_scale: Optional[float] = None) -> Launch:
        """The attention launch of plan ``i`` at target ``t`` (current ``q, k, v`` ``[B, H, n_t,
        D]``, output ``o`` ``[B, n_t, H * D]``): over the dense cache before the layer's first
        pruned target (one segment per head, already ending with the current scale when
        ``dense_append_first``), over the slab after it."""
        p = self.plans[i]
        B, H, D = self.batch, self.num_heads, self.head_dim
        n = self.tokens[t]
        scale = float(softmax_scale) if softmax_scale is not None else D ** -0.5
        dt = _native.DTYPE_CODES
        dense = t < p.first_target
        cur_in = dense and self.dense_append_first and t in p.dense_meta_cur
        # the segment metadata and head orders were uploaded at construction and no launch of
        # the step writes them: the attention kernel may stage them before its dependency wait
        sel = (int(kernel) | _native.ATTN_STATIC_META
               | (_native.ATTN_CURRENT_IN_SEGMENTS if cur_in else 0))
        if dense:
            st, en, ct, _ = p.dense_meta_cur[t] if cur_in else p.dense_meta[t]
            sk, sv = self.dense_k[i], self.dense_v[i]
            cap = H * max(p.dense_len, 1)
        else:
            st, en, ct, _ = p.slab_meta[t]
            sk, sv = self.slab_k[i], self.slab_v[i]
            cap = max(p.capacity, 1)
        flops = float(4 * n * (p.attention_slots(t) + n).sum() * D * B)
        order, splits, unsplit, imap = self.schedule[(i, t)]
        head = (_native.ptr(q), _native.ptr(sk), _native.ptr(sv), _native.ptr(st),
                _native.ptr(en), _native.ptr(ct), _native.ptr(k), _native.ptr(v),
                _native.ptr(o), dt[q.dtype], dt[k.dtype], dt[v.dtype], B, H, n, cap, D,
                int(st.shape[1]), ctypes.c_float(scale), sel, _native.ptr(order),
                int(splits), int(unsplit))
        ws = (_native.ptr(self.workspace), self.workspace.numel())
        lib = self.lib
        if imap is not None:
            launch = Launch("attention", p.layer, t, lib.heatkv_segmented_attention_mapped,
                            head + (_native.ptr(imap[0]), imap[0].numel(), imap[1]) + ws, flops)
        else:
            launch = Launch("attention", p.layer, t, lib.heatkv_segmented_attention_sched,
                            head + ws, flops)
        if cur_in:
            st0, en0, ct0, _ = p.dense_meta[t]
            launch.unflagged_meta = (_native.ptr(st0), _native.ptr(en0), _native.ptr(ct0))
        return launch

    def _pack_batched(self, t, jobs):
        """One batched pack launch for ``jobs`` (tuples as ``_pack`` takes them)."""
        dt = _native.DTYPE_CODES
        B, D = self.batch, self.head_dim
        recs = np.zeros(len(jobs), dtype=_JOB_DTYPE)
        item_job, dsts, srcs, lens = [], [], [], []
        align = 16
        nbytes = 0.0
        max_len = 0
        kd, vd = jobs[0][0].dtype, jobs[0][1].dtype
        for j, (dk, dv, sk, sv, src_rows, dst_rows, dst, src, ln, items, mx, slots) in \
                enumerate(jobs):
            if dk.dtype != kd or dv.dtype != vd:
                raise ValueError("a batched pack needs one K dtype and one V dtype")
            recs[j] = (dk.data_ptr(), dv.data_ptr(), sk.data_ptr(), sv.data_ptr(), src_rows,
                       dst_rows)
            for ptr_ in (dk.data_ptr(), dv.data_ptr(), sk.data_ptr(), sv.data_ptr()):
                while align > 1 and ptr_ % align:
                    align //= 2
            item_job.append(np.full(items, j, dtype=np.int32))
            dsts.append(dst)
            srcs.append(src)
            lens.append(ln)
            max_len = max(max_len, int(mx))
            nbytes += 2.0 * slots * B * D * (dk.element_size() + dv.element_size())
        job_dev = torch.from_numpy(recs.view(np.uint8).copy()).to(self.device)
        item_job = torch.from_numpy(np.concatenate(item_job)).to(self.device)
        dsts, srcs, lens = torch.cat(dsts), torch.cat(srcs), torch.cat(lens)
        keep = (job_dev, item_job, dsts, srcs, lens, jobs)
        launch = Launch("pack", -1, t, self.lib.heatkv_pack_kv_batched,
                        (_native.ptr(job_dev), len(jobs), _native.ptr(item_job),
                         _native.ptr(dsts), _native.ptr(srcs), _native.ptr(lens),
                         int(item_job.numel()), dt[kd], dt[vd], B, D, max_len, align), nbytes)
        launch.keep = keep
        return launch

    def _pack(self, layer, t, dk, dv, sk, sv, src_rows, dst_rows, dst, src, ln, items, mx, slots,
              row_k, row_v):
        dt = _native.DTYPE_CODES
        B, D = self.batch, self.head_dim
        nbytes = 2.0 * slots * B * (row_k + row_v)
        return Launch("pack", layer, t, self.lib.heatkv_pack_kv,
                      (_native.ptr(dk), _native.ptr(dv), _native.ptr(sk), _native.ptr(sv),
                       dt[dk.dtype], dt[dv.dtype], B, src_rows, dst_rows, D, _native.ptr(dst),
                       _native.ptr(src), _native.ptr(ln), items, mx), nbytes)

    @staticmethod
    def run(launches, stream=None, events=None) -> None:
        """Issue the launches on ``stream`` (default: current). ``events[j] = (start, end)``
        brackets launch j when given (timing events may be external graph nodes)."""
        s = stream if stream is not None else torch.cuda.current_stream()
        handle = ctypes.c_void_p(s.cuda_stream)
        if events is None:
            for launch in launches:
                launch(handle)
        else:
            for launch, ev in zip(launches, events):
                if ev is None:
                    launch(handle)
                else:
                    ev[0].record(s)
                    launch(handle)
                    ev[1].record(s)


def allocate_io(hot: HotPath, *, dtype=torch.bfloat16, seed: int = 0, device=None,
                pin_host: bool = False, fill: bool = True):
    """Seeded N(0, 1) inputs ``[plan][t] = (q, k, v)`` and outputs ``[plan][t]`` for one image of
    ``hot``. Each kind lives in one flat buffer (the views stay contiguous). With ``pin_host`` the
    buffers are pinned host memory instead."""
    device = hot.device if device is None else torch.device(device)
    B, H, D = hot.batch, hot.num_heads, hot.head_dim
    per_layer = sum(hot.tokens)
    nl = len(hot.plans)
    total = nl * B * H * per_layer * D
    kw = dict(dtype=dtype)
    if pin_host:
        bufs = [torch.empty(total, **kw).pin_memory() for _ in range(3)]
        obuf = torch.empty(total, **kw).pin_memory()
    else:
        bufs = [torch.empty(total, device=device, **kw) for _ in range(3)]
        obuf = torch.empty(total, device=device, **kw)
    if fill:
        gen = torch.Generator(device=bufs[0].device).manual_seed(seed)
        for b in bufs:
            b.normal_(generator=gen)
    inputs, outputs = [], []
    off = 0
    for _ in range(nl):
        li, lo = [], []
        for t in range(hot.num_scales):
            n = hot.tokens[t]
            sz = B * H * n * D
            li.append(tuple(b[off:off + sz].view(B, H, n, D) for b in bufs))
            lo.append(obuf[off:off + sz].view(B, n, H * D))
            off += sz
        inputs.append(li)
        outputs.append(lo)
    return inputs, outputs, bufs, obuf
