"""(batch row x head) sharding of the hot path over the GPUs of one node.

Within a (layer, scale) every (batch row, head) unit of the segmented attention is independent:
the slab is per batch row and the segments are per head. A GPU that owns a set of rows and, per
layer, a set of heads therefore needs only those rows' slab slices and those heads' segments, and
its attention and compaction launches are exactly the single-GPU ones on the smaller shapes.

Planning (host, install time):

* rows first: when the batch divides over the ranks, each rank takes ``batch / world``
  consecutive rows and every head - no unit of one output row lives on two GPUs;
* otherwise ``g = gcd(batch, world)`` row groups times ``world / g`` head groups; a layer's heads
  are split into equal-size groups, balanced by their attention work over the layer's 13 scales
  (longest-processing-time first, each head to the lightest group that still has room). Head
  groups are chosen per layer, since the pruned slab lengths differ from layer to layer.

Execution (``ShardedHotPath``): each rank runs the single-GPU engine (``hotpath.HotPath``) on its
rows x heads through a controller view restricted to its heads. When heads are split, or when
every rank must hold the full output, each attention launch is followed by an NCCL all-gather of
the rank blocks ``[rows, Lq, heads * D]`` (the collective the reference does not have: it runs on
one GPU) and by ``heatkv_gather_head_shards``, which places the gathered blocks into the
single-GPU layout ``[B, Lq, H * D]``.
"""

from __future__ import annotations

import dataclasses
import math
import ctypes
from typing import List, Optional

import numpy as np
import torch

from . import _native
from .hotpath import HotPath, Launch


# ------------------------------------------------------------------------------------------------
# work per (layer, head)
# ------------------------------------------------------------------------------------------------

def live_slots(controller, layer_idx: int) -> np.ndarray:
    """``int64 [num_scales, H]``: slab slots head ``h`` attends at target ``t``. Source scale
    ``s < t`` is attended unless it was removed at some target in ``(s, t]`` - the live interval
    rule of the static schedule (enable_real_pruning_fast.py:276-310)."""
    mask = controller.removed_mask_for_layer(layer_idx).astype(bool)   # [t, s, h]
    ranges = controller.scale_ranges
    T = len(controller.scale_schedule)
    H = mask.shape[2]
    tokens = np.array([ranges[s][1] - ranges[s][0] for s in range(T)], dtype=np.int64)
    out = np.zeros((T, H), dtype=np.int64)
    gone = np.zeros((T, H), dtype=bool)   # gone[s, h]: removed at some target so far
    for t in range(T):
        gone[:t] |= mask[t, :t, :]
        out[t] = (tokens[:t, None] * ~gone[:t]).sum(axis=0)
    return out


def head_costs(controller, num_layers: int, num_heads: int, head_dim: int = 128) -> np.ndarray:
    """``float64 [L, H]``: attention FLOPs of one batch row of (layer, head) over all scales,
    ``sum_t 4 * Lq_t * (S_t + Lq_t) * D``."""
    ranges = controller.scale_ranges
    T = len(controller.scale_schedule)
    lq = np.array([ranges[t][1] - ranges[t][0] for t in range(T)], dtype=np.float64)
    costs = np.zeros((num_layers, num_heads), dtype=np.float64)
    for l in range(num_layers):
        s = live_slots(controller, l).astype(np.float64)
        costs[l] = (4.0 * lq[:, None] * (s + lq[:, None]) * head_dim).sum(axis=0)
    return costs


def balanced_partition(costs, groups: int) -> List[List[int]]:
    """Split ``len(costs)`` items into ``groups`` groups of equal size with near-equal cost sums:
    items by decreasing cost, each to the lightest group that still has room (ties: lower group
    index, then lower item index), then pairwise swaps out of the heaviest group while they lower
    its load. Each group is returned sorted."""
    n = len(costs)
    if groups <= 0 or n % groups:
        raise ValueError(f"cannot split {n} heads into {groups} equal groups")
    size = n // groups
    order = sorted(range(n), key=lambda i: (-float(costs[i]), i))
    load = [0.0] * groups
    members: List[List[int]] = [[] for _ in range(groups)]
    for i in order:
        g = min((k for k in range(groups) if len(members[k]) < size), key=lambda k: (load[k], k))
        members[g].append(i)
        load[g] += float(costs[i])
    # refinement: swap one item of the heaviest group with one of another group while that
    # lowers the heaviest load (sizes stay equal); at most n * n rounds
    for _ in range(n * n):
        hi = max(range(groups), key=lambda k: (load[k], -k))
        best = None
        for k in range(groups):
            if k == hi:
                continue
            for a in members[hi]:
                for b in members[k]:
                    d = float(costs[a]) - float(costs[b])
                    if d <= 0:
                        continue
                    new_max = max(load[hi] - d, load[k] + d)
                    if new_max < load[hi] - 1e-9 * max(load[hi], 1.0) and \
                            (best is None or new_max < best[0]):
                        best = (new_max, k, a, b, d)
        if best is None:
            break
        _, k, a, b, d = best
        members[hi].remove(a)
        members[hi].append(b)
        members[k].remove(b)
        members[k].append(a)
        load[hi] -= d
        load[k] += d
    return [sorted(m) for m in members]


# ------------------------------------------------------------------------------------------------
# plan
# ------------------------------------------------------------------------------------------------

@dataclasses.dataclass
class ShardPlan:
    world: int
    batch: int
    num_heads: int
    row_groups: int
    head_groups: int
    heads: List[List[List[int]]]   # heads[layer][head group] -> global heads (sorted)

    @property
    def rows_per_rank(self) -> int:
        return self.batch // self.row_groups

    @property
    def heads_per_rank(self) -> int:
        return self.num_heads // self.head_groups

    @property
    def splits_heads(self) -> bool:
        return self.head_groups > 1

    def coords(self, rank: int):
        """(row group, head group) of ``rank``."""
        return rank // self.head_groups, rank % self.head_groups

    def rows_of(self, rank: int) -> List[int]:
        rg, _ = self.coords(rank)
        r = self.rows_per_rank
        return list(range(rg * r, (rg + 1) * r))

    def heads_of(self, rank: int, layer: int) -> List[int]:
        return list(self.heads[layer][self.coords(rank)[1]])

    def row_map(self) -> np.ndarray:
        """int32 ``[world * rows_per_rank]``: global row of (rank, local row)."""
        return np.array([row for r in range(self.world) for row in self.rows_of(r)],
                        dtype=np.int32)

    def head_map(self, layer: int) -> np.ndarray:
        """int32 ``[world * heads_per_rank]``: global head of (rank, local head) at ``layer``."""
        return np.array([h for r in range(self.world) for h in self.heads_of(r, layer)],
                        dtype=np.int32)

    def imbalance(self, costs: np.ndarray) -> float:
        """Sum over layers of the heaviest rank's work / sum over layers of the mean rank's work
        (1.0 = perfectly balanced). Ranks meet at every attention's gather, so the heaviest rank
        of each layer sets its time."""
        worst = mean = 0.0
        for l in range(len(self.heads)):
            loads = [costs[l, g].sum() for g in self.heads[l]]
            worst += max(loads)
            mean += sum(loads) / len(loads)
        return float(worst / mean) if mean > 0 else 1.0


def plan_shards(costs: np.ndarray, batch: int, world: int, *, split: str = "auto") -> ShardPlan:
    """Assign (row, head) units of every layer to ``world`` ranks.

    ``split``: ``"auto"`` - rows when ``batch % world == 0``, else ``gcd(batch, world)`` row
    groups x head groups; ``"heads"`` - every rank holds all rows and one head group when the
    heads divide over the ranks (else as ``"auto"`` without the rows-only case); ``"rows"`` - rows
    only (``batch % world`` must be 0)."""
    costs = np.asarray(costs, dtype=np.float64)
    num_layers, num_heads = costs.shape
    if world <= 0 or batch <= 0:
        raise ValueError("world and batch must be positive")
    if split not in ("auto", "rows", "heads"):
        raise ValueError("split must be one of: auto, rows, heads")
    if split == "rows" or (split == "auto" and batch % world == 0):
        if batch % world:
            raise ValueError(f"{batch} rows do not split over {world} ranks")
        row_groups = world
    elif split == "heads" and num_heads % world == 0:
        row_groups = 1
    else:
        row_groups = math.gcd(batch, world)
    head_groups = world // row_groups
    if num_heads % head_groups:
        raise ValueError(f"{num_heads} heads do not split into {head_groups} equal groups")
    heads = [balanced_partition(costs[l], head_groups) for l in range(num_layers)]
    return ShardPlan(world, batch, num_heads, row_groups, head_groups, heads)


# ------------------------------------------------------------------------------------------------
# controller view of one rank's heads
# ------------------------------------------------------------------------------------------------

class HeadSubsetController:
    """The pruning controller restricted, per layer, to one rank's heads (renumbered 0..k-1), so
    the static slot schedule of a rank holds only its heads' segments. The first pruned target of
    a layer (where the slab takes over from the dense cache) stays the whole layer's."""

    def __init__(self, base, heads_by_layer: List[List[int]]):
        self.base = base
        self.heads_by_layer = [list(h) for h in heads_by_layer]
        self.num_layers = base.num_layers
        self.num_heads = len(self.heads_by_layer[0])
        self.scale_schedule = base.scale_schedule
        self.scale_ranges = base.scale_ranges
        self.source_scale_start = base.source_scale_start

    def reset(self):
        return None

    def removed_mask_for_layer(self, layer_idx: int) -> np.ndarray:
        return np.ascontiguousarray(
            self.base.removed_mask_for_layer(layer_idx)[:, :, self.heads_by_layer[layer_idx]])

    def any_removed(self, layer_idx: int, target_scale_idx: int) -> bool:
        # the whole layer's answer, not the subset's: every rank then switches from the dense
        # cache to the slab at the same scale and tiles each head's keys exactly as one GPU does
        # (segment by segment), so sharded outputs are bit-identical to single-GPU ones
        return self.base.any_removed(layer_idx, target_scale_idx)

    def removed_heads_by_source_for(self, layer_idx, target_scale_idx):
        local = {g: i for i, g in enumerate(self.heads_by_layer[layer_idx])}
        full = self.base.removed_heads_by_source_for(layer_idx, target_scale_idx)
        return {s: {local[h] for h in heads if h in local} for s, heads in full.items()}


# ------------------------------------------------------------------------------------------------
# engine
# ------------------------------------------------------------------------------------------------

class _DeviceArray:
    """A raw device allocation seen by torch through the CUDA array interface (no copy)."""

    _TYPESTR = {2: "<i2", 4: "<i4"}

    def __init__(self, ptr: int, nbytes: int, itemsize: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // itemsize,), "typestr":
                                         self._TYPESTR[itemsize], "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """A zeroed device buffer on this rank's GPU that every rank of ``group`` maps (CUDA IPC
    handles exchanged over the group, mappings opened by libheatkv on the current device, peer
    access enabled): ``ptrs[r]`` is rank r's buffer as seen from this process, ``local`` this
    rank's buffer as a tensor of ``dtype``. Collective to create; ``close()`` (also collective)
    unmaps the peers and frees the buffer once no rank uses it any more."""

    def __init__(self, nbytes: int, dtype: torch.dtype, device, group=None):
        import torch.distributed as dist

        self.lib = _native.load()
        self.group = group
        self.device = torch.device(device)
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _native.check(self.lib.heatkv_peer_alloc(int(nbytes), ctypes.byref(ptr), handle),
                          "peer buffer allocation")
            got = [None] * world
            dist.all_gather_object(got, (self.device.index, handle.raw), group=group)
            self.ptrs, self._opened = [], []
            for r, (dev_r, raw) in enumerate(got):
                if r == rank:
                    self.ptrs.append(ptr.value)
                    continue
                if dev_r != self.device.index:
                    _native.check(self.lib.heatkv_enable_peer_access(int(dev_r)), "peer access")
                peer = ctypes.c_void_p()
                _native.check(self.lib.heatkv_peer_open(raw, ctypes.byref(peer)), "peer mapping")
                self.ptrs.append(peer.value)
                self._opened.append(peer.value)
        itemsize = torch.empty(0, dtype=dtype).element_size()
        self._own = ptr.value
        raw_view = torch.as_tensor(_DeviceArray(ptr.value, nbytes, itemsize), device=self.device)
        self.local = raw_view.view(dtype)

    def close(self) -> None:
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)          # nobody stores into a peer any more
        with torch.cuda.device(self.device):
            for p in self._opened:
                _native.check(self.lib.heatkv_peer_close(ctypes.c_void_p(p)), "peer unmapping")
            dist.barrier(group=self.group)      # every mapping of this buffer is closed
            self.local = None
            _native.check(self.lib.heatkv_peer_free(ctypes.c_void_p(self._own)), "peer free")
        self._own = None
        self._opened = []


class ShardedHotPath:
    """One rank's part of a sharded hot path: its rows x heads of every layer on ``device``, and
    (with ``gather``) the exchange that gives every rank the full ``[B, Lq, H*D]`` output of each
    attention call:

    * ``exchange="nccl"``: the rank's block goes to an NCCL all-gather, then
      ``heatkv_gather_head_shards`` places the gathered blocks;
    * ``exchange="p2p"``: the attention kernel itself stores each output row into every rank's
      full output over NVLink (``heatkv_segmented_attention_scatter``; the full outputs are shared
      through CUDA IPC), then ``heatkv_peer_barrier`` makes the step's rows of every rank visible
      before anything later runs - no collective library call and no reassembly pass."""

    def __init__(self, controller, num_layers: int, num_heads: int, plan: ShardPlan, rank: int,
                 device, k_dtype=torch.bfloat16, v_dtype=torch.bfloat16, head_dim: int = 128,
                 group=None, gather: Optional[bool] = None, layers: Optional[list] = None,
                 exchange: str = "nccl", plan_splits=None):
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.exchange_kind = exchange
        self.plan = plan
        self.rank = int(rank)
        self.device = torch.device(device)
        self.group = group
        self.gather = plan.splits_heads if gather is None else bool(gather)
        if plan.splits_heads and not self.gather:
            raise ValueError("a plan that splits heads needs the output gather")
        heads_by_layer = [plan.heads_of(rank, l) for l in range(num_layers)]
        # the scatter epilogue runs unsplit, so the p2p exchange never plans key-range splits
        if exchange == "p2p":
            plan_splits = 1
        self.local = HotPath(HeadSubsetController(controller, heads_by_layer), num_layers,
                             plan.heads_per_rank, plan.rows_per_rank, self.device, k_dtype,
                             v_dtype, head_dim, layers=layers, plan_splits=plan_splits)
        self.plan_index = {lp.layer: i for i, lp in enumerate(self.local.plans)}
        self.num_scales = self.local.num_scales
        self.tokens = self.local.tokens
        self.head_dim = head_dim
        self.row_map = torch.from_numpy(plan.row_map()).to(self.device)
        self.head_maps = [torch.from_numpy(plan.head_map(l)).to(self.device)
                          for l in range(num_layers)]

    def _collective(self, recv: torch.Tensor, local: torch.Tensor):
        import torch.distributed as dist

        def run(stream):
            # the current stream is the launch stream (HotPath.run issues under it)
            dist.all_gather_into_tensor(recv.view(-1), local.view(-1), group=self.group)
            return _native.HEATKV_OK
        return run

    def allocate_full_outputs(self, batch_rows: int, num_heads: int, dtype=torch.bfloat16,
                              per_layer: bool = True):
        """The ``[B, n_t, H * D]`` outputs of every (layer, scale) as views of one flat buffer,
        ``full[i][t]``, and the flat buffer; with ``per_layer=False`` one output per scale shared
        by the layers, ``full[t]``. With the p2p exchange every rank's buffer is also mapped here
        (collective: every rank calls this once, in the same order)."""
        n_tot = sum(self.tokens)
        per_layer_elems = batch_rows * n_tot * num_heads * self.head_dim
        total = (len(self.local.plans) if per_layer else 1) * per_layer_elems
        if self.exchange_kind == "p2p":
            itemsize = torch.empty(0, dtype=dtype).element_size()
            self._full_buf = PeerBuffer(total * itemsize, dtype, self.device, self.group)
            flat = self._full_buf.local
            self._flag_buf = PeerBuffer(self.plan.world * 4, torch.int32, self.device, self.group)
            self._flag_ptrs = torch.tensor(self._flag_buf.ptrs, dtype=torch.int64,
                                           device=self.device)
            self._counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        else:
            flat = torch.zeros(total, dtype=dtype, device=self.device)
        full, off = [], 0
        for _ in (self.local.plans if per_layer else [None]):
            row = []
            for n in self.tokens:
                sz = batch_rows * n * num_heads * self.head_dim
                row.append(flat[off:off + sz].view(batch_rows, n, num_heads * self.head_dim))
                off += sz
            full.append(row)
        return (full if per_layer else full[0]), flat

    def close(self) -> None:
        """Release the peer-shared buffers (collective; after the last step has completed)."""
        for name in ("_full_buf", "_flag_buf"):
            buf = getattr(self, name, None)
            if buf is not None:
                buf.close()
                setattr(self, name, None)

    def allocate_gather_buffer(self, dtype=torch.bfloat16) -> torch.Tensor:
        """Receive buffer of the all-gather, sized for the largest scale."""
        p = self.plan
        n = max(self.tokens)
        return torch.empty(p.world * p.rows_per_rank * n * p.heads_per_rank * self.head_dim,
                           dtype=dtype, device=self.device)

    def launches(self, inputs, outputs, full_outputs=None, gather_buf=None, **kw) -> list:
        """Launch list of one image for this rank. ``inputs``/``outputs`` are the rank's local
        tensors (``hotpath.allocate_io`` of ``self.local``), indexed by plan (layer) index; with
        gathering, ``full_outputs[i][t]`` are ``[B, n_t, H * D]`` tensors that receive every
        rank's block after each attention. Every rank must issue the returned launches in the
        same order (the all-gathers are collective)."""
        base = self.local.launches(inputs, outputs, **kw)
        if not self.gather:
            return base
        return self.exchange(base, outputs, full_outputs, gather_buf)

    def exchange(self, base, outputs, full_outputs, gather_buf=None) -> list:
        """``base`` (any launch list of ``self.local`` whose attention launches write
        ``outputs[i][t]``, or ``outputs[t]`` when one output per scale is shared by the layers)
        with the exchange that gives every rank the full output ``full_outputs[i][t]`` (or
        ``full_outputs[t]``) of each attention: NCCL all-gather + placement, or the peer-to-peer
        scatter + barrier."""
        if self.exchange_kind == "p2p":
            return self._p2p_launches(base, full_outputs)
        if full_outputs is None or gather_buf is None:
            raise ValueError("gathering needs full_outputs and gather_buf")
        p = self.plan
        lib = self.local.lib
        dt = _native.DTYPE_CODES
        shared = not isinstance(outputs[0], (list, tuple))
        out = []
        for launch in base:
            out.append(launch)
            if launch.kind != "attention":
                continue
            layer, t = launch.layer, launch.target
            i = self.plan_index[layer]
            n = self.tokens[t]
            local = outputs[t] if shared else outputs[i][t]
            full = full_outputs[t] if shared else full_outputs[i][t]
            nbytes = float(p.world * local.numel() * local.element_size())
            if not p.splits_heads:
                # rank r holds rows [r * rows, (r + 1) * rows): the gather is the output itself
                out.append(Launch("allgather", layer, t, self._collective(full, local), (),
                                  nbytes))
                continue
            recv = gather_buf[: p.world * local.numel()]
            out.append(Launch("allgather", layer, t, self._collective(recv, local), (), nbytes))
            out.append(Launch(
                "gather", layer, t, lib.heatkv_gather_head_shards,
                (_native.ptr(full), _native.ptr(recv), dt[full.dtype], p.world, p.rows_per_rank,
                 n, p.heads_per_rank, p.batch, p.num_heads, self.head_dim,
                 _native.ptr(self.row_map), _native.ptr(self.head_maps[layer])), 2.0 * nbytes))
        return out

    def _p2p_launches(self, base, full_outputs):
        """Each attention launch becomes a scatter into every rank's full output, followed by
        the cross-GPU barrier."""
        if getattr(self, "_full_buf", None) is None:
            raise ValueError("the p2p exchange needs allocate_full_outputs() first")
        p = self.plan
        lib = self.local.lib
        rows = torch.tensor(p.rows_of(self.rank), dtype=torch.int32, device=self.device)
        heads = {}
        out = []
        for launch in base:
            if launch.kind != "attention":
                out.append(launch)
                continue
            layer, t = launch.layer, launch.target
            i = self.plan_index[layer]
            shared = not isinstance(full_outputs[0], (list, tuple))
            full = full_outputs[t] if shared else full_outputs[i][t]
            off = full.data_ptr() - self._full_buf.local.data_ptr()
            ptrs = torch.tensor([b + off for b in self._full_buf.ptrs], dtype=torch.int64,
                                device=self.device)
            if layer not in heads:
                heads[layer] = torch.tensor(p.heads_of(self.rank, layer), dtype=torch.int32,
                                            device=self.device)
            a = launch.args
            # a: q, sk, sv, st, en, ct, k, v, out, dtq, dtk, dtv, B, H, n, cap, D, S, scale,
            #    kernel, order, splits, unsplit, [item map, slots, grid,] ws, ws_bytes
            #    (HotPath.launches); the scatter runs unsplit, in the launch's item map when
            #    it has one (planned unsplit), and takes no kernel selector: a launch whose segments already end with the current scale
            #    (HEATKV_ATTN_CURRENT_IN_SEGMENTS) is re-issued with its prefix-only segments
            meta = launch.unflagged_meta or (a[3], a[4], a[5])
            args = (a[0], a[1], a[2], meta[0], meta[1], meta[2], a[6], a[7], _native.ptr(ptrs),
                    p.world, _native.ptr(rows), _native.ptr(heads[layer]), p.batch, p.num_heads,
                    a[9], a[10], a[11], a[12], a[13], a[14], a[15], a[16], a[17], a[18], a[20])
            fn = lib.heatkv_segmented_attention_scatter
            if launch.fn is lib.heatkv_segmented_attention_mapped and int(a[21]) == 1:
                # the planner's longest-first map of this launch numbers the same unsplit items
                fn = lib.heatkv_segmented_attention_scatter_mapped
                args = args + (a[23], a[24], a[25])
            scatter = Launch("attention", layer, t, fn, args, launch.work)
            scatter.keep = (ptrs, rows, heads[layer])
            out.append(scatter)
            out.append(Launch("barrier", layer, t, lib.heatkv_peer_barrier,
                              (_native.ptr(self._flag_ptrs), _native.ptr(self._counter), p.world,
                               self.rank), 0.0))
        return out
