"""The hot path driven by QKV projections: every (scale, layer) runs projection -> q/k/v preparation
-> segmented attention -> compaction, as the patched attention forward does per call
(enable_real_pruning_fast.py:2040-2072 for the projection and preparation, :2123-2155 for the
attention, :2218-2225 for the append), for every layer of a model and all 13 scales.

Per (scale ``t``, layer ``l``), on one stream:

1.-2. ``heatkv_qkv_project`` - the layer's ``mat_qkv`` projection of the scale's layer input
   ``x_t`` ``[rows, n_t, C]`` on the tensor cores, whose epilogue does the cos-attention
   normalisation (``scale_mul``), the 2-D RoPE and the ``[B, H, L, D]`` layout (the q/v biases of
   the reference's ``F.linear`` are zero at initialisation and left out). The same epilogue writes
   the scale's K/V rows into the layer's cache wherever that is safe before the attention: into
   the dense cache at every scale before the layer's first pruned target (the attention then reads
   the scale as the tail of each head's one segment), and into the slab for the heads whose new
   segment overlaps no slot the scale's attention reads (``scheduler.prep_append_split``). With
   ``fused_projection=False`` these are two launches: a cuBLAS GEMM (``torch.mm``) and
   ``heatkv_qkv_prepare_append``;
3. the segmented attention (``HotPath.attention_launch``; softmax scale 1 with cos-attention, as
   the model's ``self.scale``);
4. the rest of the append (heads whose slots the attention still reads) with ``heatkv_pack_kv``.

After the last layer of the scale before a layer's first pruned target, one batched launch packs
the retained segments of the dense caches into the slabs (the activation,
enable_real_pruning_fast.py:1999-2037). The scratch tensors (projection output, q/k/v) are shared
by all (scale, layer) calls, so the launches are serial on the stream; the attention output of
scale ``t`` is one ``[rows, n_t, C]`` tensor that every layer overwrites (the last layer's output
remains).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _native, synthetic
from .hotpath import HotPath, Launch, _dev
from .qkv_prep import rope_pair_groups
from .scheduler import copy_descriptors, prep_append_split


class ProjectedHotPath:
    """Projection-driven launches over ``hot`` (a ``HotPath`` of ``rows`` rows and ``hot.num_heads``
    local heads). ``global_heads[i]`` lists the model heads behind plan ``i``'s local heads (default:
    all heads, identity): the projection then uses those heads' rows of ``W_l`` and the
    cos-attention scale of those heads. ``embed_dim`` is the model width ``C`` (default: local
    heads x 128). ``biases[i]`` is plan ``i``'s ``[3C]`` projection bias, ``cat(q_bias,
    zero_k_bias, v_bias)`` (infinity/models/basic.py:226-227, :278); ``None`` applies none, which
    equals the zero biases of a random-initialised model."""

    def __init__(self, hot: HotPath, *, global_heads: Optional[Sequence[Sequence[int]]] = None,
                 embed_dim: Optional[int] = None, weight_seed: int = 0,
                 cos_attention: bool = True, rope: bool = True, scale_mul: float = None,
                 weights: Optional[List[torch.Tensor]] = None,
                 biases: Optional[List[Optional[torch.Tensor]]] = None,
                 fused_projection: bool = True):
        if hot.head_dim != 128:
            raise ValueError("the projected path needs head_dim 128")
        if not hot.dense_append_first:
            raise ValueError("the projected path appends dense scales before their attention")
        if hot.k_dtype not in (torch.bfloat16, torch.float16) or hot.v_dtype != hot.k_dtype:
            raise ValueError("the projected path runs 16-bit q/k/v")
        self.hot = hot
        # one heatkv_qkv_project launch per (scale, layer) (projection with the preparation and
        # the early appends in its epilogue), or a cuBLAS GEMM followed by heatkv_qkv_prepare*
        self.fused_projection = bool(fused_projection) and hot.num_heads % 2 == 0
        self.device = hot.device
        self.dtype = hot.k_dtype
        H, D = hot.num_heads, hot.head_dim
        self.num_heads = H
        self.embed_dim = int(embed_dim) if embed_dim is not None else H * D
        C = self.embed_dim
        if global_heads is None:
            global_heads = [list(range(H)) for _ in hot.plans]
        self.global_heads = [list(map(int, g)) for g in global_heads]
        if any(len(g) != H for g in self.global_heads):
            raise ValueError("global_heads must list one model head per local head")
        self.rows = hot.batch
        self.tokens = hot.tokens
        self.num_scales = hot.num_scales
        self.starts = [int(sum(self.tokens[:t])) for t in range(self.num_scales)]
        total = sum(self.tokens)
        nmax = max(self.tokens)
        B = self.rows
        # projection weights: the [3, H_local, D] rows of the layer's [3C, C] mat_qkv weight
        self.weights = []
        self.biases = []
        for i, p in enumerate(hot.plans):
            w = weights[i] if weights is not None else synthetic.qkv_weight(
                p.layer, C, seed=weight_seed, dtype=self.dtype, device=self.device)
            if tuple(w.shape) != (3 * C, C):
                raise ValueError("a QKV weight must be [3 * embed_dim, embed_dim]")
            idx = torch.tensor(self.global_heads[i], dtype=torch.long)
            rows = (torch.arange(3)[:, None, None] * C + idx[None, :, None] * D
                    + torch.arange(D)[None, None, :]).reshape(-1)
            if rows.numel() == 3 * C and torch.equal(rows, torch.arange(3 * C)):
                self.weights.append(w.to(self.device, self.dtype).contiguous())
            else:
                self.weights.append(w.to(self.device, self.dtype)[rows.to(w.device)].contiguous())
            b = biases[i] if biases is not None else None
            if b is not None:
                if tuple(b.shape) != (3 * C,):
                    raise ValueError("a QKV bias must be [3 * embed_dim]")
                # the values F.linear adds: the bias in the projection dtype, held as fp32
                b = b.to(self.device, self.dtype)[rows.to(b.device)].float().contiguous()
            self.biases.append(b)
        self.softmax_scale = 1.0 if cos_attention else D ** -0.5
        sm = synthetic.COS_ATTN_SCALE_MUL if scale_mul is None else float(scale_mul)
        self.scale_mul = (torch.full((H,), sm, dtype=torch.float32, device=self.device)
                          if cos_attention else None)
        if rope:
            cos, sin = synthetic.rope2d_rows()
            if cos.shape[0] < total:
                raise ValueError("rope table shorter than the schedule")
            self.rope_cos, self.rope_sin = cos.to(self.device), sin.to(self.device)
            # the fused projection reads the pair-group-major order (coalesced per warp)
            self.rope_cos_g = rope_pair_groups(self.rope_cos)
            self.rope_sin_g = rope_pair_groups(self.rope_sin)
        else:
            self.rope_cos = self.rope_sin = None
        # scratch shared by every (scale, layer) call (the projection output only without the
        # fused projection)
        self.qkv = torch.empty(0 if self.fused_projection else B * nmax * 3 * H * D,
                               dtype=self.dtype, device=self.device)
        self.q, self.k, self.v = (torch.empty(B * H * nmax * D, dtype=self.dtype,
                                              device=self.device) for _ in range(3))
        # per plan and scale: where the preparation writes the scale's K/V (dense cache, slab or
        # nowhere) and the append copy left for after the attention
        self.prep_target = {}
        self.rest_append = {}
        self.early_slots = 0
        self.rest_slots = 0
        for i, p in enumerate(hot.plans):
            ld = max(p.dense_len, 1)
            for t in range(self.num_scales):
                if t in p.dense_append:
                    off = np.arange(H, dtype=np.int64) * ld + int(p.ranges[t][0])
                    self.prep_target[(i, t)] = (hot.dense_k[i], hot.dense_v[i], H * ld,
                                                _dev(off, self.device), H)
                    self.early_slots += H * self.tokens[t]
                elif t >= p.first_target and t + 1 < self.num_scales:
                    split = prep_append_split(p.schedule, t, H)
                    if split is None:
                        continue
                    if (split["offsets"] >= 0).any():
                        self.prep_target[(i, t)] = (hot.slab_k[i], hot.slab_v[i],
                                                    max(p.capacity, 1),
                                                    _dev(split["offsets"], self.device),
                                                    int((split["offsets"] >= 0).sum()))
                        self.early_slots += split["early_slots"]
                    d = copy_descriptors(split["rest_runs"])
                    if d is not None:
                        self.rest_append[(i, t)] = (_dev(d["dst_starts"], self.device),
                                                    _dev(d["src_starts"], self.device),
                                                    _dev(d["lengths"], self.device),
                                                    d["item_count"], d["max_length"], d["slots"])
                        self.rest_slots += d["slots"]

    # ------------------------------------------------------------------ buffers
    def allocate_inputs(self, row_ids: Sequence[int], *, seed: int = 0, dtype=None):
        """The layer inputs ``x[t]`` ``[rows, n_t, C]`` of every scale, each contiguous, as views
        of one flat buffer (scale-major). Row ``r`` of the batch is N(0, 1) from its own generator
        (``seed`` and the global row id ``r``) over all its tokens, so a rank holding rows 8..15
        of a 64-row batch gets the same values as one GPU holding all 64. Returns ``(x, flat)``."""
        dtype = self.dtype if dtype is None else dtype
        total = sum(self.tokens)
        C = self.embed_dim
        if len(row_ids) != self.rows:
            raise ValueError("one row id per row")
        flat = torch.empty(self.rows * total * C, dtype=dtype, device=self.device)
        x, off = [], 0
        for n in self.tokens:
            sz = self.rows * n * C
            x.append(flat[off:off + sz].view(self.rows, n, C))
            off += sz
        for j, r in enumerate(row_ids):
            gen = torch.Generator(device=self.device).manual_seed(seed * 7919 + int(r))
            tmp = torch.empty(total, C, dtype=torch.float32, device=self.device)
            tmp.normal_(generator=gen)
            for t, (s0, n) in enumerate(zip(self.starts, self.tokens)):
                x[t][j].copy_(tmp[s0:s0 + n])
            del tmp
        return x, flat

    def allocate_outputs(self):
        """One output ``[rows, n_t, H * D]`` per scale (shared by the layers, contiguous) as
        views of one flat buffer. Returns ``(out, flat)``."""
        H, D = self.num_heads, self.hot.head_dim
        total = sum(self.tokens)
        flat = torch.empty(self.rows * total * H * D, dtype=self.dtype, device=self.device)
        out, off = [], 0
        for n in self.tokens:
            sz = self.rows * n * H * D
            out.append(flat[off:off + sz].view(self.rows, n, H * D))
            off += sz
        return out, flat

    def current(self, t: int):
        """The scratch q, k, v ``[rows, H, n_t, D]`` and projection output ``[rows * n_t, 3C_l]``
        (None with the fused projection) of scale ``t``."""
        B, H, D, n = self.rows, self.num_heads, self.hot.head_dim, self.tokens[t]
        q, k, v = (b[:B * H * n * D].view(B, H, n, D) for b in (self.q, self.k, self.v))
        qkv = (None if self.fused_projection
               else self.qkv[:B * n * 3 * H * D].view(B * n, 3 * H * D))
        return q, k, v, qkv

    # ------------------------------------------------------------------ launches
    def launches(self, x, out, *, kernel: int = _native.ATTN_AUTO) -> list:
        """The step's launches: for every scale, for every layer: projection, preparation (with
        the early appends), attention into ``out[t]``, the rest of the append; then the scale's
        batched activation packs. ``x``/``out`` come from ``allocate_inputs``/``allocate_outputs``
        and must stay alive while the launches are used; ``out`` may also hold one list of
        per-scale outputs per plan (``out[i][t]``), to keep every layer's output."""
        hot = self.hot
        lib = hot.lib
        dt = _native.DTYPE_CODES
        B, H, D = self.rows, self.num_heads, hot.head_dim
        C = self.embed_dim
        code = dt[self.dtype]
        row = D * torch.empty(0, dtype=self.dtype).element_size()
        out_launches = []
        for t in range(self.num_scales):
            n = self.tokens[t]
            q, k, v, qkv = self.current(t)
            if not x[t].is_contiguous():
                raise ValueError("the layer inputs must be contiguous per scale")
            x2d = x[t].view(B * n, C)
            activations = []
            for i, p in enumerate(hot.plans):
                w = self.weights[i]
                flops = 2.0 * B * n * C * w.shape[0]
                target = self.prep_target.get((i, t))
                cos = sin = cos_g = sin_g = None
                if self.rope_cos is not None:
                    cos = ctypes.c_void_p(self.rope_cos.data_ptr() + self.starts[t] * 64 * 4)
                    sin = ctypes.c_void_p(self.rope_sin.data_ptr() + self.starts[t] * 64 * 4)
                    cos_g = ctypes.c_void_p(self.rope_cos_g.data_ptr() + self.starts[t] * 4 * 4)
                    sin_g = ctypes.c_void_p(self.rope_sin_g.data_ptr() + self.starts[t] * 4 * 4)
                    group_stride = 4 * self.rope_cos_g.shape[1]
                written = 0 if target is None else target[4]
                if self.fused_projection:
                    # x read once per column panel from HBM, q/k/v and the early cache rows written
                    nbytes = float(B * n * (C * 2 + H * 3 * row + written * 2 * row))
                    sk, sv, rows_, offs = (None, None, 0, None) if target is None else target[:4]
                    out_launches.append(Launch(
                        "proj", p.layer, t, lib.heatkv_qkv_project,
                        (_native.ptr(x2d), _native.ptr(w), _native.ptr(self.biases[i]),
                         _native.ptr(q), _native.ptr(k),
                         _native.ptr(v), code, code, B, n, H, C, _native.ptr(self.scale_mul),
                         ctypes.c_float(1e-12), cos_g, sin_g,
                         group_stride if cos_g is not None else 0, _native.ptr(sk),
                         _native.ptr(sv), rows_, _native.ptr(offs)), flops))
                    out_launches[-1].nbytes = nbytes
                else:
                    def gemm(stream, x2d=x2d, w=w, qkv=qkv, b=self.biases[i]):
                        if b is None:
                            torch.mm(x2d, w.t(), out=qkv)
                        else:
                            torch.addmm(b.to(qkv.dtype), x2d, w.t(), out=qkv)
                        return _native.HEATKV_OK
                    out_launches.append(Launch("gemm", p.layer, t, gemm, (), flops))
                    common = (_native.ptr(qkv), _native.ptr(q), _native.ptr(k), _native.ptr(v),
                              code, code, B, n, H, D, _native.ptr(self.scale_mul),
                              ctypes.c_float(1e-12), cos, sin, 64)
                    nbytes = float(B * n * H * (3 * row + 3 * row) + B * n * written * 2 * row)
                    if target is None:
                        prep = Launch("prep", p.layer, t, lib.heatkv_qkv_prepare, common, nbytes)
                    else:
                        sk, sv, rows_, offs, written = target
                        prep = Launch("prep", p.layer, t, lib.heatkv_qkv_prepare_append,
                                      common + (_native.ptr(sk), _native.ptr(sv), rows_,
                                                _native.ptr(offs)), nbytes)
                    out_launches.append(prep)
                o = out[i][t] if isinstance(out[0], (list, tuple)) else out[t]
                out_launches.append(hot.attention_launch(i, t, q, k, v, o, kernel=kernel,
                                                         softmax_scale=self.softmax_scale))
                rest = self.rest_append.get((i, t))
                if rest is not None:
                    dst, src, ln, items, mx, slots = rest
                    out_launches.append(hot._pack(p.layer, t, hot.slab_k[i], hot.slab_v[i],
                                                  k.view(B, H * n, D), v.view(B, H * n, D),
                                                  H * n, max(p.capacity, 1), dst, src, ln, items,
                                                  mx, slots, row, row))
                if t + 1 == p.first_target and p.activation is not None:
                    dst, src, ln, items, mx, slots = p.activation
                    activations.append((hot.slab_k[i], hot.slab_v[i], hot.dense_k[i],
                                        hot.dense_v[i], H * max(p.dense_len, 1),
                                        max(p.capacity, 1), dst, src, ln, items, mx, slots))
            if activations:
                out_launches.append(hot._pack_batched(t, activations))
        return out_launches

    @staticmethod
    def run(launches, stream=None, events=None) -> None:
        """Issue the launches on ``stream`` (default: current), with torch's current stream set to
        it for the projection GEMMs."""
        s = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            HotPath.run(launches, s, events)
