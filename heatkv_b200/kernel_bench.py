"""Micro-benchmark of one libheatkv kernel shape (used for tuning sweeps and ncu captures).

    python -m heatkv_b200.kernel_bench attention --rows 2 --heads 16 --q-len 4096 --slots 650
    python -m heatkv_b200.kernel_bench attention --dtype f32qk   # fp32 q/k, bf16 v (tf32 kernel)
    python -m heatkv_b200.kernel_bench pack --rows 2 --heads 16 --q-len 4096

``attention``: one call shaped like a fused target of the 2B model - per head six slab segments
(1, 4, 16, 36, 64 and the rest of ``--slots`` slots) plus ``--q-len`` current tokens.
``pack``: the append of one scale (every head's ``--q-len`` tokens) into a slab.
``pack-batched``: the same append for ``--layers`` layers (one slab and one source per layer) as
one ``heatkv_pack_kv_batched`` launch, as the pre-planned step issues a scale's appends.
``scas``: one layer's S-CAS update at a scale (``heatkv_scas_mass``) against the PyTorch
probabilities it avoids.
``qkv-prep``: one layer's q/k/v preparation (``heatkv_qkv_prepare``: cos-attention + RoPE under
autocast) against the PyTorch chain it replaces.
``qkv-project``: one layer's fused projection (``heatkv_qkv_project``: tcgen05 GEMM with cos-attention,
RoPE and the q/k/v layout in its epilogue) for ``--rows`` x ``--q-len`` tokens and ``--heads``
heads of 128 (embed dim = heads x 128), against cuBLAS (``torch.mm``) of the same projection.
``projected-step``: the whole projection-driven step of ``bench.py``'s default workload
(``heatkv_b200.projected``: 2B, 10 % budget, every layer and scale) for ``--rows`` rows, run
eagerly ``--iters`` times after ``--warmup`` (for ncu launch lists of exactly one step).
Prints per-call device time (CUDA events, warm, back to back) and the achieved TFLOP/s or GB/s.
"""

from __future__ import annotations

import argparse
import math

import torch

from . import _native
from .real_pruning_fused_attention import (fused_real_pruning_flat_segmented_attention,
                                           pack_flat_segments_kv)


def attention_case(rows, heads, q_len, slots, dtype=torch.bfloat16, device="cuda", seed=0,
                   vdtype=None):
    """Inputs of one attention call; q, k and the K slab in ``dtype``, v and the V slab in
    ``vdtype`` (default ``dtype``)."""
    vdtype = dtype if vdtype is None else vdtype
    g = torch.Generator(device=device).manual_seed(seed)
    q, k, v = (torch.randn(rows, heads, q_len, 128, device=device, generator=g).to(dt)
               for dt in (dtype, dtype, vdtype))
    cap = heads * slots
    pk, pv = (torch.randn(rows, cap, 128, device=device, generator=g).to(dt)
              for dt in (dtype, vdtype))
    lens = [n for n in (1, 4, 16, 36, 64) if n <= slots]
    while sum(lens) > slots:
        lens.pop()
    lens.append(slots - sum(lens))
    st = torch.zeros(heads, len(lens), dtype=torch.int32)
    en = torch.zeros_like(st)
    for h in range(heads):
        off = h * slots
        for i, n in enumerate(lens):
            st[h, i], en[h, i] = off, off + n
            off += n
    ct = torch.full((heads,), len(lens), dtype=torch.int32)
    kw = dict(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st.to(device),
              segment_ends=en.to(device), segment_counts=ct.to(device), current_k=k, current_v=v,
              softmax_scale=1.0 / math.sqrt(128))
    flops = 4.0 * q_len * (slots + q_len) * 128 * rows * heads
    return kw, flops


def time_call(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("kernel", choices=["attention", "pack", "pack-batched", "qkv-prep", "scas",
                                       "projected-step", "qkv-project"])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--rows", type=int, default=2)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--q-len", type=int, default=4096)
    ap.add_argument("--slots", type=int, default=650)
    ap.add_argument("--no-cos", action="store_true",
                    help="qkv-project: without the cos-attention normalisation")
    ap.add_argument("--no-rope", action="store_true", help="qkv-project: without the RoPE")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--dtype", choices=["bf16", "f16", "f32", "f32qk"], default="bf16",
                    help="f32qk: fp32 q/k with bf16 v, the real model's cos-attention dtypes")
    args = ap.parse_args(argv)
    dtype = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32,
             "f32qk": torch.float32}[args.dtype]
    if args.kernel == "qkv-project":
        import ctypes
        B, L, H = args.rows, args.q_len, args.heads
        C = H * 128
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(B * L, C, device="cuda", generator=g).bfloat16()
        w = (torch.randn(3 * C, C, device="cuda", generator=g) * 0.02).bfloat16()
        q, k, v = (torch.empty(B, H, L, 128, device="cuda", dtype=torch.bfloat16)
                   for _ in range(3))
        sm = torch.full((H,), 4.0, device="cuda")
        ang = torch.rand(L, 64, device="cuda", generator=g) * 6
        from .qkv_prep import rope_pair_groups
        cos, sin = rope_pair_groups(torch.cos(ang)), rope_pair_groups(torch.sin(ang))
        lib = _native.load()
        stream = _native.stream_handle(torch.device("cuda"))
        out = torch.empty(B * L, 3 * C, device="cuda", dtype=torch.bfloat16)

        def fused():
            _native.check(lib.heatkv_qkv_project(
                _native.ptr(x), _native.ptr(w), None, _native.ptr(q), _native.ptr(k),
                _native.ptr(v), _native.DTYPE_CODES[torch.bfloat16],
                _native.DTYPE_CODES[torch.bfloat16], B, L, H, C,
                None if args.no_cos else _native.ptr(sm), ctypes.c_float(1e-12),
                None if args.no_rope else _native.ptr(cos), None if args.no_rope else _native.ptr(sin),
                4 * L, None, None, 0, None, stream), "heatkv_qkv_project")
        flops = 2.0 * B * L * C * 3 * C
        ms = time_call(fused, args.iters, args.warmup)
        ms_mm = time_call(lambda: torch.mm(x, w.t(), out=out), args.iters, args.warmup)
        mode = ("" if not args.no_cos else " no-cos") + ("" if not args.no_rope else " no-rope")
        print(f"qkv-project rows={B} q_len={L} heads={H}{mode}: fused {ms * 1e3:.1f} us "
              f"({flops / ms / 1e9:.1f} TFLOP/s), cuBLAS GEMM alone {ms_mm * 1e3:.1f} us "
              f"({flops / ms_mm / 1e9:.1f} TFLOP/s)", flush=True)
    elif args.kernel == "projected-step":
        import os
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import bench
        from .hotpath import HotPath
        from .projected import ProjectedHotPath
        ctrl, layers, heads = bench.build_controller("2b", 0.10)
        hot = HotPath(ctrl, layers, heads, args.rows, torch.device("cuda"))
        proj = ProjectedHotPath(hot)
        x, _ = proj.allocate_inputs(list(range(args.rows)), seed=1)
        out, _ = proj.allocate_outputs()
        launches = proj.launches(x, out)
        stream = torch.cuda.current_stream()
        for _ in range(args.warmup):
            proj.run(launches, stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # the timed steps sit in an NVTX range, so a profiler can select exactly their launches
        # (ncu --nvtx --nvtx-include "projected_step/")
        torch.cuda.nvtx.range_push("projected_step")
        e0.record()
        for _ in range(args.iters):
            proj.run(launches, stream)
        e1.record()
        torch.cuda.nvtx.range_pop()
        e1.synchronize()
        att = sum(l.work for l in launches if l.kind == "attention")
        ms = e0.elapsed_time(e1) / args.iters
        print(f"projected step rows={args.rows}: {len(launches)} launches, {ms:.2f} ms/step, "
              f"attention {att / ms / 1e9:.1f} TFLOP/s over the step", flush=True)
    elif args.kernel == "attention":
        vdtype = torch.bfloat16 if args.dtype == "f32qk" else dtype
        kw, flops = attention_case(args.rows, args.heads, args.q_len, args.slots, dtype,
                                   vdtype=vdtype)
        ms = time_call(lambda: fused_real_pruning_flat_segmented_attention(**kw), args.iters,
                       args.warmup)
        print(f"attention rows={args.rows} heads={args.heads} q_len={args.q_len} "
              f"slots={args.slots} {args.dtype}: {ms * 1e3:.1f} us/call, "
              f"{flops / ms / 1e9:.1f} TFLOP/s", flush=True)
    elif args.kernel == "qkv-prep":
        # one layer's q/k/v preparation at a scale: qkv [rows, Lq, 3, heads, 128] bf16 -> fp32 q, k
        # and bf16 v with cos-attention and RoPE under autocast, against the PyTorch chain
        import torch.nn.functional as F

        from .qkv_prep import prepare_qkv
        B, L, H = args.rows, args.q_len, args.heads
        qkv = torch.randn(B, L, 3, H, 128, device="cuda").bfloat16()
        sm = torch.full((1, H, 1, 1), 4.0, device="cuda")
        ang = torch.rand(L, 64, device="cuda") * 6
        cos, sin = torch.cos(ang), torch.sin(ang)

        def torch_chain():
            q, k, v = qkv.unbind(dim=2)
            q, k, v = (x.permute(0, 2, 1, 3).contiguous() for x in (q, k, v))
            q = F.normalize(q, dim=-1, eps=1e-12).mul(sm).contiguous()
            k = F.normalize(k, dim=-1, eps=1e-12).contiguous()
            qk = torch.stack((q, k), dim=0)
            with torch.autocast("cuda", enabled=False):
                qk = qk.reshape(*qk.shape[:-1], -1, 2)
                qk = torch.stack([cos * qk[..., 0] - sin * qk[..., 1],
                                  sin * qk[..., 0] + cos * qk[..., 1]], dim=-1)
                qk = qk.reshape(*qk.shape[:-2], -1)
            return qk[0], qk[1], v

        with torch.autocast("cuda", dtype=torch.bfloat16):
            ms = time_call(lambda: prepare_qkv(qkv, scale_mul=sm, rope=(cos, sin)), args.iters,
                           args.warmup)
            ms_t = time_call(torch_chain, args.iters, args.warmup)
        nbytes = B * L * H * 128 * (3 * 2 + 2 * 4 + 2) + L * 64 * 2 * 4
        print(f"qkv-prep rows={B} heads={H} q_len={L}: {ms * 1e3:.1f} us/call, "
              f"{nbytes / ms / 1e6:.1f} GB/s; PyTorch chain {ms_t * 1e3:.1f} us "
              f"({ms_t / ms:.1f}x)", flush=True)
    elif args.kernel == "scas":
        # one layer's S-CAS update at a scale: --q-len queries over --slots earlier keys plus
        # themselves (every key so far), fp32 q/k, 12 source scales; against the reference's form
        # (PyTorch fp32 probabilities of both batch rows, then the per-scale sums of row 0)
        from .scas import ScasAccumulator
        B, L, H = args.rows, args.q_len, args.heads
        sched = list(__import__("heatkv_b200.synthetic", fromlist=["x"]).SCALE_SCHEDULE_1M)
        total = sum(a * b * c for a, b, c in sched)
        acc = ScasAccumulator(num_layers=1, num_heads=H, scale_schedule=sched, sink_scales=0,
                              device="cuda")
        K = min(total, args.slots + L)
        q = torch.randn(B, H, L, 128, device="cuda")
        k = torch.randn(B, H, K, 128, device="cuda")
        t = 12 if K == total else max(i for i in range(13) if sum(a * b * c for a, b, c in sched[:i]) + L <= K)
        ms = time_call(lambda: acc.update_from_qk(layer_idx=0, scale_ind=t, q=q, k=k, scale=0.0884),
                       args.iters, args.warmup)
        torch.backends.cuda.matmul.allow_tf32 = False

        def ref_form():
            probs = torch.softmax(torch.matmul(q.float(), k.float().transpose(-2, -1)) * 0.0884, -1)
            acc.update(layer_idx=0, scale_ind=t, probs=probs)
        ms_r = time_call(ref_form, max(2, args.iters // 4), 1)
        flops = 2.0 * L * K * 128 * H
        print(f"scas rows(ref)={B} heads={H} q_len={L} keys={K}: {ms * 1e3:.1f} us/call "
              f"({flops / ms / 1e9:.1f} TFLOP/s of row-0 QK); reference form {ms_r * 1e3:.1f} us "
              f"({ms_r / ms:.1f}x)", flush=True)
    elif args.kernel == "pack-batched":
        import numpy as np

        from .hotpath import _JOB_DTYPE
        H, n, B, L = args.heads, args.q_len, args.rows, args.layers
        lib = _native.load()
        srcs = [(torch.randn(B, H * n, 128, device="cuda").to(dtype),
                 torch.randn(B, H * n, 128, device="cuda").to(dtype)) for _ in range(L)]
        dsts = [(torch.zeros(B, H * n + 1000, 128, device="cuda", dtype=dtype),
                 torch.zeros(B, H * n + 1000, 128, device="cuda", dtype=dtype)) for _ in range(L)]
        jobs = np.zeros(L, dtype=_JOB_DTYPE)
        for j in range(L):
            jobs[j] = (dsts[j][0].data_ptr(), dsts[j][1].data_ptr(), srcs[j][0].data_ptr(),
                       srcs[j][1].data_ptr(), H * n, H * n + 1000)
        job_dev = torch.from_numpy(jobs.view(np.uint8).copy()).cuda()
        item_job = torch.arange(L, device="cuda", dtype=torch.int32).repeat_interleave(H)
        dst = (torch.arange(H, device="cuda", dtype=torch.int64) * n + 7).repeat(L)
        src = (torch.arange(H, device="cuda", dtype=torch.int64) * n).repeat(L)
        ln = torch.full((L * H,), n, device="cuda", dtype=torch.int64)
        stream = _native.stream_handle(torch.device("cuda"))
        dt = _native.DTYPE_CODES[dtype]

        def fn():
            _native.check(lib.heatkv_pack_kv_batched(
                _native.ptr(job_dev), L, _native.ptr(item_job), _native.ptr(dst),
                _native.ptr(src), _native.ptr(ln), L * H, dt, dt, B, 128, n, 16, stream),
                "pack batched")
        ms = time_call(fn, args.iters, args.warmup)
        nbytes = 2.0 * L * B * H * n * 128 * dsts[0][0].element_size() * 2
        print(f"pack-batched layers={L} rows={B} heads={H} tokens={n} {args.dtype}: "
              f"{ms * 1e3:.1f} us/call, {nbytes / ms / 1e6:.1f} GB/s", flush=True)
    else:
        H, n, B = args.heads, args.q_len, args.rows
        src_k = torch.randn(B, H * n, 128, device="cuda").to(dtype)
        src_v = torch.randn(B, H * n, 128, device="cuda").to(dtype)
        dst_k = torch.zeros(B, H * n + 1000, 128, device="cuda", dtype=dtype)
        dst_v = torch.zeros_like(dst_k)
        dst = torch.arange(H, device="cuda", dtype=torch.int64) * n + 7
        src = torch.arange(H, device="cuda", dtype=torch.int64) * n
        ln = torch.full((H,), n, device="cuda", dtype=torch.int64)
        fn = lambda: pack_flat_segments_kv(dst_k=dst_k, dst_v=dst_v, src_k=src_k, src_v=src_v,  # noqa: E731
                                           dst_starts=dst, src_starts=src, lengths=ln, max_length=n)
        ms = time_call(fn, args.iters, args.warmup)
        nbytes = 2.0 * B * H * n * 128 * dst_k.element_size() * 2
        print(f"pack rows={B} heads={H} tokens={n} {args.dtype}: {ms * 1e3:.1f} us/call, "
              f"{nbytes / ms / 1e6:.1f} GB/s", flush=True)
    flags = _native.device_status()
    assert flags == 0, f"device status flags {flags:#x}"


if __name__ == "__main__":
    main()
