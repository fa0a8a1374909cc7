#!/usr/bin/env python
"""Benchmark of the HeatKV hot path on B200: segmented attention + slab compaction per image.

Workload: Infinity-2B attention stack at 1024x1024 - 32 layers x 16
heads x head_dim 128, 13 scales (10,521 tokens), batch 1 doubled to 2 rows for CFG, keep-mask of
the 10 % budget from orders/2b.json (strict schedule, 3 protected scales, source scales 3..11).
Q/K/V are seeded N(0, 1) bf16 tensors for every (layer, scale) - no weights exist on the box.

One step = one image: for every scale and layer, the attention call (dense-prefix scales and
fused-segmented scales, both through the tcgen05 kernel) and every compaction pack (dense-cache
append, slab activation, slab append). The step is captured once per timed step as a CUDA graph
with timing events around every launch; the inputs of a step (8.3 GB) exceed the 126 MB L2.

Output: one JSON line (rank 0). ``value`` = algorithmic attention TFLOP/s of the whole job
(sum over ranks of FLOPs / max over ranks of the step time), ``ms_per_image`` beside it;
``roofline`` for the attention kernel (tensor-bound) and ``roofline_pack`` for compaction
(HBM-bound); ``e2e`` = the same metric through the C-ABI with Q/K/V copied from pinned host memory
and outputs copied back every step; ``cpu_baseline`` = the CPU oracle on a bounded sample.
``--impl reference`` times the reference's CPU algorithm (the oracle port) instead.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "segmented-attn TFLOP/s & ms/image (2B shape, 1024^2, 10% budget)"
WORKLOAD = ("configs[1]: Infinity-2B attention stack at 1024^2 - 32 layers x 16 heads x 128, "
            "13 scales, batch 1 (+CFG = 2 rows) per GPU, 10% budget from orders/2b.json")
WORKLOAD_SHARDED = ("Infinity-2B attention stack at 1024^2, 10% budget from orders/2b.json: one "
                    "fixed batch sharded by (row, head) units over the GPUs, outputs all-gathered")
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def build_controller(model: str, budget: float):
    from heatkv_b200 import budget as bud
    from heatkv_b200.enable_pruning import (ScaleSpecificPruningController,
                                            _validate_and_normalize_removed_heads_by_scale_specific)
    layers, heads = (32, 16) if model == "2b" else (40, 28)

    class _M:
        num_heads = heads

    view = bud.strict_removed_heads_by_scale_specific_for_budget(
        budget, bud.orders(model_type=int(model[0])), num_layers=layers, num_heads=heads,
        source_scale_start=3, protected_prefix_scales=3)
    norm = _validate_and_normalize_removed_heads_by_scale_specific(
        view["removed_heads_by_scale"], [_M()] * layers, source_scale_start=3)
    ctrl = ScaleSpecificPruningController(num_layers=layers, num_heads=heads,
                                          static_removed_heads_by_scale=norm, source_scale_start=3)
    return ctrl, layers, heads


class ClockSampler:
    """nvidia-smi samples every 100 ms while the timed region runs. The sampler waits (at most
    3 s) for nvidia-smi's first line before the region starts and keeps only the lines that
    arrive after that, so the summary describes the timed region, not the idle GPU before it."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 100):
        self.gpu = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self._raw = []
        self.lines = []

    def _read(self):
        for line in self.proc.stdout:
            self._raw.append((time.monotonic(), line))

    def __enter__(self):
        import threading
        self._raw = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
        except (OSError, ValueError):
            self.proc = None
        if self.proc is not None:
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
            t0 = time.monotonic()
            while not self._raw and self.proc.poll() is None and time.monotonic() - t0 < 3.0:
                time.sleep(0.01)
        self.t_start = time.monotonic()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self._thread.join(timeout=5)
        self.lines = [l for t, l in self._raw if t >= self.t_start and l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# CPU baseline: the oracle (numpy restatement of the reference's torch CPU path)
# ------------------------------------------------------------------------------------------------

def cpu_sample(hot_cpu_plan, batch: int, layer_targets, seed: int = 0):
    """Run the oracle on one layer's fused targets (slab built by the oracle pack from the dense
    cache + appends), fp32 like the reference's CPU path. Returns (seconds, flops)."""
    import torch

    from oracle.attention import segmented_attention
    from oracle.pack import pack_flat_segments

    p = hot_cpu_plan
    H, D = p.num_heads, 128
    rng = np.random.default_rng(seed)
    tok = p.tokens
    t0 = p.first_target
    sched = p.schedule
    cap = max(p.capacity, 1)
    # dense cache of scales < t0 and the activation pack (not timed: install-like preparation)
    ld = int(p.ranges[t0][0])
    dense_k = rng.standard_normal((batch, H * ld, D), dtype=np.float32)
    dense_v = rng.standard_normal((batch, H * ld, D), dtype=np.float32)
    slab_k = np.zeros((batch, cap, D), np.float32)
    slab_v = np.zeros((batch, cap, D), np.float32)
    items = [(s["offset"], s["head"] * ld + s["scale_start"], s["length"])
             for s in sched["segments_by_target"][t0]]
    if items:
        a = np.array(items)
        pack_flat_segments(slab_k, slab_v, dense_k, dense_v, a[:, 0], a[:, 1], a[:, 2])
    flops = 0
    elapsed = 0.0
    from heatkv_b200.scheduler import copy_descriptors
    for t in layer_targets:
        n = tok[t]
        q, k, v = (rng.standard_normal((batch, H, n, D), dtype=np.float32) for _ in range(3))
        st, en, ct = sched["metadata_cpu_by_target"][t]
        t1 = time.perf_counter()
        segmented_attention(q=q, persisted_k=slab_k, persisted_v=slab_v, segment_starts=st,
                            segment_ends=en, segment_counts=ct, current_k=k, current_v=v,
                            softmax_scale=D ** -0.5, compute_dtype=np.float32)
        if t + 1 < p.num_scales:
            d = copy_descriptors(sched["append_runs_by_key"].get((t, t + 1), []))
            if d is not None:
                pack_flat_segments(slab_k, slab_v, k.reshape(batch, H * n, D),
                                   v.reshape(batch, H * n, D), d["dst_starts"], d["src_starts"],
                                   d["lengths"])
        elapsed += time.perf_counter() - t1
        flops += 4 * n * int((p.attention_slots(t) + n).sum()) * D * batch
    del torch
    return elapsed, flops


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:  # pragma: no cover
        pass
    return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> None:
    """``--impl reference``: the reference's CPU algorithm (oracle port), rank 0 only."""
    if rank != 0:
        return
    import torch  # noqa: F401  (same interpreter state as the GPU arm)
    from heatkv_b200.hotpath import LayerPlan
    ctrl, layers, heads = build_controller(args.model, args.budget)
    plan = LayerPlan(ctrl, 0, heads, "cpu")
    targets = list(range(plan.first_target, plan.num_scales))[: args.ref_targets]
    total_flops = image_flops(ctrl, layers, heads, args.rows)
    times = []
    for i in range(args.warmup + args.steps):
        sec, flops = cpu_sample(plan, args.rows, targets, seed=i)
        if i >= args.warmup:
            times.append((sec, flops))
    sec = sum(t for t, _ in times)
    flops = sum(f for _, f in times)
    tflops = flops / sec / 1e12
    ms_image = total_flops / (tflops * 1e12) * 1e3 / (args.rows / 2)
    sample = (f"layer 0 of {args.model.upper()}, targets {targets[0]}..{targets[-1]} "
              f"(fused slab scales), {args.rows} rows, fp32 numpy/BLAS attention + pack")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tflops, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec / len(times) * 1e3, 3),
        "ms_per_image": round(ms_image, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows_per_gpu": args.rows, "budget": args.budget},
        "cpu_baseline": {"value": round(tflops, 4), "unit": "TFLOP/s", "cores": cpu_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(tflops, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def image_flops(ctrl, layers, heads, rows) -> float:
    """Algorithmic attention FLOPs of one step (all layers, all scales) for ``rows`` rows."""
    from heatkv_b200.hotpath import LayerPlan
    total = 0.0
    for l in range(layers):
        p = LayerPlan(ctrl, l, heads, "cpu")
        for t in range(p.num_scales):
            n = p.tokens[t]
            total += 4.0 * n * float((p.attention_slots(t) + n).sum()) * 128 * rows
    return total


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------

class _Workload:
    """What one rank runs per step: its launch list, the buffers copied in the e2e leg, and the
    work counted for the JSON line."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def _image_workload(args, ctrl, layers, heads, rank, world, dev):
    """Default: every rank runs its own image (``--rows`` rows) - weak scaling, no collective."""
    import torch

    from heatkv_b200.hotpath import HotPath, allocate_io
    hot = HotPath(ctrl, layers, heads, args.rows, dev, torch.bfloat16, torch.bfloat16)
    inputs, outputs, in_bufs, out_buf = allocate_io(hot, seed=1000 + rank)
    launches = hot.launches(inputs, outputs)
    att = sum(l.work for l in launches if l.kind == "attention")
    return _Workload(
        engine=hot, launches=launches, keep=(inputs, outputs), in_bufs=in_bufs, out_buf=out_buf,
        att_flops=att, job_flops=att * world, images=args.rows / 2 * world, scaling="weak",
        rows_label={"rows_per_gpu": args.rows}, slab_bytes=hot.slab_bytes(), plan=None)


def _sharded_workload(args, ctrl, layers, heads, rank, world, dev):
    """``--shard``: one fixed batch of ``--global-rows`` rows split over the ranks by (row, head)
    units (``heatkv_b200.sharding``); after every attention the rank blocks are all-gathered
    over NCCL and reassembled, so each rank holds the full output - strong scaling."""
    import torch

    from heatkv_b200 import sharding
    from heatkv_b200.hotpath import allocate_io
    costs = sharding.head_costs(ctrl, layers, heads)
    plan = sharding.plan_shards(costs, args.global_rows, world, split=args.shard)
    sh = sharding.ShardedHotPath(ctrl, layers, heads, plan, rank, dev, torch.bfloat16,
                                 torch.bfloat16, gather=True, exchange=args.exchange)
    inputs, outputs, in_bufs, _ = allocate_io(sh.local, seed=1000 + rank)
    # the full [B, n_t, H * D] outputs every rank receives
    full, full_buf = sh.allocate_full_outputs(args.global_rows, heads)
    gbuf = sh.allocate_gather_buffer()
    launches = sh.launches(inputs, outputs, full, gbuf)
    att = sum(l.work for l in launches if l.kind == "attention")
    job = image_flops(ctrl, layers, heads, args.global_rows)
    return _Workload(
        engine=sh.local, launches=launches, keep=(inputs, outputs, full, gbuf), in_bufs=in_bufs,
        out_buf=full_buf if rank == 0 else None, att_flops=att, job_flops=job,
        images=args.global_rows / 2, scaling="strong", close=sh.close,
        rows_label={"global_rows": args.global_rows, "shard": args.shard,
                    "exchange": args.exchange,
                    "row_groups": plan.row_groups, "head_groups": plan.head_groups,
                    "head_imbalance": round(plan.imbalance(costs), 4)},
        slab_bytes=sh.local.slab_bytes(), plan=plan)


def run_gpu(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from heatkv_b200 import _native
    from heatkv_b200.hotpath import HotPath

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    peaks, peak_src = load_peaks()
    ctrl, layers, heads = build_controller(args.model, args.budget)
    make = _image_workload if args.shard == "image" else _sharded_workload
    wl = make(args, ctrl, layers, heads, rank, world, dev)
    hot, launches = wl.engine, wl.launches
    n_att = sum(1 for l in launches if l.kind == "attention")
    att_flops = wl.att_flops
    pack_bytes = sum(l.work for l in launches if l.kind == "pack")
    n_own = sum(1 for l in launches if l.kind in ("attention", "pack", "gather", "barrier"))

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            hot.run(launches, stream)
    stream.synchronize()

    # The timed steps replay one CUDA graph of the step's launches. A second set of graphs, with
    # external timing events around every launch, is replayed after the timed region for the
    # per-kernel figures (the events cost ~1 us per launch, so they stay out of `value`).
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=stream):
        hot.run(launches, stream)
    graphs, ev_sets = [], []
    mk = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
    timed_kinds = ("attention", "pack")
    for _ in range(args.steps):
        evs = [(mk(), mk()) if l.kind in timed_kinds else None for l in launches]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            hot.run(launches, stream, evs)
        graphs.append(g)
        ev_sets.append(evs)
    for i in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize(dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk, torch.cuda.stream(stream):
        start.record(stream)
        for i in range(args.steps):
            step_graph.replay()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    step_ms = start.elapsed_time(end) / args.steps
    # attribution pass: the same steps with per-launch events
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for g in graphs:
            g.replay()
        a1.record(stream)
        a1.synchronize()
    step_ms_events = a0.elapsed_time(a1) / args.steps
    att_ms, pack_ms = 0.0, 0.0
    by_target = [0.0] * hot.num_scales
    for i in range(args.steps):
        for launch, ev in zip(launches, ev_sets[i]):
            if ev is None:
                continue
            d = ev[0].elapsed_time(ev[1])
            if launch.kind == "attention":
                att_ms += d
                by_target[launch.target] += d / args.steps
            else:
                pack_ms += d
    att_ms /= args.steps
    pack_ms /= args.steps
    status = _native.device_status(dev)

    # e2e: pinned host inputs -> device, every launch through the C ABI, outputs -> host
    in_bufs, out_buf = wl.in_bufs, wl.out_buf
    e2e_steps = 0 if args.no_e2e else max(1, min(args.steps, args.e2e_steps))
    h_in = [torch.empty_like(b, device="cpu").pin_memory() for b in in_bufs] if e2e_steps else []
    for hb, db in zip(h_in, in_bufs):
        hb.copy_(db)
    h_out = (torch.empty_like(out_buf, device="cpu").pin_memory()
             if out_buf is not None and e2e_steps else None)

    def e2e_step_serial():
        for hb, db in zip(h_in, in_bufs):
            db.copy_(hb, non_blocking=True)
        hot.run(launches, stream)
        if h_out is not None:
            h_out.copy_(out_buf, non_blocking=True)

    # Pipelined form (single-image workload): the Q/K/V of each (layer, scale) are copied on a
    # copy stream in launch order and its attention waits only for them; each output goes back
    # on a third stream as soon as its attention is done. The copy stream starts a step after
    # the previous step's compute (the device buffers are reused) and the step ends when every
    # output has landed in host memory.
    def host_view(h, d, base):
        off = (d.data_ptr() - base.data_ptr()) // d.element_size()
        return h.view(-1)[off:off + d.numel()].view(d.shape)

    def e2e_step_pipelined():
        inputs, outputs = wl.keep[0], wl.keep[1]
        copy_s.wait_stream(stream)
        handle = ctypes.c_void_p(stream.cuda_stream)
        copied = {}
        # the small scales of a layer (a leading run of targets, each under 4 MB of Q/K/V) sit
        # next to each other in the layer-major input buffers: one copy per layer and tensor
        # kind brings them all, instead of one per scale
        small = 0
        while (small < len(inputs[0])
               and sum(x.numel() * x.element_size() for x in inputs[0][small]) < (4 << 20)):
            small += 1

        def bring(key):
            # the Q/K/V of one (layer, scale), copied once, when a launch first needs them
            if key not in copied:
                i, t = key
                with torch.cuda.stream(copy_s):
                    if t < small:
                        for kind, (hb, db) in enumerate(zip(h_in, in_bufs)):
                            first, last = inputs[i][0][kind], inputs[i][small - 1][kind]
                            off = (first.data_ptr() - db.data_ptr()) // db.element_size()
                            end = ((last.data_ptr() - db.data_ptr()) // db.element_size()
                                   + last.numel())
                            db[off:end].copy_(hb[off:end], non_blocking=True)
                    else:
                        for x, hb, db in zip(inputs[i][t], h_in, in_bufs):
                            x.copy_(host_view(hb, x, db), non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_s)
                for tt in (range(small) if t < small else (t,)):
                    copied[(i, tt)] = ev
            return copied[key]

        for launch in launches:
            # an attention reads its own inputs; a pack before the attentions (dense appends)
            # reads the K/V of the layers it appends
            keys = ([(launch.layer, launch.target)] if launch.kind == "attention"
                    else list(launch.sources))
            for key in keys:
                stream.wait_event(bring(key))
            launch(handle)
            if launch.kind == "attention":
                i, t = launch.layer, launch.target
                if t < small - 1:
                    continue  # the small scales' outputs return together after the last one
                if t == small - 1:
                    first, last = outputs[i][0], outputs[i][t]
                    off = (first.data_ptr() - out_buf.data_ptr()) // out_buf.element_size()
                    end = ((last.data_ptr() - out_buf.data_ptr()) // out_buf.element_size()
                           + last.numel())
                    src, dst = out_buf[off:end], h_out.view(-1)[off:end]
                else:
                    src = outputs[i][t]
                    dst = host_view(h_out, src, out_buf)
                ev = torch.cuda.Event()
                ev.record(stream)
                d2h_s.wait_event(ev)
                with torch.cuda.stream(d2h_s):
                    dst.copy_(src, non_blocking=True)
        stream.wait_stream(d2h_s)

    pipelined = args.shard == "image" and h_out is not None
    copy_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e2e_step = e2e_step_pipelined if pipelined else e2e_step_serial

    with torch.cuda.stream(stream):
        for _ in range(2 if e2e_steps else 0):  # warm the copy engines
            e2e_step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps if e2e_steps else float("nan")
    h2d = sum(b.numel() * b.element_size() for b in in_bufs)
    d2h = out_buf.numel() * out_buf.element_size() if out_buf is not None else 0

    # max over ranks of the step times, sum of work
    vals = torch.tensor([step_ms, e2e_ms, att_ms, pack_ms, float(status)], dtype=torch.float64,
                        device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms, att_ms_max, pack_ms_max, status = vals.tolist()
    # graphs that hold NCCL work are released before the process group goes away
    del graphs, ev_sets, step_graph
    torch.cuda.synchronize(dev)
    if getattr(wl, "close", None) is not None:
        wl.close()   # collective: peer-shared buffers are unmapped and freed on every rank
    if rank != 0:
        return

    tflops = wl.job_flops / (step_ms * 1e-3) / 1e12
    e2e_tflops = wl.job_flops / (e2e_ms * 1e-3) / 1e12 if e2e_steps else None
    att_achieved = att_flops / (att_ms * 1e-3) / 1e12
    sustained = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    burst = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    pack_achieved = pack_bytes / (pack_ms * 1e-3) / 1e9 if pack_ms > 0 else None

    # CPU baseline (rank 0, N = 1 only): the oracle on a bounded sample
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from heatkv_b200.hotpath import LayerPlan
        sec = flops = 0.0
        for layer in range(args.ref_layers):
            plan = LayerPlan(ctrl, layer, heads, "cpu")
            targets = list(range(plan.first_target, plan.num_scales))[: args.ref_targets]
            s_, f_ = cpu_sample(plan, args.rows, targets, seed=layer)
            sec += s_
            flops += f_
        cpu = {"value": round(flops / sec / 1e12, 4), "unit": "TFLOP/s", "cores": cpu_threads(),
               "kind": "port",
               "sample": (f"layers 0..{args.ref_layers - 1}, up to {args.ref_targets} fused slab "
                          f"targets each, {args.rows} rows, fp32 numpy/BLAS oracle, "
                          f"{flops / 1e12:.2f} TFLOP in {sec:.1f} s")}

    config = {"workload": WORKLOAD if args.shard == "image" else WORKLOAD_SHARDED,
              **wl.rows_label, "budget": args.budget, "images_per_step": wl.images,
              "l2": "inputs 8.3 GB per image > 126 MB L2",
              "mode": "cuda-graph replay, one graph per timed step",
              "attention_tflop_per_step_per_gpu": round(att_flops / 1e12, 4),
              "pack_gb_per_step_per_gpu": round(pack_bytes / 1e9, 4),
              "slab_gb_per_gpu": round(wl.slab_bytes / 1e9, 3)}
    line = {
        "metric": METRIC, "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "ms_per_image": round(step_ms / wl.images * (world if wl.scaling == "weak" else 1), 3),
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config,
        "roofline": {"bound": "tensor", "achieved": round(att_achieved, 1),
                     "peak": sustained, "unit": "TFLOP/s",
                     "frac": round(att_achieved / sustained, 4),
                     # DRAM bytes of one target-12 launch (the largest share of the step) from an
                     # ncu capture of that shape (read + write)
                     "traffic": 124575232, "traffic_launch": "target 12 (Lq 4096, 2 rows x 16 heads)",
                     "peak_kind": f"bf16_tflops_sustained ({peak_src})",
                     "frac_of_burst": round(att_achieved / burst, 4),
                     "kernel": "attn_sm100_cs64_kernel", "launches_per_step": n_att,
                     "ms_per_step": round(att_ms, 3),
                     "step_ms_with_launch_events": round(step_ms_events, 3),
                     "ms_by_target": [round(x, 3) for x in by_target]},
        "roofline_pack": {"bound": "hbm", "achieved": round(pack_achieved, 1) if pack_achieved else None,
                          "peak": hbm, "unit": "GB/s",
                          "frac": round(pack_achieved / hbm, 4) if pack_achieved else None,
                          "kernel": "pack_kv_batched_kernel", "ms_per_step": round(pack_ms, 3),
                          # ncu capture of one scale's appends for 32 layers (604 MB algorithmic)
                          "traffic": 558111000, "traffic_launch": "32-layer append of a 576-token scale",
                          "launches_per_step": sum(1 for l in launches if l.kind == "pack")},
        "cpu_baseline": cpu,
        "e2e": None if not e2e_steps else {"value": round(e2e_tflops, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "path": ("C ABI, inputs from pinned host memory, outputs back to host"
                         + (", copies pipelined per (layer, scale), the small scales of a layer in one copy each way" if pipelined else ""))},
        "clocks": clk.summary(),
        "gpu_launches": n_own * args.steps,
        "device_status": int(status),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description="HeatKV hot-path benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["heatkv", "reference"], default="heatkv")
    ap.add_argument("--model", choices=["2b", "8b"], default="2b")
    ap.add_argument("--budget", type=float, default=0.10)
    ap.add_argument("--rows", type=int, default=2, help="batch rows per GPU (image + CFG = 2)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-memory leg (for configurations too large to pin on the host)")
    ap.add_argument("--ref-targets", type=int, default=5,
                    help="fused targets in the CPU sample (bounds the CPU time)")
    ap.add_argument("--ref-layers", type=int, default=3,
                    help="layers in the cpu_baseline sample of the GPU arm (about 4 s each)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", choices=["image", "auto", "rows", "heads"], default="image",
                    help="image: each GPU runs its own image (weak scaling); auto/rows/heads: "
                         "one batch of --global-rows rows sharded over the GPUs (strong scaling)")
    ap.add_argument("--global-rows", type=int, default=2)
    ap.add_argument("--exchange", choices=["nccl", "p2p"], default="p2p",
                    help="sharded modes: NCCL all-gather + reassembly, or the attention kernel "
                         "storing into every rank's output over NVLink + a peer barrier")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch.distributed as dist
    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
