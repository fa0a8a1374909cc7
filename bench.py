#!/usr/bin/env python
"""Benchmark of the HeatKV hot path on B200: segmented attention + slab compaction.

Default workload (``--workload c5``, BASELINE.json configs[4], the metric's "at 1/2/4/8 GPU"
configuration): Infinity-2B at 1024x1024 - 32 layers x 16 heads x head_dim 128, 13 scales (10,521
tokens), batch 32 doubled to 64 rows for CFG, keep-mask of the 10 % budget from orders/2b.json
(strict schedule, 3 protected scales, source scales 3..11). Every (scale, layer) generates its
Q/K/V on the device from random-init N(0, 0.02) Infinity-2B QKV weights (``heatkv_b200.projected``:
projection GEMM, cos-attention normalisation and 2-D RoPE with the early cache appends, then the
segmented attention and the rest of the compaction). The layer inputs are seeded N(0, 1) per row.
With N GPUs the 64 rows are sharded over the ranks by the (row, head) planner
(``heatkv_b200.sharding``), rows only when they divide: every output row is then used on the GPU
that computed it, so no exchange is needed (strong scaling: the total work is fixed).

``--workload c2``: one image (2 rows) of pre-generated N(0, 1) bf16 Q/K/V per
(layer, scale); ``--shard`` splits one batch over the GPUs by (row, head) with an output exchange.

One step = the whole workload once (every layer and scale). The step is replayed as a CUDA graph;
a second set of graphs with timing events around every launch gives the per-kernel figures.
Output: one JSON line (rank 0). ``value`` = algorithmic attention TFLOP/s of the whole job
(attention FLOPs of all ranks / max over ranks of the step time, the step including the QKV
generation), ``ms_per_image`` beside it; ``roofline`` for the attention kernel (tensor-bound),
``roofline_pack`` for compaction and ``roofline_prep`` for the preparation (HBM-bound);
``e2e`` = the same step with the layer inputs copied from pinned host memory and the step's
outputs copied back; ``cpu_baseline`` = the reference's CPU path restated in torch CPU fp32
(``oracle/bench_sample.py``) on a bounded sample. ``--impl reference`` times that CPU path alone,
on the same sample, without loading any code of ``heatkv_b200``.
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
WORKLOAD_C5 = ("configs[4]: Infinity-2B at 1024^2 - 32 layers x 16 heads x 128, 13 scales, "
               "batch 32 + CFG = 64 rows, 10% budget from orders/2b.json; Q/K/V generated per "
               "(layer, scale) from random-init N(0, 0.02) QKV weights (cos-attention, 2-D RoPE); "
               "rows sharded over the GPUs")
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
# CPU baseline and reference arm: the reference's CPU path restated in torch CPU fp32 on the slab
# schedule recorded from the reference (oracle/bench_sample.py) - no code of heatkv_b200 loads
# ------------------------------------------------------------------------------------------------

def config_of(args) -> dict:
    """The ``config`` object of the JSON line, identical in both arms (derived from the command
    line only)."""
    if args.workload == "c5":
        return {"workload": WORKLOAD_C5, "global_rows": args.global_rows, "budget": args.budget,
                "qkv": "generated on the device every step (projection + cos-norm + RoPE)",
                "l2": "inputs and caches far larger than the 126 MB L2"}
    if args.shard == "image":
        return {"workload": WORKLOAD, "rows_per_gpu": args.rows, "budget": args.budget,
                "l2": "inputs 8.3 GB per image > 126 MB L2"}
    return {"workload": WORKLOAD_SHARDED, "global_rows": args.global_rows, "shard": args.shard,
            "exchange": args.exchange, "budget": args.budget,
            "l2": "inputs 8.3 GB per image > 126 MB L2"}


def cpu_baseline_sample(args):
    """The bounded CPU sample both arms time: the first ``--ref-targets`` fused targets of layers
    ``0..--ref-layers-1``, 2 rows (one image), with the projection when the workload has it.
    Returns ``(seconds, flops, description)``."""
    from oracle.bench_sample import cpu_sample
    return cpu_sample(layers=tuple(range(args.ref_layers)), n_targets=args.ref_targets, rows=2,
                      model=args.model, budget=args.budget, project=args.workload == "c5")


def cpu_baseline_line(args, world: int):
    """The GPU arm's ``cpu_baseline`` object (rank 0 at N = 1 only, unless disabled)."""
    if world != 1 or args.no_cpu_baseline:
        return None
    import torch
    sec, flops, desc = cpu_baseline_sample(args)
    return {"value": round(flops / sec / 1e12, 4), "unit": "TFLOP/s",
            "cores": int(torch.get_num_threads()), "kind": "port", "sample": desc}


def run_reference(args, rank: int, world: int) -> None:
    """``--impl reference``: the reference's CPU path (restated in torch CPU fp32), rank 0 only;
    each warm-up and timed step runs the same bounded sample as the GPU arm's ``cpu_baseline``."""
    if rank != 0:
        return
    import torch

    from oracle.bench_sample import image_attention_flops
    times = []
    desc = ""
    for i in range(args.warmup + args.steps):
        sec, flops, desc = cpu_baseline_sample(args)
        if i >= args.warmup:
            times.append((sec, flops))
    sec = sum(t for t, _ in times)
    flops = sum(f for _, f in times)
    tflops = flops / sec / 1e12
    ms_image = image_attention_flops(rows=2, model=args.model, budget=args.budget) / (
        tflops * 1e12) * 1e3
    leaked = [m for m in _loaded_native() if "heatkv" in m]
    if leaked:
        raise SystemExit(f"reference arm loaded native code of this repository: {leaked}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tflops, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec / len(times) * 1e3, 3),
        "ms_per_image": round(ms_image, 1), "higher_is_better": True,
        "scaling": "strong" if args.workload == "c5" or args.shard != "image" else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args),
        "cpu_baseline": {"value": round(tflops, 4), "unit": "TFLOP/s",
                         "cores": int(torch.get_num_threads()), "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(tflops, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _loaded_native():
    """Shared objects mapped into this process (Linux), for the reference arm's self-check."""
    try:
        with open("/proc/self/maps") as fh:
            return sorted({l.split()[-1] for l in fh if l.rstrip().endswith(".so")})
    except OSError:
        return []


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

    cpu = cpu_baseline_line(args, world)
    config = config_of(args)
    details = {**wl.rows_label, "images_per_step": wl.images,
               "mode": "cuda-graph replay, one graph per timed step",
               "attention_tflop_per_step_per_gpu": round(att_flops / 1e12, 4),
               "pack_gb_per_step_per_gpu": round(pack_bytes / 1e9, 4),
               "slab_gb_per_gpu": round(wl.slab_bytes / 1e9, 3)}
    line = {
        "metric": METRIC, "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "ms_per_image": round(step_ms / wl.images * (world if wl.scaling == "weak" else 1), 3),
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config, "details": details,
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


def _timed_replays(graph, steps, stream, dev, world, local_rank):
    """Replay ``graph`` ``steps`` times between CUDA events on ``stream`` (barrier + synchronise
    before), sampling the clocks meanwhile. Returns (ms per step, clock summary)."""
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk, torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    return start.elapsed_time(end) / steps, clk.summary()


def _attribution(proj, launches, stream, steps, kinds):
    """Per-launch CUDA-event times (ms per step, summed by kind and by (kind, target)) from
    ``steps`` replays of graphs that bracket every launch with external events."""
    import torch
    mk = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
    graphs, ev_sets = [], []
    for _ in range(steps):
        evs = [(mk(), mk()) if l.kind in kinds else None for l in launches]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            proj.run(launches, stream, evs)
        graphs.append(g)
        ev_sets.append(evs)
    with torch.cuda.stream(stream):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for g in graphs:
            g.replay()
        a1.record(stream)
        a1.synchronize()
    by_kind, by_target = {k: 0.0 for k in kinds}, {}
    for evs in ev_sets:
        for launch, ev in zip(launches, evs):
            if ev is None:
                continue
            d = ev[0].elapsed_time(ev[1]) / steps
            by_kind[launch.kind] += d
            key = (launch.kind, launch.target)
            by_target[key] = by_target.get(key, 0.0) + d
    del graphs
    return by_kind, by_target, a0.elapsed_time(a1) / steps


def c2_history(args, dev, peaks):
    """configs[1] (one 2-row image of pre-generated Q/K/V, the previous headline) on this GPU: a
    short graph-replay timing kept beside the main line so results stay comparable over time."""
    import torch

    from heatkv_b200.hotpath import HotPath, allocate_io
    ctrl, layers, heads = build_controller(args.model, args.budget)
    hot = HotPath(ctrl, layers, heads, 2, dev, torch.bfloat16, torch.bfloat16)
    inputs, outputs, _, _ = allocate_io(hot, seed=1000)
    launches = hot.launches(inputs, outputs)
    att = sum(l.work for l in launches if l.kind == "attention")
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            hot.run(launches, stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        hot.run(launches, stream)
    for _ in range(3):
        g.replay()
    ms, _ = _timed_replays(g, max(5, args.steps), stream, dev, 1, dev.index)
    by_kind, _, _ = _attribution(hot, launches, stream, 1, ("attention", "pack"))
    sustained = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    out = {"workload": WORKLOAD, "value": round(att / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "ms_per_image": round(ms, 3),
           "attention_frac_of_sustained": round(att / (by_kind["attention"] * 1e-3) / 1e12
                                                / sustained, 4)}
    del g, inputs, outputs, hot
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return out


def apply_rotary_emb(q, k, scale_schedule, rope2d_freqs_grid, pad_to_multiplier,
                     rope2d_normalized_by_hw, scale_ind):
    """Infinity's 2-D rotary embedding (infinity/models/basic.py:97-117) beside the stand-in
    attention module below: the installer looks it up in the module's defining Python module."""
    import torch
    qk = torch.stack((q, k), dim=0)
    with torch.autocast(device_type="cuda", enabled=False):
        seq_len = qk.shape[3]
        start = sum(a * b * c for a, b, c in scale_schedule[:scale_ind]) if scale_ind >= 1 else 0
        cache = rope2d_freqs_grid[str(tuple(scale_schedule))][:, :, :, :, start:start + seq_len]
        qk = qk.reshape(*qk.shape[:-1], -1, 2)
        qk = torch.stack([cache[0] * qk[..., 0] - cache[1] * qk[..., 1],
                          cache[1] * qk[..., 0] + cache[0] * qk[..., 1]], dim=-1)
        q, k = qk.reshape(*qk.shape[:-2], -1).unbind(dim=0)
    return q, k


def dropin_image(args, dev):
    """One image (2 rows) through the public installer on 32 Infinity-2B-shaped self-attention
    modules (random N(0, 0.02) weights, fp32 parameters under bf16 autocast as the model runs:
    fp32 q/k after cos-attention, bf16 v), every scale's forward of every layer: QKV projection,
    fused preparation, the segmented kernel (dense prefix included) and the output projection.
    Returns the attention TFLOP/s of the image and its time."""
    import math

    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    from heatkv_b200 import budget as bud, synthetic
    from heatkv_b200.enable_real_pruning_fast import \
        enable_real_pruning_scale_specific_fused_segmented
    from oracle.bench_sample import image_attention_flops

    class SelfAttention(nn.Module):
        """The attributes and forward of infinity/models/basic.py:196-316 that the installer
        uses (cos-attention, no flash)."""

        def __init__(self, C, H):
            super().__init__()
            self.num_heads, self.head_dim, self.cos_attn, self.scale = H, C // H, True, 1
            self.scale_mul_1H11 = nn.Parameter(torch.full((1, H, 1, 1), 4.0).log())
            self.max_scale_mul = math.log(100)
            self.mat_qkv = nn.Linear(C, 3 * C, bias=False)
            self.q_bias, self.v_bias = nn.Parameter(torch.zeros(C)), nn.Parameter(torch.zeros(C))
            self.register_buffer("zero_k_bias", torch.zeros(C))
            self.proj, self.proj_drop = nn.Linear(C, C), nn.Identity()
            self.caching, self.cached_k, self.cached_v = False, None, None
            self.pad_to_multiplier, self.rope2d_normalized_by_hw = 1, 2

        def kv_caching(self, enable):
            self.caching, self.cached_k, self.cached_v = enable, None, None

        def forward(self, x, attn_bias_or_two_vector, attn_fn=None, scale_schedule=None,
                    rope2d_freqs_grid=None, scale_ind=0):
            raise NotImplementedError("replaced by the installer")

    SelfAttention.__module__ = __name__
    layers, heads, C = 32, 16, 2048
    torch.manual_seed(0)
    model = nn.ModuleList([SelfAttention(C, heads) for _ in range(layers)])
    for m in model:
        nn.init.normal_(m.mat_qkv.weight, 0.0, 0.02)
        nn.init.normal_(m.proj.weight, 0.0, 0.02)
    model = model.to(dev)
    enable_real_pruning_scale_specific_fused_segmented(
        model, args.budget, bud.orders(model_type=2), protected_prefix_scales=3,
        source_scale_start=3, fused_qkv_prep=True)
    sched = [tuple(x) for x in synthetic.SCALE_SCHEDULE_1M]
    cos, sin = synthetic.rope2d_rows()
    grid = {str(tuple(sched)): torch.stack([cos, sin])[:, None, None, None].to(dev)}
    gen = torch.Generator(device=dev).manual_seed(2)
    xs = [torch.randn(2, h * w, C, device=dev, generator=gen) for _, h, w in sched]

    def image():
        for m in model:
            m.kv_caching(True)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            for t in range(len(sched)):
                for m in model:
                    m(xs[t], None, scale_schedule=sched, rope2d_freqs_grid=grid, scale_ind=t)

    for _ in range(3):
        image()
    torch.cuda.synchronize(dev)
    n = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        image()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n
    flops = image_attention_flops(rows=2, budget=args.budget)
    del model, xs
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return {"value": round(flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_image": round(ms, 3), "images": n,
            "path": ("enable_real_pruning_scale_specific_fused_segmented(fused_qkv_prep=True) on "
                     "32 Infinity-2B-shaped self-attention modules, fp32 parameters under bf16 "
                     "autocast (fp32 q/k, bf16 v: the tf32 tcgen05 mode), eager PyTorch forward "
                     "per (scale, layer) including the QKV and output projections")}


def run_projected(args, rank: int, world: int, local_rank: int) -> None:
    """64 rows, Q/K/V generated every (layer, scale) from the QKV projection."""
    import torch
    import torch.distributed as dist

    from heatkv_b200 import _native, sharding
    from heatkv_b200.hotpath import HotPath
    from heatkv_b200.projected import ProjectedHotPath

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    peaks, peak_src = load_peaks()
    history = dropin = None
    if world == 1 and not args.no_c2_history:
        history = c2_history(args, dev, peaks)
    if world == 1 and not args.no_dropin:
        dropin = dropin_image(args, dev)
    ctrl, layers, heads = build_controller(args.model, args.budget)
    costs = sharding.head_costs(ctrl, layers, heads)
    plan = sharding.plan_shards(costs, args.global_rows, world, split=args.shard)
    rows = plan.rows_per_rank
    sh = None
    if plan.splits_heads:
        # heads split over the GPUs: each rank projects and attends its heads of its rows, and
        # every attention output is exchanged so each rank holds the full [rows, n, H * D]
        sh = sharding.ShardedHotPath(ctrl, layers, heads, plan, rank, dev, torch.bfloat16,
                                     torch.bfloat16, gather=True, exchange=args.exchange)
        hot = sh.local
        proj = ProjectedHotPath(hot, global_heads=[plan.heads_of(rank, l) for l in range(layers)],
                                embed_dim=heads * 128, weight_seed=0,
                                fused_projection=not args.unfused_projection)
    else:
        hot = HotPath(ctrl, layers, heads, rows, dev, torch.bfloat16, torch.bfloat16)
        proj = ProjectedHotPath(hot, weight_seed=0, fused_projection=not args.unfused_projection)
    x, x_flat = proj.allocate_inputs(plan.rows_of(rank), seed=1)
    out, out_flat = proj.allocate_outputs()
    launches = proj.launches(x, out)
    if sh is not None:
        full, full_flat = sh.allocate_full_outputs(plan.batch, heads, per_layer=False)
        gbuf = sh.allocate_gather_buffer()
        launches = sh.exchange(launches, out, full, gbuf)
        out, out_flat = full, full_flat   # the step's result: every rank's full outputs
    xchg_kinds = ("allgather", "gather", "barrier")
    xchg_bytes = sum(l.work for l in launches if l.kind == "allgather")
    att_flops = sum(l.work for l in launches if l.kind == "attention")
    gemm_flops = sum(l.work for l in launches if l.kind in ("gemm", "proj"))
    pack_bytes = sum(l.work for l in launches if l.kind == "pack")
    prep_bytes = sum(l.work for l in launches if l.kind == "prep")
    proj_bytes = sum(l.nbytes for l in launches if l.kind == "proj")
    n_att = sum(1 for l in launches if l.kind == "attention")
    n_own = sum(1 for l in launches if l.kind in ("attention", "pack", "prep", "proj", "gather",
                                                   "barrier"))

    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            proj.run(launches, stream)
    stream.synchronize()
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=stream):
        proj.run(launches, stream)
    step_graph.replay()       # one untimed replay of the captured step
    step_ms, clocks = _timed_replays(step_graph, args.steps, stream, dev, world, local_rank)
    if world > 1:
        dist.barrier()
    kinds = ("proj", "gemm", "prep", "attention", "pack") + xchg_kinds
    by_kind, by_target, step_ms_events = _attribution(proj, launches, stream,
                                                      max(1, args.attrib_steps), kinds)
    xchg_ms = sum(by_kind[k] for k in xchg_kinds)
    status = _native.device_status(dev)

    # e2e: the layer inputs of each scale come from pinned host memory (copy stream, in scale
    # order), the step's outputs (the last layer's attention output of every scale) go back to
    # pinned host memory (third stream) as soon as the scale's last attention is done
    e2e_steps = 0 if args.no_e2e else max(1, min(args.steps, args.e2e_steps))
    h_x = torch.empty_like(x_flat, device="cpu").pin_memory() if e2e_steps else None
    h_out = torch.empty_like(out_flat, device="cpu").pin_memory() if e2e_steps else None
    if e2e_steps:
        h_x.copy_(x_flat)
    copy_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    first_of = {}
    last_att = {}
    for j, l in enumerate(launches):
        first_of.setdefault(l.target, j)
        if l.kind == "attention":
            last_att[l.target] = j
    offs_x = [t_.data_ptr() - x_flat.data_ptr() for t_ in x]
    offs_o = [t_.data_ptr() - out_flat.data_ptr() for t_ in out]
    esz = x_flat.element_size()

    def e2e_step():
        copy_s.wait_stream(stream)          # the device buffers are reused step after step
        ready = {}
        for t in range(proj.num_scales):
            with torch.cuda.stream(copy_s):
                n = x[t].numel()
                x[t].view(-1).copy_(h_x[offs_x[t] // esz: offs_x[t] // esz + n],
                                    non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_s)
            ready[t] = ev
        for j, l in enumerate(launches):
            if first_of.get(l.target) == j:
                stream.wait_event(ready[l.target])
            proj.run([l], stream)
            if last_att.get(l.target) == j:
                t = l.target
                ev = torch.cuda.Event()
                ev.record(stream)
                d2h_s.wait_event(ev)
                with torch.cuda.stream(d2h_s):
                    n = out[t].numel()
                    h_out[offs_o[t] // esz: offs_o[t] // esz + n].copy_(out[t].view(-1),
                                                                       non_blocking=True)
        stream.wait_stream(d2h_s)

    e2e_ms = float("nan")
    if e2e_steps:
        with torch.cuda.stream(stream):
            e2e_step()                      # warm the copy engines
            stream.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(e2e_steps):
                e2e_step()
            e1.record(stream)
            e1.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = x_flat.numel() * x_flat.element_size()
    d2h = out_flat.numel() * out_flat.element_size()

    vals = torch.tensor([step_ms, e2e_ms, by_kind["attention"], by_kind["pack"], by_kind["prep"],
                         by_kind["gemm"], by_kind["proj"], xchg_ms, float(status)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms, att_ms, pack_ms, prep_ms, gemm_ms, proj_ms, xchg_ms, status = vals.tolist()
    # graphs that hold NCCL work are released before the process group goes away
    del step_graph
    torch.cuda.synchronize(dev)
    if sh is not None:
        sh.close()   # collective: peer-shared buffers are unmapped and freed on every rank
    if rank != 0:
        return

    job_att = att_flops * world
    images = args.global_rows / 2
    tflops = job_att / (step_ms * 1e-3) / 1e12
    sustained = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    burst = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    att_achieved = att_flops / (att_ms * 1e-3) / 1e12
    ms_by_target = [round(by_target.get(("attention", t), 0.0), 3)
                    for t in range(proj.num_scales)]
    line = {
        "metric": METRIC, "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "ms_per_image": round(step_ms / images, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_of(args),
        "details": {
            "rows_per_gpu": rows, "row_groups": plan.row_groups, "head_groups": plan.head_groups,
            "exchange": ({"kind": args.exchange, "ms_per_step": round(xchg_ms, 3),
                          "gb_all_gathered_per_step_per_gpu": round(xchg_bytes / 1e9, 3),
                          "head_imbalance": round(plan.imbalance(costs), 4)}
                         if sh is not None else
                         "none: rows only, every output row is used on the GPU that computed it"),
            "images_per_step": images, "mode": "cuda-graph replay of the whole step",
            "attention_tflop_per_step_per_gpu": round(att_flops / 1e12, 3),
            "qkv_gemm_tflop_per_step_per_gpu": round(gemm_flops / 1e12, 3),
            "slab_gb_per_gpu": round(hot.slab_bytes() / 1e9, 3),
            "early_append_slots_per_row": proj.early_slots,
            "pack_append_slots_per_row": proj.rest_slots,
            "qkv": ("fused: heatkv_qkv_project (tcgen05 projection, preparation and early "
                    "appends in its epilogue)" if proj.fused_projection else
                    "unfused: cuBLAS GEMM + heatkv_qkv_prepare_append"),
            "ms_by_stage": {"qkv_project_fused": round(proj_ms, 3),
                            "qkv_gemm_cublas": round(gemm_ms, 3), "prep": round(prep_ms, 3),
                            "attention": round(att_ms, 3), "pack": round(pack_ms, 3),
                            "step_with_launch_events": round(step_ms_events, 3)},
            "qkv_projection_tflops": round(gemm_flops / ((gemm_ms + proj_ms) * 1e-3) / 1e12, 1),
            "configs1_image": history,
            "dropin_image": dropin,
        },
        "roofline": {"bound": "tensor", "achieved": round(att_achieved, 1), "peak": sustained,
                     "unit": "TFLOP/s", "frac": round(att_achieved / sustained, 4),
                     "traffic": round(args.att_traffic_per_row * rows),
                     "traffic_launch": ("target 12 (Lq 4096): ncu DRAM read + write of the 8-row "
                                        "launch, scaled by rows to this GPU's rows"),
                     "peak_kind": f"bf16_tflops_sustained ({peak_src})",
                     "frac_of_burst": round(att_achieved / burst, 4),
                     "kernel": "attn_sm100_cs64_kernel", "launches_per_step": n_att,
                     "ms_per_step": round(att_ms, 3), "ms_by_target": ms_by_target},
        "roofline_pack": {"bound": "hbm", "peak": hbm, "unit": "GB/s",
                          "achieved": round(pack_bytes / (pack_ms * 1e-3) / 1e9, 1),
                          "frac": round(pack_bytes / (pack_ms * 1e-3) / 1e9 / hbm, 4),
                          "kernel": "pack_kv_kernel / pack_kv_batched_kernel",
                          "ms_per_step": round(pack_ms, 3),
                          "gb_per_step": round(pack_bytes / 1e9, 3),
                          "launches_per_step": sum(1 for l in launches if l.kind == "pack")},
        "roofline_qkv": ({"bound": "tensor", "peak": sustained, "unit": "TFLOP/s",
                          "achieved": round(gemm_flops / (proj_ms * 1e-3) / 1e12, 1),
                          "frac": round(gemm_flops / (proj_ms * 1e-3) / 1e12 / sustained, 4),
                          "kernel": "qkv_project_pair_kernel", "ms_per_step": round(proj_ms, 3),
                          "hbm_gb_per_step": round(proj_bytes / 1e9, 3)}
                         if proj.fused_projection else
                         {"bound": "hbm", "peak": hbm, "unit": "GB/s",
                          "achieved": round(prep_bytes / (prep_ms * 1e-3) / 1e9, 1),
                          "frac": round(prep_bytes / (prep_ms * 1e-3) / 1e9 / hbm, 4),
                          "kernel": "qkv_prepare_kernel (after a cuBLAS GEMM)",
                          "ms_per_step": round(prep_ms, 3),
                          "gb_per_step": round(prep_bytes / 1e9, 3)}),
        "cpu_baseline": cpu_baseline_line(args, world),
        "e2e": None if not e2e_steps else {
            "value": round(job_att / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
            "path": ("eager launches through the C ABI; layer inputs of every scale from pinned "
                     "host memory, the last layer's attention outputs back to pinned host memory, "
                     "copies on their own streams overlapping the compute")},
        "clocks": clocks,
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
    ap.add_argument("--workload", choices=["c5", "c2"], default="c5",
                    help="c5: configs[4] (64 rows, Q/K/V from the QKV projection); c2: configs[1] "
                         "(one 2-row image of pre-generated Q/K/V)")
    ap.add_argument("--ref-targets", type=int, default=5,
                    help="fused targets per layer in the CPU sample (bounds the CPU time)")
    ap.add_argument("--ref-layers", type=int, default=2,
                    help="layers in the CPU sample (both arms)")
    ap.add_argument("--attrib-steps", type=int, default=1,
                    help="replays of the per-launch event graphs for the per-kernel figures")
    ap.add_argument("--no-c2-history", action="store_true",
                    help="skip the configs[1] timing kept beside the configs[4] line")
    ap.add_argument("--unfused-projection", action="store_true",
                    help="configs[4]: cuBLAS GEMM + heatkv_qkv_prepare_append instead of the fused "
                         "heatkv_qkv_project")
    ap.add_argument("--no-dropin", action="store_true",
                    help="skip the one-image timing through the public installer")
    ap.add_argument("--att-traffic-per-row", type=float, default=569.9e6 / 8,
                    help="DRAM bytes per batch row of the target-12 attention launch (ncu capture "
                         "at 8 rows, profiles/attn_sm100_cs64_kernel_2b_q4096_rows8.md)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", choices=["image", "auto", "rows", "heads"], default="image",
                    help="image: each GPU runs its own image (weak scaling); auto/rows/heads: "
                         "one batch of --global-rows rows sharded over the GPUs (strong scaling)")
    ap.add_argument("--global-rows", type=int, default=None,
                    help="rows of the whole job (default 64 for c5, 2 for a sharded c2)")
    ap.add_argument("--exchange", choices=["nccl", "p2p"], default="p2p",
                    help="sharded modes: NCCL all-gather + reassembly, or the attention kernel "
                         "storing into every rank's output over NVLink + a peer barrier")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.global_rows is None:
        args.global_rows = 64 if args.workload == "c5" else 2
    if args.workload == "c5" and args.shard == "image":
        args.shard = "auto"
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
        if args.workload == "c5":
            run_projected(args, rank, world, local_rank)
        else:
            run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
