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
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

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

def run_gpu(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from heatkv_b200 import _native
    from heatkv_b200.hotpath import HotPath, allocate_io

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    peaks, peak_src = load_peaks()
    ctrl, layers, heads = build_controller(args.model, args.budget)
    hot = HotPath(ctrl, layers, heads, args.rows, dev, torch.bfloat16, torch.bfloat16)
    inputs, outputs, in_bufs, out_buf = allocate_io(hot, seed=1000 + rank)
    launches = hot.launches(inputs, outputs)
    n_att = sum(1 for l in launches if l.kind == "attention")
    att_flops = sum(l.work for l in launches if l.kind == "attention")
    pack_bytes = sum(l.work for l in launches if l.kind == "pack")

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            hot.run(launches, stream)
    stream.synchronize()

    # one graph per timed step, each with its own external timing events around every launch
    graphs, ev_sets = [], []
    mk = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
    for _ in range(args.steps + args.warmup):
        evs = [(mk(), mk()) for _ in launches]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            hot.run(launches, stream, evs)
        graphs.append(g)
        ev_sets.append(evs)
    for i in range(args.warmup):
        graphs[i].replay()
    torch.cuda.synchronize(dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk, torch.cuda.stream(stream):
        start.record(stream)
        for i in range(args.steps):
            graphs[args.warmup + i].replay()
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    step_ms = start.elapsed_time(end) / args.steps
    att_ms, pack_ms = 0.0, 0.0
    by_target = [0.0] * hot.num_scales
    for i in range(args.steps):
        for launch, (e0, e1) in zip(launches, ev_sets[args.warmup + i]):
            d = e0.elapsed_time(e1)
            if launch.kind == "attention":
                att_ms += d
                by_target[launch.target] += d / args.steps
            else:
                pack_ms += d
    att_ms /= args.steps
    pack_ms /= args.steps
    status = _native.device_status(dev)

    # e2e: pinned host inputs -> device, every launch through the C ABI, outputs -> host
    h_in = [torch.empty_like(b, device="cpu").pin_memory() for b in in_bufs]
    for hb, db in zip(h_in, in_bufs):
        hb.copy_(db)
    h_out = torch.empty_like(out_buf, device="cpu").pin_memory()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    with torch.cuda.stream(stream):
        for _ in range(2):  # warm the copy engines
            for hb, db in zip(h_in, in_bufs):
                db.copy_(hb, non_blocking=True)
            hot.run(launches, stream)
            h_out.copy_(out_buf, non_blocking=True)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            for hb, db in zip(h_in, in_bufs):
                db.copy_(hb, non_blocking=True)
            hot.run(launches, stream)
            h_out.copy_(out_buf, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = sum(b.numel() * b.element_size() for b in in_bufs)
    d2h = out_buf.numel() * out_buf.element_size()

    # max over ranks of the step times, sum of work
    vals = torch.tensor([step_ms, e2e_ms, att_ms, pack_ms, float(status)], dtype=torch.float64,
                        device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms, att_ms_max, pack_ms_max, status = vals.tolist()
    if rank != 0:
        return

    tflops = att_flops * world / (step_ms * 1e-3) / 1e12
    e2e_tflops = att_flops * world / (e2e_ms * 1e-3) / 1e12
    images_per_step = args.rows / 2 * world
    att_achieved = att_flops / (att_ms * 1e-3) / 1e12
    sustained = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    burst = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    pack_achieved = pack_bytes / (pack_ms * 1e-3) / 1e9 if pack_ms > 0 else None

    # CPU baseline (rank 0, N = 1 only): the oracle on a bounded sample
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from heatkv_b200.hotpath import LayerPlan
        plan = LayerPlan(ctrl, 0, heads, "cpu")
        targets = list(range(plan.first_target, plan.num_scales))[: args.ref_targets]
        sec, flops = cpu_sample(plan, args.rows, targets)
        cpu = {"value": round(flops / sec / 1e12, 4), "unit": "TFLOP/s", "cores": cpu_threads(),
               "kind": "port",
               "sample": (f"layer 0, targets {targets[0]}..{targets[-1]} (fused slab scales), "
                          f"{args.rows} rows, fp32 numpy/BLAS oracle, {sec:.1f} s")}

    line = {
        "metric": METRIC, "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "ms_per_image": round(step_ms / (args.rows / 2), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows_per_gpu": args.rows, "budget": args.budget,
                   "images_per_step": images_per_step, "l2": "inputs 8.3 GB per step > 126 MB L2",
                   "mode": "cuda-graph replay, one graph per timed step",
                   "attention_tflop_per_step_per_gpu": round(att_flops / 1e12, 4),
                   "pack_gb_per_step_per_gpu": round(pack_bytes / 1e9, 4),
                   "slab_gb_per_gpu": round(hot.slab_bytes() / 1e9, 3)},
        "roofline": {"bound": "tensor", "achieved": round(att_achieved, 1),
                     "peak": sustained, "unit": "TFLOP/s",
                     "frac": round(att_achieved / sustained, 4), "traffic": None,
                     "peak_kind": f"bf16_tflops_sustained ({peak_src})",
                     "frac_of_burst": round(att_achieved / burst, 4),
                     "kernel": "attn_sm100_kernel", "launches_per_step": n_att,
                     "ms_per_step": round(att_ms, 3),
                     "ms_by_target": [round(x, 3) for x in by_target]},
        "roofline_pack": {"bound": "hbm", "achieved": round(pack_achieved, 1) if pack_achieved else None,
                          "peak": hbm, "unit": "GB/s",
                          "frac": round(pack_achieved / hbm, 4) if pack_achieved else None,
                          "kernel": "pack_kv_kernel", "ms_per_step": round(pack_ms, 3),
                          "launches_per_step": len(launches) - n_att},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_tflops, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "path": "C ABI, inputs from pinned host memory, outputs back to host"},
        "clocks": clk.summary(),
        "gpu_launches": len(launches) * args.steps,
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
    ap.add_argument("--ref-targets", type=int, default=5,
                    help="fused targets in the CPU sample (bounds the CPU time)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
