"""Generate the golden fixtures under tests/golden/ by running the HeatKV reference itself.

This script is test infrastructure. It is run by hand, in a container that holds a
read-only checkout of the reference (``--reference PATH``); its outputs are committed so
the tests never need the reference at run time.

What it records (every value comes from the reference's own Python functions):

* ``budget_<cfg>.npz`` - the keep-mask policy: ``strict_removed_heads_by_scale_specific_for_budget``
  (tools/utils.py:525-597) as a uint8 mask ``removed[target, source-3, layer, head]`` plus the
  per-target removed counts.
* ``schedule_<cfg>.npz`` - per layer, the static slab schedule of
  ``_segmented_flat_build_static_slot_schedule`` (enable_real_pruning_fast.py:260-558):
  capacities, allocated segments, per-target ``[H, S]`` segment metadata and the flattened copy
  descriptors (``dst_start, src_start, length``) that ``_segmented_flat_static_copy_metadata_for_runs``
  (enable_real_pruning_fast.py:610-671) would upload.
* ``pack_c1.npz`` - SHA-256 digests of the K/V slab bytes after the activation pack and after
  each per-scale append of config 1, produced by the reference's CPU copy path
  (``_segmented_flat_static_copy_precomputed_runs``, enable_real_pruning_fast.py:763-869).
* ``attention_cases.npz`` - outputs of the reference's CPU attention oracle
  ``_flat_segmented_attention_reference`` (real_pruning_fused_attention.py:312-361) on small
  seeded cases, including empty segments, zero-count heads and an empty slab.
* ``attention_c1.npz`` - per fused call of the config-1 pipeline: the reference oracle's
  output checksums plus its first rows verbatim.
* ``scas_c1.npz`` - the reference's S-CAS ``ScasAccumulator`` (tools/compute_scas.py:92-152) on
  the 7-scale schedule, fed the capture forward's fp32 probabilities of seeded cos-attention-like
  q/k (``synthetic.scas_inputs``): ``accum``, ``scores`` and ``orders``.

Inputs are generated with ``heatkv_b200.synthetic`` so the tests regenerate the identical tensors.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from heatkv_b200 import synthetic  # noqa: E402


def _install_import_stubs() -> None:
    """The reference's package imports pull in timm and pytz at module level; neither is used
    on the code paths exercised here, so empty stand-ins are enough to import it."""

    def stub(name, **attrs):
        mod = types.ModuleType(name)
        mod.__path__ = []
        mod.__dict__.update(attrs)
        sys.modules.setdefault(name, mod)

    class _Identity(torch.nn.Module):
        def __init__(self, *args, **kwargs):
            super().__init__()

        def forward(self, x):
            return x

    stub("timm")
    stub("timm.loss", SoftTargetCrossEntropy=_Identity)
    stub("timm.models", register_model=lambda fn: fn, create_model=None)
    stub("timm.models.layers", DropPath=_Identity, drop_path=lambda x, *a, **k: x)
    stub("pytz")


def _load_reference(path: str):
    _install_import_stubs()
    sys.path.insert(0, path)
    import enable_real_pruning_fast as erpf  # type: ignore
    import enable_pruning as ep  # type: ignore
    import real_pruning_fused_attention as rpfa  # type: ignore
    from tools import utils  # type: ignore

    return erpf, ep, rpfa, utils


class _ModuleStandIn:
    """Only ``num_heads`` is read by the reference's order/mask validators."""

    def __init__(self, num_heads: int):
        self.num_heads = num_heads


# --------------------------------------------------------------------------------------------
# Budget policy + static schedule
# --------------------------------------------------------------------------------------------

BUDGET_CONFIGS = {
    # name: (orders source, num_layers, num_heads, budget, layers recorded in the schedule file)
    "2b_b05": ("2b", 32, 16, 0.05, None),
    "2b_b10": ("2b", 32, 16, 0.10, None),
    "2b_b25": ("2b", 32, 16, 0.25, None),
    "2b_b50": ("2b", 32, 16, 0.50, None),
    "2b_b100": ("2b", 32, 16, 1.00, (0, 31)),
    "8b_b10": ("8b", 40, 28, 0.10, None),
    "rand_b05": ("rand", 32, 16, 0.05, (0, 5, 17, 31)),
    "rand_b10": ("rand", 32, 16, 0.10, (0, 5, 17, 31)),
    "rand_b25": ("rand", 32, 16, 0.25, (0, 5, 17, 31)),
    "rand_b50": ("rand", 32, 16, 0.50, (0, 5, 17, 31)),
    "rand_b100": ("rand", 32, 16, 1.00, (0, 31)),
}
SOURCE_SCALE_START = 3
PROTECTED_PREFIX_SCALES = 3


def _orders_for(kind: str, num_layers: int, num_heads: int):
    if kind == "rand":
        return synthetic.random_removal_orders(num_layers, num_heads, seed=1234)
    with open(os.path.join(REPO, "heatkv_b200", "orders", f"{kind}.json")) as fh:
        return json.load(fh)


def _schedule_arrays(erpf, controller, layer_idx: int, num_heads: int, num_scales: int) -> dict:
    sched = erpf._segmented_flat_build_static_slot_schedule(
        controller, layer_idx=layer_idx, num_heads=num_heads
    )
    out = {}
    pre = f"L{layer_idx}_"
    out[pre + "caps"] = np.array(
        [sched["capacity"], sched["capacity_bound"], sched["allocated_capacity"],
         sched.get("overalloc_slots", 0)],
        dtype=np.int64,
    )
    seg = [
        [s["source_scale"], s["head"], s["start_target"], s["end_target"], s["length"], s["offset"]]
        for s in sched["segments"]
    ]
    out[pre + "segments"] = np.array(seg, dtype=np.int32).reshape(-1, 6)
    md_rows = []
    for t in range(1, num_scales):
        starts, ends, counts = sched["metadata_cpu_by_target"][t]
        width = int(starts.shape[1])
        for h in range(num_heads):
            md_rows.append(
                [t, h, int(counts[h]), width]
                + [int(x) for x in starts[h].tolist()]
                + [-1] * (16 - width)
                + [int(x) for x in ends[h].tolist()]
                + [-1] * (16 - width)
            )
    out[pre + "metadata"] = np.array(md_rows, dtype=np.int32)

    def items(runs):
        rows = []
        for run in runs:
            for it in run["copy_items"]:
                rows.append([it["dst_start"], it["src_start"], it["length"]])
        return rows

    pack_rows = []
    for t, runs in sorted(sched["old_pack_runs_by_target"].items()):
        seq = sched["old_pack_cache_lens_by_target"][t]
        for r in items(runs):
            pack_rows.append([t, seq] + r)
    out[pre + "old_pack"] = np.array(pack_rows, dtype=np.int64).reshape(-1, 5)
    app_rows = []
    for (cur, nxt), runs in sorted(sched["append_runs_by_key"].items()):
        for r in items(runs):
            app_rows.append([cur, nxt] + r)
    out[pre + "append"] = np.array(app_rows, dtype=np.int64).reshape(-1, 5)
    return out


def make_budget_and_schedule(erpf, ep, utils, name: str) -> None:
    kind, num_layers, num_heads, budget, layers = BUDGET_CONFIGS[name]
    orders = _orders_for(kind, num_layers, num_heads)
    view = utils.strict_removed_heads_by_scale_specific_for_budget(
        budget,
        orders,
        num_layers=num_layers,
        num_heads=num_heads,
        source_scale_start=SOURCE_SCALE_START,
        protected_prefix_scales=PROTECTED_PREFIX_SCALES,
    )
    num_scales = len(utils.get_scale_schedule())
    removed = np.zeros((num_scales, 9, num_layers, num_heads), dtype=np.uint8)
    for t, by_source in view["removed_heads_by_scale"].items():
        for s, by_layer in by_source.items():
            for layer, heads in by_layer.items():
                for h in heads:
                    removed[int(t), int(s) - SOURCE_SCALE_START, int(layer), int(h)] = 1
    counts = np.array([view["removed_counts_by_scale"][t] for t in range(num_scales)], dtype=np.int64)
    remaining = np.array(
        [view["remaining_atoms_by_scale"][t] for t in range(num_scales)], dtype=np.int64
    )
    budget_arrays = {"removed": removed, "removed_counts": counts, "remaining_atoms": remaining}
    if kind == "rand":
        budget_arrays["orders"] = np.array(orders, dtype=np.int16)
    np.savez_compressed(os.path.join(HERE, f"budget_{name}.npz"), **budget_arrays)

    modules = [_ModuleStandIn(num_heads) for _ in range(num_layers)]
    normalized = ep._validate_and_normalize_removed_heads_by_scale_specific(
        view["removed_heads_by_scale"], modules, source_scale_start=SOURCE_SCALE_START
    )
    controller = ep.ScaleSpecificPruningController(
        num_layers=num_layers,
        num_heads=num_heads,
        static_removed_heads_by_scale=normalized,
        source_scale_start=SOURCE_SCALE_START,
    )
    arrays = {}
    for layer in layers if layers is not None else range(num_layers):
        arrays.update(_schedule_arrays(erpf, controller, layer, num_heads, num_scales))
    np.savez_compressed(os.path.join(HERE, f"schedule_{name}.npz"), **arrays)
    print(f"{name}: removed counts {counts.tolist()}")


# --------------------------------------------------------------------------------------------
# Config 1: 7-scale single layer, seeded keep-mask, fp32
# --------------------------------------------------------------------------------------------


class _SevenScaleController:
    """Duck-typed controller for the 7-scale config. The reference's static scheduler reads only
    ``scale_schedule``, ``scale_ranges`` and ``removed_heads_by_source_for``
    (enable_real_pruning_fast.py:215-218, :273-292)."""

    def __init__(self, ep, removed_pairs):
        self.scale_schedule = synthetic.C1_SCALE_SCHEDULE
        self.scale_ranges = ep._scale_token_ranges(self.scale_schedule)
        self._removed = removed_pairs  # set of (source, head), removed for every target

    def removed_heads_by_source_for(self, layer_idx, target_scale_idx):
        out = {}
        for source, head in self._removed:
            if source < target_scale_idx:
                out.setdefault(source, set()).add(head)
        return out


def _sha(t: torch.Tensor) -> bytes:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).digest()


def make_config1(erpf, ep, rpfa) -> None:
    cfg = synthetic.config1()
    controller = _SevenScaleController(ep, cfg.removed_pairs)
    num_scales = len(controller.scale_schedule)
    sched_arrays = _schedule_arrays(erpf, controller, 0, cfg.num_heads, num_scales)
    np.savez_compressed(os.path.join(HERE, "schedule_c1.npz"), **sched_arrays)

    sched = erpf._segmented_flat_build_static_slot_schedule(
        controller, layer_idx=0, num_heads=cfg.num_heads
    )
    qkv = synthetic.config1_qkv(cfg)
    first_target = synthetic.first_pruned_target(controller.removed_heads_by_source_for, num_scales)
    cap = int(sched["capacity"])
    slab_k = torch.zeros((cfg.batch, cap, cfg.head_dim), dtype=torch.float32)
    slab_v = torch.zeros_like(slab_k)

    digests = []
    # Activation pack from the dense cache that holds scales 0..first_target-1
    # (enable_real_pruning_fast.py:2020-2037 -> :871-967, static precomputed runs).
    dense_k = torch.cat([qkv[s][1] for s in range(first_target)], dim=2)
    dense_v = torch.cat([qkv[s][2] for s in range(first_target)], dim=2)
    erpf._segmented_flat_static_copy_precomputed_runs(
        dst_k=slab_k, dst_v=slab_v, src_k=dense_k, src_v=dense_v,
        runs=sched["old_pack_runs_by_target"][first_target],
    )
    digests.append([first_target, -1] + list(_sha(slab_k)) + list(_sha(slab_v)))

    attn_rows = {}
    for t in range(first_target, num_scales):
        q, k, v = qkv[t]
        starts, ends, counts = sched["metadata_cpu_by_target"][t]
        out = rpfa._flat_segmented_attention_reference(
            q=q, persisted_k=slab_k, persisted_v=slab_v,
            segment_starts=starts, segment_ends=ends, segment_counts=counts,
            current_k=k, current_v=v, softmax_scale=cfg.softmax_scale,
        )
        attn_rows[f"t{t}_head_rows"] = out[:, :4, :].contiguous().numpy()
        attn_rows[f"t{t}_checksums"] = synthetic.output_checksums(out.numpy())
        if t + 1 < num_scales:
            erpf._segmented_flat_static_copy_precomputed_runs(
                dst_k=slab_k, dst_v=slab_v, src_k=k, src_v=v,
                runs=sched["append_runs_by_key"][(t, t + 1)],
            )
            digests.append([t, t + 1] + list(_sha(slab_k)) + list(_sha(slab_v)))
    np.savez_compressed(
        os.path.join(HERE, "pack_c1.npz"),
        digests=np.array(digests, dtype=np.int64),
        capacity=np.array([cap]),
        first_target=np.array([first_target]),
    )
    np.savez_compressed(os.path.join(HERE, "attention_c1.npz"), **attn_rows)
    print(f"config1: capacity {cap}, first pruned target {first_target}")


# --------------------------------------------------------------------------------------------
# Small direct attention cases through the reference CPU oracle
# --------------------------------------------------------------------------------------------


def make_attention_cases(rpfa) -> None:
    arrays = {}
    for case in synthetic.ATTENTION_CASES:
        inputs = synthetic.attention_case_inputs(case)
        out = rpfa._flat_segmented_attention_reference(
            q=inputs["q"], persisted_k=inputs["persisted_k"], persisted_v=inputs["persisted_v"],
            segment_starts=inputs["segment_starts"], segment_ends=inputs["segment_ends"],
            segment_counts=inputs["segment_counts"], current_k=inputs["current_k"],
            current_v=inputs["current_v"], softmax_scale=inputs["softmax_scale"],
        )
        if out.dtype == torch.bfloat16:
            arrays[case.name] = out.view(torch.int16).numpy()
        else:
            arrays[case.name] = out.numpy()
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **arrays)
    print(f"attention cases: {sorted(arrays)}")


# --------------------------------------------------------------------------------------------
# S-CAS accumulation (tools/compute_scas.py:92-152)
# --------------------------------------------------------------------------------------------

SCAS_LAYERS, SCAS_HEADS, SCAS_SINK, SCAS_PROMPTS = 2, 16, 3, 2


def make_scas(reference_path: str) -> None:
    """The reference's ScasAccumulator fed, per (prompt, layer, scale), the probabilities of its
    capture forward (softmax of q k^T in fp32 over every key so far, :217-218): accum, scores and
    orders on the 7-scale schedule."""
    import tools  # type: ignore  (the reference's package; run_infinity is not needed here)

    stub = types.ModuleType("tools.run_infinity")
    sys.modules.setdefault("tools.run_infinity", stub)
    tools.run_infinity = sys.modules["tools.run_infinity"]
    from tools import compute_scas  # type: ignore

    schedule = list(synthetic.C1_SCALE_SCHEDULE)
    acc = compute_scas.ScasAccumulator(num_layers=SCAS_LAYERS, num_heads=SCAS_HEADS,
                                       scale_schedule=schedule, sink_scales=SCAS_SINK,
                                       device=torch.device("cpu"))
    for prompt in range(SCAS_PROMPTS):
        for layer in range(SCAS_LAYERS):
            qk = synthetic.scas_inputs(prompt, layer, schedule, heads=SCAS_HEADS)
            for t in range(len(schedule)):
                q = qk[t][0]
                k = torch.cat([qk[s][1] for s in range(t + 1)], dim=2)
                probs = torch.softmax(torch.matmul(q.float(), k.float().transpose(-2, -1)) * 1.0,
                                      dim=-1)
                acc.update(layer_idx=layer, scale_ind=t, probs=probs)
    scores = acc.scores(SCAS_PROMPTS)
    orders = acc.orders_from_scores(scores)
    np.savez_compressed(os.path.join(HERE, "scas_c1.npz"), accum=acc.accum.numpy(),
                        scores=scores.numpy(), orders=np.array(orders, dtype=np.int16))
    print(f"scas: accum {tuple(acc.accum.shape)}, {len(orders)} orders")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    parser.add_argument("--reference", required=True, help="path of the reference checkout")
    parser.add_argument("--only", default=None, help="comma list: budget,c1,attention,scas")
    args = parser.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    erpf, ep, rpfa, utils = _load_reference(args.reference)
    only = set(args.only.split(",")) if args.only else {"budget", "c1", "attention", "scas"}
    if "budget" in only:
        for name in BUDGET_CONFIGS:
            make_budget_and_schedule(erpf, ep, utils, name)
    if "c1" in only:
        make_config1(erpf, ep, rpfa)
    if "attention" in only:
        make_attention_cases(rpfa)
    if "scas" in only:
        make_scas(args.reference)


if __name__ == "__main__":
    main()
