"""(batch row x head) sharding across GPUs: planner, per-rank schedules, and the all-gather +
reassembly of head-sharded outputs on two gloo ranks (CPU; the CUDA reassembly kernel and the
NCCL path are covered by the GPU tests).

The two-rank test computes each rank's attention with the CPU oracle over the rank's own slot
schedule, gathers the rank blocks with ``all_gather_into_tensor`` and places them with the plan's
row/head maps; the result must equal the single-process computation over all heads.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from heatkv_b200 import sharding, synthetic
from heatkv_b200.hotpath import LayerPlan
from heatkv_b200.scheduler import build_static_slot_schedule
from oracle.attention import segmented_attention

from test_host_golden import config1_controller


@pytest.fixture(scope="module")
def ctrl_2b():
    ctrl, layers, heads = bench.build_controller("2b", 0.10)
    return ctrl, layers, heads


def test_live_slots_match_the_slot_schedule(ctrl_2b):
    ctrl, layers, heads = ctrl_2b
    for layer in (0, 7, 19, 31):
        plan = LayerPlan(ctrl, layer, heads, "cpu")
        live = sharding.live_slots(ctrl, layer)
        for t in range(plan.num_scales):
            np.testing.assert_array_equal(live[t], plan.attention_slots(t), err_msg=f"{layer}/{t}")


def test_head_costs_sum_to_the_image_flops(ctrl_2b):
    ctrl, layers, heads = ctrl_2b
    costs = sharding.head_costs(ctrl, layers, heads)
    assert costs.shape == (layers, heads)
    # one row: 8.362 TFLOP fused + 0.144 TFLOP dense prefix (reference schedule, 2B / 10 %)
    total = bench.image_flops(ctrl, layers, heads, 1)
    assert abs(costs.sum() - total) <= 1e-9 * total
    assert abs(total / 1e12 - (8.362 + 0.144)) < 0.01


@pytest.mark.parametrize("groups", [1, 2, 4, 8, 16])
def test_balanced_partition(groups):
    rng = np.random.default_rng(groups)
    costs = rng.gamma(2.0, 1.0, size=16)
    parts = sharding.balanced_partition(costs, groups)
    assert len(parts) == groups
    assert sorted(h for p in parts for h in p) == list(range(16))
    assert all(len(p) == 16 // groups for p in parts)
    loads = [costs[p].sum() for p in parts]
    assert max(loads) <= costs.sum() / groups + costs.max() + 1e-12
    with pytest.raises(ValueError):
        sharding.balanced_partition(costs, 3)


@pytest.mark.parametrize("batch,world,split,row_groups", [
    (2, 1, "auto", 1), (2, 2, "auto", 2), (2, 4, "auto", 2), (2, 8, "auto", 2),
    (16, 8, "auto", 8), (64, 8, "auto", 8), (2, 2, "heads", 1), (2, 8, "heads", 1),
    (16, 4, "rows", 4), (6, 4, "auto", 2),
])
def test_plan_covers_every_unit_once(ctrl_2b, batch, world, split, row_groups):
    ctrl, layers, heads = ctrl_2b
    costs = sharding.head_costs(ctrl, layers, heads)
    plan = sharding.plan_shards(costs, batch, world, split=split)
    assert plan.row_groups == row_groups and plan.head_groups * row_groups == world
    for layer in range(layers):
        seen = np.zeros((batch, heads), dtype=np.int64)
        for r in range(world):
            for row in plan.rows_of(r):
                for h in plan.heads_of(r, layer):
                    seen[row, h] += 1
        assert (seen == 1).all()
        hm = plan.head_map(layer)
        assert hm.shape == (world * plan.heads_per_rank,)
    rm = plan.row_map()
    assert rm.shape == (world * plan.rows_per_rank,)
    if 1 < plan.head_groups <= 4:
        # equal-size head groups of 16 heads stay within 10 % of perfect balance per layer
        assert plan.imbalance(costs) < 1.10


def test_plan_rejects_impossible_splits(ctrl_2b):
    ctrl, layers, heads = ctrl_2b
    costs = sharding.head_costs(ctrl, layers, heads)
    with pytest.raises(ValueError):
        sharding.plan_shards(costs, 3, 2, split="rows")
    with pytest.raises(ValueError):
        sharding.plan_shards(costs[:, :12], 1, 8)   # 12 heads into 8 groups


def test_rank_schedules_hold_exactly_their_heads(ctrl_2b):
    ctrl, layers, heads = ctrl_2b
    costs = sharding.head_costs(ctrl, layers, heads)
    plan = sharding.plan_shards(costs, 2, 8)
    for layer in (0, 13, 31):
        full = LayerPlan(ctrl, layer, heads, "cpu")
        for r in range(8):
            hs = plan.heads_of(r, layer)
            sub = sharding.HeadSubsetController(ctrl, [plan.heads_of(r, l) for l in range(layers)])
            local = LayerPlan(sub, layer, len(hs), "cpu")
            assert local.capacity <= full.capacity
            assert local.first_target == full.first_target   # same dense -> slab switch
            for t in range(full.num_scales):
                np.testing.assert_array_equal(local.attention_slots(t), full.attention_slots(t)[hs])


# ------------------------------------------------------------------------------------------------
# two gloo ranks: oracle attention per rank, all-gather, reassembly by the plan's maps
# ------------------------------------------------------------------------------------------------

def _slab_for_target(sched, t, k_seq, v_seq, heads_global):
    """Slab [B, cap, D] holding the live segments at target t, read from the per-head token
    sequences k_seq/v_seq [B, H_global, T, D] (local head i -> global heads_global[i])."""
    B, _, _, D = k_seq.shape
    cap = max(int(sched["capacity"]), 1)
    sk = np.zeros((B, cap, D), k_seq.dtype)
    sv = np.zeros_like(sk)
    for seg in sched["segments_by_target"][t]:
        g = heads_global[seg["head"]]
        lo, n, off = seg["scale_start"], seg["length"], seg["offset"]
        sk[:, off:off + n] = k_seq[:, g, lo:lo + n]
        sv[:, off:off + n] = v_seq[:, g, lo:lo + n]
    return sk, sv


def _attention(ctrl, heads_global, rows, qkv, t):
    """Oracle output [len(rows), n_t, len(heads) * D] of target t for the given rows and heads."""
    sched = build_static_slot_schedule(ctrl, layer_idx=0, num_heads=len(heads_global))
    k_seq = np.concatenate([k for _, k, _ in qkv[:t]], axis=2)[rows]
    v_seq = np.concatenate([v for _, _, v in qkv[:t]], axis=2)[rows]
    k_seq = np.ascontiguousarray(k_seq)
    sk, sv = _slab_for_target(sched, t, k_seq, v_seq, heads_global)
    st, en, ct = sched["metadata_cpu_by_target"][t]
    q, k, v = (x[rows][:, heads_global] for x in qkv[t])
    return segmented_attention(q=q, persisted_k=sk, persisted_v=sv, segment_starts=st,
                               segment_ends=en, segment_counts=ct, current_k=k, current_v=v,
                               softmax_scale=128 ** -0.5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, split, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, ctrl = config1_controller()
        costs = sharding.head_costs(ctrl, 1, cfg.num_heads)
        plan = sharding.plan_shards(costs, cfg.batch, world, split=split)
        qkv = [tuple(x.numpy().astype(np.float64) for x in s) for s in synthetic.config1_qkv(cfg)]
        heads = plan.heads_of(rank, 0)
        sub = sharding.HeadSubsetController(ctrl, [heads])
        rows = plan.rows_of(rank)
        D = cfg.head_dim
        for t in (4, 6):
            local = _attention(sub, heads, rows, qkv, t)            # [rows, n, hpr * D]
            recv = torch.empty(world * local.size, dtype=torch.float64)
            dist.all_gather_into_tensor(recv, torch.from_numpy(np.ascontiguousarray(local)).view(-1))
            recv = recv.view((world,) + local.shape)
            full = np.full((cfg.batch, local.shape[1], cfg.num_heads * D), np.nan)
            rm, hm = plan.row_map(), plan.head_map(0)
            for r in range(world):
                for i in range(plan.rows_per_rank):
                    for j in range(plan.heads_per_rank):
                        h = hm[r * plan.heads_per_rank + j]
                        full[rm[r * plan.rows_per_rank + i], :, h * D:(h + 1) * D] = \
                            recv[r, i, :, j * D:(j + 1) * D].numpy()
            if rank == 0:
                ref = _attention(ctrl, list(range(cfg.num_heads)), list(range(cfg.batch)), qkv, t)
                err = float(np.abs(full - ref).max())
                queue.put((t, plan.row_groups, plan.head_groups, err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", ["heads", "auto"])
def test_two_gloo_ranks_reassemble_the_single_process_output(split):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, split, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [queue.get(timeout=10) for _ in range(2)]
    for t, rg, hg, err in results:
        assert (rg, hg) == ((1, 2) if split == "heads" else (2, 1))
        assert err <= 1e-12, (t, err)
