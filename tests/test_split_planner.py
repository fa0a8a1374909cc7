"""The length-aware launch planner (``hotpath.plan_attention``, CPU): head order, and the tail of
query blocks split in two key ranges, for the kernels' 128-row blocks."""

import numpy as np
import pytest

from heatkv_b200.hotpath import _makespan, plan_attention

import bench


def _costs(lengths, q_len, batch, block_rows, order, unsplit, item_cost, merge_cost):
    tiles = np.array([sum(-(-n // 128) for n in segs if n > 0) + -(-q_len // 128)
                      for segs in lengths])
    nblk = -(-q_len // block_rows)
    nq = [block_rows // 128] * nblk
    nq[-1] = -(-(q_len - (nblk - 1) * block_rows) // 128)
    costs = []
    for k, (rank, b, qb) in enumerate((r, b, qb) for r in range(len(order)) for b in range(batch)
                                      for qb in range(nblk)):
        t, q = int(tiles[order[rank]]), nq[qb]
        if k < unsplit:
            costs.append(t * q + item_cost)
        else:
            costs += [(t // 2) * q + item_cost + merge_cost, (t - t // 2) * q + item_cost + merge_cost]
    return np.array(costs, dtype=np.float64)


def _first_pruned_target_lengths():
    """Segment lengths per head of layer 0 at target 8 of the 2B/10 % schedule (Lq 576)."""
    from heatkv_b200.hotpath import LayerPlan
    ctrl, _, heads = bench.build_controller("2b", 0.1)
    plan = LayerPlan(ctrl, 0, heads, "cpu")
    return plan.segment_lengths(8)


@pytest.mark.parametrize("block_rows,merge_cost", [(128, 4.0)])
def test_plan_lowers_the_makespan_it_models(block_rows, merge_cost):
    lengths = _first_pruned_target_lengths()
    q_len, batch = 576, 2
    order, splits, unsplit = plan_attention(lengths, q_len, batch, block_rows=block_rows)
    blocks = len(lengths) * batch * -(-q_len // block_rows)
    assert sorted(order.tolist()) == list(range(len(lengths)))
    tiles = [sum(-(-n // 128) for n in segs if n > 0) for segs in lengths]
    assert [tiles[h] for h in order] == sorted(tiles, reverse=True)  # longest head first
    assert 0 <= unsplit <= blocks and splits in (1, 2) and (splits == 2) == (unsplit < blocks)
    whole = _makespan(_costs(lengths, q_len, batch, block_rows, order, blocks, 1.5, merge_cost), 148)
    got = _makespan(_costs(lengths, q_len, batch, block_rows, order, unsplit, 1.5, merge_cost), 148)
    assert got <= whole
    if splits == 2:
        assert got <= whole * 0.97


def test_column_split_blocks_split_the_first_pruned_target():
    """160 blocks of 128 rows on 148 SMs leave a second wave for 12 CTAs: the planner splits."""
    lengths = _first_pruned_target_lengths()
    order, splits, unsplit = plan_attention(lengths, 576, 2, block_rows=128)
    assert splits == 2 and unsplit < 160


def test_full_waves_stay_unsplit():
    """148 equal blocks fill one wave: splitting can only add merge work."""
    lengths = [[512, 256]] * 74
    order, splits, unsplit = plan_attention(lengths, 128, 2, block_rows=128)
    assert (splits, unsplit) == (1, 148)


def test_block_rows_must_be_a_kernel_block():
    for rows in (64, 256):
        with pytest.raises(ValueError):
            plan_attention([[10]], 64, 1, block_rows=rows)


@pytest.mark.parametrize("splits", [None, 1, 2, 3])
def test_column_split_item_map_covers_every_item_once(splits):
    from heatkv_b200.hotpath import plan_column_split
    lengths = _first_pruned_target_lengths()
    order, nsplit, unsplit, item_map, grid = plan_column_split(lengths, 576, 2, splits=splits)
    blocks = 16 * 2 * 5
    n_items = unsplit + (blocks - unsplit) * nsplit
    assert grid == min(148, n_items) and len(item_map) % grid == 0
    got = sorted(int(x) for x in item_map if x >= 0)
    assert got == list(range(n_items))
    # a CTA's empty slots come after its items
    per_cta = item_map.reshape(-1, grid).T
    for row in per_cta:
        filled = row >= 0
        assert not np.any(filled[1:] & ~filled[:-1])
    # shortest head first: the split tail holds the longest blocks
    tiles = [sum(-(-n // 128) for n in segs if n > 0) for segs in lengths]
    assert [tiles[h] for h in order] == sorted(tiles)
    if splits is not None:
        assert nsplit == splits and unsplit == (blocks if splits == 1 else 0)


def test_greedy_map_beats_round_robin_at_the_first_pruned_target():
    from heatkv_b200.hotpath import _greedy_map
    lengths = _first_pruned_target_lengths()
    tiles = np.array([sum(-(-n // 128) for n in segs if n > 0) + 5 for segs in lengths])
    costs = np.repeat(np.sort(tiles)[::-1], 2 * 5).astype(float) + 1.5
    item_map, grid, span = _greedy_map(costs, 148)
    assert span < _makespan(costs, 148)
    loads = np.zeros(grid)
    for slot, item in enumerate(item_map):
        if item >= 0:
            loads[slot % grid] += costs[item]
    assert np.isclose(loads.max(), span)
