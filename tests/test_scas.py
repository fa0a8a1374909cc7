"""Host logic of the S-CAS accumulator (tools/compute_scas.py:57-64, :93-152): token bounds,
which source scales an update touches, scores and the removal orders (CPU)."""

import math

import torch

from heatkv_b200.scas import ScasAccumulator, scale_token_bounds

SCHED_7 = [(1, 1, 1), (1, 2, 2), (1, 4, 4), (1, 6, 6), (1, 8, 8), (1, 12, 12), (1, 16, 16)]


def test_scale_token_bounds():
    assert scale_token_bounds(SCHED_7)[:4] == [(0, 1), (1, 5), (5, 21), (21, 57)]
    assert scale_token_bounds(SCHED_7)[-1] == (265, 521)


def test_sources_of_an_update():
    acc = ScasAccumulator(num_layers=1, num_heads=1, scale_schedule=SCHED_7, sink_scales=2,
                          device="cpu")
    assert acc._sources(2, 521) == []          # sink scales never update
    assert acc._sources(3, 521) == [2]
    assert acc._sources(6, 521) == [2, 3, 4, 5]
    assert acc._sources(7, 521) == []          # past the last scale
    assert acc._sources(6, 60) == [2, 3]       # sources not complete among the keys are skipped


def test_update_scores_and_orders_on_cpu_probabilities():
    acc = ScasAccumulator(num_layers=2, num_heads=3, scale_schedule=SCHED_7, sink_scales=1,
                          device="cpu")
    g = torch.Generator().manual_seed(0)
    for layer in range(2):
        for t in range(7):
            end = scale_token_bounds(SCHED_7)[t][1]
            n = SCHED_7[t][1] * SCHED_7[t][2]
            probs = torch.softmax(torch.randn(2, 3, n, end, generator=g), dim=-1)
            acc.update(layer_idx=layer, scale_ind=t, probs=probs)
    sc = acc.scores(num_prompts=4)
    assert torch.isnan(sc[:, :, 0]).all() and torch.isnan(sc[:, :, 6]).all()
    assert torch.allclose(sc[:, :, 1], acc.accum[:, :, 1] / (4 * 5))
    orders = acc.orders_from_scores(sc)
    assert len(orders) == 5 and all(len(o) == 6 for o in orders)
    for s, order in zip(range(1, 6), orders):
        vals = [float(sc[l, h, s]) for h, l in order]
        assert vals == sorted(vals)
    # ties: by head, then layer
    tie = torch.zeros_like(sc)
    assert acc.orders_from_scores(tie)[0] == [(0, 0), (0, 1), (1, 0), (1, 1), (2, 0), (2, 1)]
    assert not math.isnan(float(sc[0, 0, 1]))


def _replay_fixture_inputs(acc, update):
    from heatkv_b200 import synthetic
    sched = list(synthetic.C1_SCALE_SCHEDULE)
    for prompt in range(2):
        for layer in range(2):
            qk = synthetic.scas_inputs(prompt, layer, sched, heads=16)
            for t in range(len(sched)):
                q = qk[t][0]
                k = torch.cat([qk[s][1] for s in range(t + 1)], dim=2)
                update(acc, layer, t, q, k)


def test_probability_update_matches_the_reference_fixture(golden_dir):
    """``update`` from the capture forward's fp32 probabilities against the reference's own
    ScasAccumulator (tests/golden/scas_c1.npz): accum and scores within 1e-12 relative, orders
    identical."""
    import os

    import numpy as np

    from heatkv_b200 import synthetic
    fx = np.load(os.path.join(golden_dir, "scas_c1.npz"))
    acc = ScasAccumulator(num_layers=2, num_heads=16, scale_schedule=list(synthetic.C1_SCALE_SCHEDULE),
                          sink_scales=3, device="cpu")

    def update(a, layer, t, q, k):
        probs = torch.softmax(torch.matmul(q.float(), k.float().transpose(-2, -1)), dim=-1)
        a.update(layer_idx=layer, scale_ind=t, probs=probs)

    _replay_fixture_inputs(acc, update)
    assert np.allclose(acc.accum.numpy(), fx["accum"], rtol=1e-12, atol=0)
    sc = acc.scores(2).numpy()
    assert np.array_equal(np.isnan(sc), np.isnan(fx["scores"]))
    assert np.allclose(np.nan_to_num(sc), np.nan_to_num(fx["scores"]), rtol=1e-12, atol=0)
    assert np.array_equal(np.array(acc.orders_from_scores(acc.scores(2)), dtype=np.int16),
                          fx["orders"])
