"""GPU parity of the one-pass S-CAS accumulation (heatkv_scas_mass via
ScasAccumulator.update_from_qk) against the reference's form: probabilities
softmax(q k^T * scale) computed in fp32 with PyTorch (tools/compute_scas.py:217-218), reduced by
ScasAccumulator.update (:114-128). Tolerance: fp32 (1e-5 relative on the float64 accumulator)."""

import math

import numpy as np
import pytest
import torch

from heatkv_b200 import _native, synthetic
from heatkv_b200.scas import ScasAccumulator

pytestmark = pytest.mark.gpu

SCHED_7 = [(1, 1, 1), (1, 2, 2), (1, 4, 4), (1, 6, 6), (1, 8, 8), (1, 12, 12), (1, 16, 16)]


@pytest.fixture(params=["tensor_cores", "cuda_cores"])
def scas_kernel(request, monkeypatch):
    """The tensor-core kernel (default for fp32: three tf32 products a score) and the CUDA-core
    kernel (fp32 products)."""
    monkeypatch.setenv("HEATKV_SCAS_KERNEL", request.param)
    return request.param


def _probs(q, k, scale):
    scores = torch.matmul(q.float(), k.float().transpose(-2, -1)) * float(scale)
    return torch.softmax(scores, dim=-1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("schedule,sink,layers", [(SCHED_7, 1, 2), (synthetic.SCALE_SCHEDULE_1M[:11], 2, 1)])
def test_update_from_qk_matches_probabilities(dtype, schedule, sink, layers, scas_kernel):
    dev = torch.device("cuda", 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    H = 16
    ref = ScasAccumulator(num_layers=layers, num_heads=H, scale_schedule=schedule,
                          sink_scales=sink, device=dev)
    ours = ScasAccumulator(num_layers=layers, num_heads=H, scale_schedule=schedule,
                           sink_scales=sink, device=dev)
    g = torch.Generator(device="cuda").manual_seed(len(schedule))
    total = sum(a * b * c for a, b, c in schedule)
    scale = 1.0 / math.sqrt(128)
    for layer in range(layers):
        # cos-attention-like rows: unit norm times a head scale, so the softmax is peaked
        keys = torch.randn(2, H, total, 128, device=dev, generator=g)
        keys = torch.nn.functional.normalize(keys, dim=-1).to(dtype)
        queries = torch.randn(2, H, total, 128, device=dev, generator=g)
        queries = (torch.nn.functional.normalize(queries, dim=-1) * 12.0).to(dtype)
        start = 0
        for t, (a, b, c) in enumerate(schedule):
            n = a * b * c
            q = queries[:, :, start:start + n]
            k = keys[:, :, :start + n]
            ref.update(layer_idx=layer, scale_ind=t, probs=_probs(q, k, scale))
            ours.update_from_qk(layer_idx=layer, scale_ind=t, q=q, k=k, scale=scale)
            start += n
    torch.cuda.synchronize()
    a, b = ours.accum.cpu().numpy(), ref.accum.cpu().numpy()
    assert np.abs(b).max() > 0
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-9)
    assert ours.orders_from_scores(ours.scores(1)) == ref.orders_from_scores(ref.scores(1))
    assert _native.device_status(dev) == 0


def test_sources_missing_from_the_keys_are_skipped():
    """A source scale whose tokens are not all among the keys is skipped, as the reference's
    `continue` does; only batch row 0 counts."""
    dev = torch.device("cuda", 0)
    acc = ScasAccumulator(num_layers=1, num_heads=2, scale_schedule=SCHED_7, sink_scales=1,
                          device=dev)
    q = torch.randn(3, 2, 36, 128, device=dev)
    k = torch.randn(3, 2, 10, 128, device=dev)   # scales 0-1 complete, scale 2 cut short
    acc.update_from_qk(layer_idx=0, scale_ind=3, q=q, k=k, scale=0.1)
    torch.cuda.synchronize()
    row = acc.accum[0].cpu()
    assert torch.all(row[:, 2:] == 0) and torch.all(row[:, 1] > 0) and torch.all(row[:, 0] == 0)
    ref = ScasAccumulator(num_layers=1, num_heads=2, scale_schedule=SCHED_7, sink_scales=1,
                          device=dev)
    ref.update(layer_idx=0, scale_ind=3, probs=_probs(q, k, 0.1))
    np.testing.assert_allclose(acc.accum.cpu().numpy(), ref.accum.cpu().numpy(), rtol=1e-5)


def test_update_from_qk_matches_the_reference_fixture(golden_dir, scas_kernel):
    """``update_from_qk`` on the GPU against the reference's own ScasAccumulator
    (tests/golden/scas_c1.npz, recorded from tools/compute_scas.py:92-152 on the capture
    forward's fp32 probabilities of the same seeded q/k): accum within 1e-5 relative, the removal
    orders identical."""
    import os
    fx = np.load(os.path.join(golden_dir, "scas_c1.npz"))
    dev = torch.device("cuda", 0)
    sched = list(synthetic.C1_SCALE_SCHEDULE)
    acc = ScasAccumulator(num_layers=2, num_heads=16, scale_schedule=sched, sink_scales=3,
                          device=dev)
    for prompt in range(2):
        for layer in range(2):
            qk = synthetic.scas_inputs(prompt, layer, sched, heads=16)
            for t in range(len(sched)):
                k = torch.cat([qk[s][1] for s in range(t + 1)], dim=2).to(dev)
                acc.update_from_qk(layer_idx=layer, scale_ind=t, q=qk[t][0].to(dev), k=k,
                                   scale=1.0)
    torch.cuda.synchronize()
    assert np.abs(fx["accum"]).max() > 0
    np.testing.assert_allclose(acc.accum.cpu().numpy(), fx["accum"], rtol=1e-5, atol=1e-9)
    orders = np.array(acc.orders_from_scores(acc.scores(2)), dtype=np.int16)
    assert np.array_equal(orders, fx["orders"])
    assert _native.device_status(dev) == 0
