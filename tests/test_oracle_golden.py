"""Pin the CPU oracle to outputs recorded from the reference itself.

* attention: ``oracle.attention.segmented_attention`` vs the reference's
  ``_flat_segmented_attention_reference`` on the seeded edge cases (fp32 1e-5; bf16/fp16 within
  the rounding of the reference's low-precision CPU path);
* config-1 pipeline: activation pack + per-scale appends with ``oracle.pack`` reproduce the
  reference's slab bytes (SHA-256, bit-exact), and the oracle's attention outputs reproduce the
  reference's checksums and leading rows at every fused target.
"""

import hashlib
import os

import numpy as np
import pytest
import torch

from heatkv_b200 import synthetic
from heatkv_b200.scheduler import build_static_slot_schedule, copy_descriptors
from oracle.attention import segmented_attention
from oracle.pack import pack_flat_segments

from test_host_golden import config1_controller


@pytest.mark.parametrize("case", synthetic.ATTENTION_CASES, ids=lambda c: c.name)
def test_oracle_attention_cases(case, golden_dir):
    g = np.load(os.path.join(golden_dir, "attention_cases.npz"))
    ref = g[case.name]
    if case.dtype == "bf16":
        ref = torch.from_numpy(ref).view(torch.bfloat16).float().numpy()
    inputs = synthetic.attention_case_inputs(case)
    out = segmented_attention(**inputs)
    if case.dtype == "f32":
        np.testing.assert_allclose(out, ref, atol=1e-5, rtol=1e-5)
    else:
        # the reference's CPU path computes and rounds in bf16/fp16; compare after rounding
        dt = torch.bfloat16 if case.dtype == "bf16" else torch.float16
        mine = torch.from_numpy(out).to(dt).float().numpy()
        np.testing.assert_allclose(mine, ref, atol=2e-2, rtol=0)


def _sha(a: np.ndarray) -> list:
    return list(hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest())


def test_oracle_config1_pipeline(golden_dir):
    cfg, ctrl = config1_controller()
    sched = build_static_slot_schedule(ctrl, layer_idx=0, num_heads=cfg.num_heads)
    pk = np.load(os.path.join(golden_dir, "pack_c1.npz"))
    ga = np.load(os.path.join(golden_dir, "attention_c1.npz"))
    qkv = [(q.numpy(), k.numpy(), v.numpy()) for q, k, v in synthetic.config1_qkv(cfg)]
    first = synthetic.first_pruned_target(ctrl.removed_heads_by_source_for, len(qkv))
    assert first == int(pk["first_target"][0])
    cap = sched["capacity"]
    slab_k = np.zeros((cfg.batch, cap, cfg.head_dim), dtype=np.float32)
    slab_v = np.zeros_like(slab_k)
    digests = pk["digests"].tolist()

    dense_k = np.concatenate([qkv[s][1] for s in range(first)], axis=2)
    dense_v = np.concatenate([qkv[s][2] for s in range(first)], axis=2)
    d = copy_descriptors(sched["old_pack_runs_by_target"][first])
    B, H, T, D = dense_k.shape
    pack_flat_segments(slab_k, slab_v, dense_k.reshape(B, H * T, D), dense_v.reshape(B, H * T, D),
                       d["dst_starts"], d["src_starts"], d["lengths"])
    assert [first, -1] + _sha(slab_k) + _sha(slab_v) == digests[0]
    step = 1
    for t in range(first, len(qkv)):
        q, k, v = qkv[t]
        st, en, ct = sched["metadata_cpu_by_target"][t]
        out = segmented_attention(q=q, persisted_k=slab_k, persisted_v=slab_v, segment_starts=st,
                                  segment_ends=en, segment_counts=ct, current_k=k, current_v=v,
                                  softmax_scale=cfg.softmax_scale)
        np.testing.assert_allclose(out[:, :4, :], ga[f"t{t}_head_rows"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(synthetic.output_checksums(out), ga[f"t{t}_checksums"],
                                   rtol=1e-6, atol=1e-4)
        if t + 1 < len(qkv):
            d = copy_descriptors(sched["append_runs_by_key"][(t, t + 1)])
            B, H, T, D = k.shape
            pack_flat_segments(slab_k, slab_v, k.reshape(B, H * T, D), v.reshape(B, H * T, D),
                               d["dst_starts"], d["src_starts"], d["lengths"])
            assert [t, t + 1] + _sha(slab_k) + _sha(slab_v) == digests[step]
            step += 1
    assert step == len(digests)
