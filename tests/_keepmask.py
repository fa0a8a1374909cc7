"""Attention over exactly the tokens a keep-mask retains, in plain PyTorch fp32 (test helper).

For target scale ``t`` and head ``h`` the keys are scales ``0..t-1`` minus the (source, head)
pairs the controller removes at ``t`` (``removed_mask_for_layer``), then the whole current
scale: the semantics of the reference's static slab schedule
(enable_real_pruning_fast.py:260-412) and of its fused kernel
(real_pruning_fused_attention.py:76-267), written without slabs, segments or offsets, so it
checks the schedule, the pack descriptors and the kernel together.
"""

import math

import torch


def retained_tokens(ctrl, layer, target, head):
    """Token indices (global, scale-major) of the cached scales head ``head`` attends at
    ``target``."""
    ranges = ctrl.scale_ranges
    mask = ctrl.removed_mask_for_layer(layer)
    idx = []
    for s in range(target):
        if mask[target, s, head]:
            continue
        idx.append(torch.arange(ranges[s][0], ranges[s][1]))
    return torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long)


def keep_mask_attention(ctrl, layer, t, inputs_layer, softmax_scale=None, heads=None):
    """``inputs_layer[s] = (q, k, v)`` ``[B, H, n_s, D]`` for every scale ``s <= t``; returns the
    fp32 output ``[B, n_t, H * D]``. ``heads[j]`` maps local head j to the controller's head
    (default: the identity)."""
    q, k, v = inputs_layer[t]
    B, H, n, D = q.shape
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    full_k = torch.cat([inputs_layer[s][1] for s in range(t + 1)], dim=2).float()
    full_v = torch.cat([inputs_layer[s][2] for s in range(t + 1)], dim=2).float()
    start = ctrl.scale_ranges[t][0]
    out = torch.empty(B, n, H, D, device=q.device)
    for h in range(H):
        gh = h if heads is None else int(heads[h])
        idx = torch.cat([retained_tokens(ctrl, layer, t, gh),
                         torch.arange(start, start + n)]).to(q.device)
        s = torch.einsum("bnd,bsd->bns", q[:, h].float(), full_k[:, h, idx]) * scale
        out[:, :, h] = torch.softmax(s, -1) @ full_v[:, h, idx]
    return out.reshape(B, n, H * D)
