"""The pair-group-major rope table that heatkv_qkv_project reads (CPU): element (group g, token l,
i) of rope_pair_groups(t) is t[l, 4 g + i], and a scale starting at token s is the same table read
from offset s * 4 with group stride 4 * T."""

import pytest
import torch

from heatkv_b200.qkv_prep import rope_pair_groups


def test_pair_groups_hold_each_tokens_pairs():
    T = 37
    t = torch.arange(T * 64, dtype=torch.float32).reshape(T, 64)
    g = rope_pair_groups(t)
    assert g.shape == (16, T, 4) and g.is_contiguous()
    for grp in (0, 5, 15):
        for l in (0, 17, T - 1):
            assert torch.equal(g[grp, l], t[l, 4 * grp:4 * grp + 4])
    # the kernel's addressing: base + s * 4, element (grp, l) at grp * 4T + 4 l + i
    flat = g.reshape(-1)
    s, stride = 9, 4 * T
    for grp, l, i in ((3, 0, 1), (15, 27, 3), (0, 5, 0)):
        assert flat[s * 4 + grp * stride + 4 * l + i] == t[s + l, 4 * grp + i]


def test_pair_groups_reject_other_widths():
    with pytest.raises(ValueError):
        rope_pair_groups(torch.zeros(4, 32))
