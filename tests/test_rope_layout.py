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


def test_rope_groups_of_a_cache_grid_cover_every_token():
    from heatkv_b200.qkv_prep import rope_groups
    sched = [(1, 1, 1), (1, 2, 2), (1, 4, 4)]
    T = 21
    angles = torch.rand(1, 1, 1, T, 64)
    grid = {str(tuple(sched)): torch.stack([torch.cos(angles), torch.sin(angles)])}
    cg, sg = rope_groups(grid, sched, "cpu")
    assert cg.shape == sg.shape == (16, T, 4)
    assert torch.equal(cg, rope_pair_groups(torch.cos(angles)[0, 0, 0]))
    assert torch.equal(sg, rope_pair_groups(torch.sin(angles)[0, 0, 0]))
    assert rope_groups(grid, sched, "cpu")[0] is cg   # built once


def test_project_qkv_rejects_bad_arguments_before_any_launch():
    from heatkv_b200.qkv_prep import project_qkv
    x = torch.zeros(1, 4, 256, dtype=torch.bfloat16)
    w = torch.zeros(3 * 2 * 128, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        project_qkv(x, w, None, 2)
    with pytest.raises(RuntimeError, match="16-bit"):
        project_qkv(x.float(), w, None, 2)
    with pytest.raises(ValueError, match="weight"):
        project_qkv(x, w[:-1], None, 2)
    with pytest.raises(ValueError, match="x shaped"):
        project_qkv(x[0], w, None, 2)


def test_installer_uses_the_fused_projection_only_where_it_stands_for_the_chain():
    import torch.nn as nn
    from heatkv_b200.enable_real_pruning_fast import _fused_project_dtype

    class M(nn.Module):
        def __init__(self, C=256, H=2):
            super().__init__()
            self.num_heads, self.head_dim, self.cos_attn = H, 128, True
            self.mat_qkv = nn.Linear(C, 3 * C, bias=False)
            self._heatkv_fused_qkv_prep = True

    m = M()
    x = torch.zeros(1, 4, 256)
    assert _fused_project_dtype(m, x) is None          # CPU tensors
    m._heatkv_fused_qkv_prep = False
    assert _fused_project_dtype(m, x) is None
