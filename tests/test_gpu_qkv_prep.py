"""GPU parity of ``heatkv_qkv_prepare`` (``qkv_prep.prepare_qkv``): the one-pass q/k/v
preparation against the PyTorch chain of the reference's patched forward
(enable_real_pruning_fast.py:2040-2072) and the rotary embedding of
infinity/models/basic.py:97-117, restated below.

Without cos-attention every output is bit-identical (the permute is a copy and the rotary
embedding rounds each product and sum exactly as the elementwise ops do). With cos-attention the
row norm is a reduction whose order differs from PyTorch's, so q and k agree to fp32 rounding:
max |err| <= 1e-6 on unit-norm rows scaled by at most 100. With ``append=`` the given heads' k/v
rows also land in the slab, bit for bit (the reference's append copy,
enable_real_pruning_fast.py:969-1024).
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from heatkv_b200 import _native
from heatkv_b200.qkv_prep import prepare_qkv, rope_rows

pytestmark = pytest.mark.gpu


def _reference_rope(q, k, cos, sin):
    """apply_rotary_emb (infinity/models/basic.py:97-117) on explicit rope rows, autocast off."""
    qk = torch.stack((q, k), dim=0)
    with torch.autocast(device_type="cuda", enabled=False):
        qk = qk.reshape(*qk.shape[:-1], -1, 2)
        c, s = cos[None, None, None], sin[None, None, None]
        qk = torch.stack([c * qk[..., 0] - s * qk[..., 1], s * qk[..., 0] + c * qk[..., 1]], dim=-1)
        qk = qk.reshape(*qk.shape[:-2], -1)
        q, k = qk.unbind(dim=0)
    return q, k


def _reference_prep(qkv, scale_mul, cos, sin):
    q, k, v = qkv.unbind(dim=2)
    q = q.permute(0, 2, 1, 3).contiguous()
    k = k.permute(0, 2, 1, 3).contiguous()
    v = v.permute(0, 2, 1, 3).contiguous()
    if scale_mul is not None:
        q = F.normalize(q, dim=-1, eps=1e-12).mul(scale_mul).contiguous()
        k = F.normalize(k, dim=-1, eps=1e-12).contiguous()
    if cos is not None:
        q, k = _reference_rope(q, k, cos, sin)
    return q, k, v


def _inputs(B, L, H, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = (torch.randn(B, L, 3, H, 128, device="cuda", generator=g) * 3).to(dtype)
    scale_mul = torch.empty(1, H, 1, 1, device="cuda").uniform_(0.5, math.log(100), generator=g).exp()
    grid = torch.rand(2, 1, 1, 1, L + 37, 64, device="cuda", generator=g) * 6.0
    grid = torch.stack([torch.cos(grid[0]), torch.sin(grid[0])])  # a [2, 1, 1, 1, N, 64] cache
    return qkv, scale_mul, grid


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,L,H", [(2, 1, 16), (1, 4, 16), (2, 577, 16), (2, 4096, 16), (1, 9, 28)])
def test_rope_only_is_bit_identical(dtype, B, L, H):
    qkv, _, grid = _inputs(B, L, H, dtype, seed=L)
    start = 37 if L > 1 else 0
    cos, sin = grid[0, 0, 0, 0, start:start + L], grid[1, 0, 0, 0, start:start + L]
    q, k, v = prepare_qkv(qkv, rope=(cos, sin))
    rq, rk, rv = _reference_prep(qkv, None, cos, sin)
    assert q.dtype == rq.dtype == torch.float32 and v.dtype == dtype
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("B,L,H", [(2, 1, 16), (2, 36, 16), (2, 1024, 16), (1, 129, 28)])
def test_cos_attention_under_autocast(rope, B, L, H):
    """cos-attention under bf16 autocast (the real model): q, k fp32 to fp32 rounding of the
    row norm; v bit-identical."""
    qkv, scale_mul, grid = _inputs(B, L, H, torch.bfloat16, seed=L + 1)
    cos = sin = None
    if rope:
        cos, sin = grid[0, 0, 0, 0, :L], grid[1, 0, 0, 0, :L]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        q, k, v = prepare_qkv(qkv, scale_mul=scale_mul, rope=None if cos is None else (cos, sin))
        rq, rk, rv = _reference_prep(qkv, scale_mul, cos, sin)
    assert q.dtype == rq.dtype == torch.float32 and k.dtype == rk.dtype == torch.float32
    assert torch.equal(v, rv)
    np.testing.assert_allclose(q.cpu().numpy(), rq.cpu().numpy(), atol=1e-6 * 100, rtol=1e-5)
    np.testing.assert_allclose(k.cpu().numpy(), rk.cpu().numpy(), atol=1e-6, rtol=1e-5)


def test_plain_permute_keeps_dtype():
    qkv, _, _ = _inputs(2, 50, 16, torch.bfloat16, seed=3)
    q, k, v = prepare_qkv(qkv)
    rq, rk, rv = _reference_prep(qkv, None, None, None)
    assert q.dtype == torch.bfloat16
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)


def test_rope_rows_slice_the_schedule():
    """rope_rows takes the rows apply_rotary_emb takes: the tokens of the earlier scales skipped."""
    schedule = [(1, 1, 1), (1, 2, 2), (1, 4, 4)]
    grid = torch.arange(2 * 21 * 64, dtype=torch.float32).reshape(2, 1, 1, 1, 21, 64)
    freqs = {str(tuple(schedule)): grid}
    cos, sin = rope_rows(freqs, schedule, 2, 16, "cuda")
    assert torch.equal(cos.cpu(), grid[0, 0, 0, 0, 5:21]) and torch.equal(sin.cpu(), grid[1, 0, 0, 0, 5:21])
    with pytest.raises(ValueError):
        rope_rows(freqs, schedule, 2, 17, "cuda")


def test_validation_errors():
    qkv = torch.zeros(1, 4, 3, 2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim=128"):
        prepare_qkv(qkv)
    qkv = torch.zeros(1, 4, 3, 2, 128, dtype=torch.bfloat16, device="cuda")
    bad = torch.zeros(4, 32, device="cuda")
    with pytest.raises(ValueError, match="rope rows"):
        prepare_qkv(qkv, rope=(bad, bad))
    with pytest.raises(ValueError, match="one value per head"):
        prepare_qkv(qkv, scale_mul=torch.ones(3, device="cuda"))
    assert _native.device_status() == 0


def _append_case(B, L, H, rope, seed):
    qkv, _, grid = _inputs(B, L, H, torch.bfloat16, seed=seed)
    rows = (grid[0, 0, 0, 0, :L], grid[1, 0, 0, 0, :L]) if rope else None
    qk_dtype = torch.float32 if rope else torch.bfloat16
    cap = 3 * H * L + 11
    slab_k = torch.full((B, cap, 128), 7.0, dtype=qk_dtype, device="cuda")
    slab_v = torch.full((B, cap, 128), -7.0, dtype=torch.bfloat16, device="cuda")
    return qkv, rows, slab_k, slab_v, cap


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("B,L,H", [(2, 1, 16), (2, 36, 16), (1, 576, 28)])
def test_append_writes_the_given_heads_into_the_slab(rope, B, L, H):
    """``append=``: head h's k/v rows land in slab[:, offsets[h] + l] bit for bit, heads with
    offset -1 and every other slot keep their contents, and q/k/v are those of the plain call."""
    qkv, rows, slab_k, slab_v, cap = _append_case(B, L, H, rope, seed=L + H)
    offs = np.full(H, -1, dtype=np.int64)
    for j, h in enumerate(range(0, H, 3)):
        offs[h] = 11 + (2 * j + 1) * L  # disjoint segments, gaps between them
    offsets = torch.from_numpy(offs).cuda()
    want_k, want_v = slab_k.clone(), slab_v.clone()
    q, k, v = prepare_qkv(qkv, rope=rows, append=(slab_k, slab_v, offsets))
    rq, rk, rv = prepare_qkv(qkv, rope=rows)
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
    for h in range(H):
        if offs[h] >= 0:
            want_k[:, offs[h]:offs[h] + L] = k[:, h]
            want_v[:, offs[h]:offs[h] + L] = v[:, h]
    assert torch.equal(slab_k, want_k) and torch.equal(slab_v, want_v)
    assert _native.device_status() == 0


def test_append_outside_the_slab_is_skipped_and_flagged():
    """A segment that would leave the slab is not written (the other heads are) and raises
    HEATKV_DEVICE_PACK_OUT_OF_RANGE (0x1)."""
    B, L, H = 2, 36, 16
    qkv, rows, slab_k, slab_v, cap = _append_case(B, L, H, False, seed=4)
    offs = np.full(H, -1, dtype=np.int64)
    offs[2], offs[5] = 0, cap - L + 1
    want_k, want_v = slab_k.clone(), slab_v.clone()
    _, k, v = prepare_qkv(qkv, append=(slab_k, slab_v, torch.from_numpy(offs).cuda()))
    want_k[:, :L] = k[:, 2]
    want_v[:, :L] = v[:, 2]
    assert _native.device_status() == 0x1
    assert torch.equal(slab_k, want_k) and torch.equal(slab_v, want_v)


def test_append_validation():
    qkv = torch.zeros(1, 4, 3, 2, 128, dtype=torch.bfloat16, device="cuda")
    sk = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    offs = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="dtypes"):
        prepare_qkv(qkv, rope=(torch.zeros(4, 64, device="cuda"),) * 2, append=(sk, sk, offs))
    with pytest.raises(ValueError, match="int64"):
        prepare_qkv(qkv, append=(sk, sk, offs.int()))
    with pytest.raises(ValueError, match="capacity"):
        prepare_qkv(qkv, append=(sk, sk[:, :4, :64], offs))
    assert _native.device_status() == 0
