"""The fused QKV projection (``heatkv_qkv_project``: tcgen05 GEMM with the q/k/v preparation and
the cache append in its epilogue) against the unfused path it replaces: the projection by torch
(cuBLAS, rounded to the 16-bit dtype), then ``heatkv_qkv_prepare_append``. Only the summation
order of the projection and of the row norms differ, so an element may land one 16-bit rounding
step away; tolerance: max |err| <= 1e-2 * max |ref| per tensor, and at least 99 % of the elements
bit-identical. Cache rows are written for exactly the heads given an offset, and an offset past
the cache is skipped and flagged."""

import ctypes

import pytest
import torch

from heatkv_b200 import _native
from heatkv_b200.qkv_prep import prepare_qkv, rope_pair_groups

pytestmark = pytest.mark.gpu


def _project(x, w, B, L, H, scale_mul=None, rope=None, cache=None, bias=None, qk_dtype=None):
    lib = _native.load()
    dev = x.device
    qk_dtype = x.dtype if qk_dtype is None else qk_dtype
    q, k = (torch.empty(B, H, L, 128, dtype=qk_dtype, device=dev) for _ in range(2))
    v = torch.empty(B, H, L, 128, dtype=x.dtype, device=dev)
    cos = sin = None
    if rope is not None:
        cos, sin = (rope_pair_groups(t) for t in rope)
    ck, cv, rows, offs = cache if cache is not None else (None, None, 0, None)
    _native.check(lib.heatkv_qkv_project(
        _native.ptr(x), _native.ptr(w), _native.ptr(bias), _native.ptr(q), _native.ptr(k),
        _native.ptr(v), _native.DTYPE_CODES[x.dtype], _native.DTYPE_CODES[qk_dtype], B, L, H,
        x.shape[-1], _native.ptr(scale_mul),
        ctypes.c_float(1e-12), _native.ptr(cos), _native.ptr(sin),
        0 if cos is None else 4 * cos.shape[1], _native.ptr(ck), _native.ptr(cv), rows,
        _native.ptr(offs), _native.stream_handle(dev)), "heatkv_qkv_project")
    return q, k, v


def _close(a, b):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    same = (a == b).float().mean().item()
    return err <= 1e-2 * max(b.abs().max().item(), 1e-6) and same >= 0.99, (err, same)


def _close32(a, b):
    """fp32 q/k: elements whose 16-bit projection rounded alike agree to fp32 rounding (the row
    norm's summation order and reciprocal differ), the rest by a 16-bit rounding step."""
    a, b = a.float(), b.float()
    err = (a - b).abs()
    near = (err <= 1e-5 * b.abs().max().clamp_min(1e-6)).float().mean().item()
    return err.max().item() <= 1e-2 * max(b.abs().max().item(), 1e-6) and near >= 0.99, (
        err.max().item(), near)


@pytest.mark.parametrize("dtype,B,L,H,C,cos_attn,rope", [
    (torch.bfloat16, 2, 400, 16, 2048, True, True),
    (torch.bfloat16, 3, 64, 2, 512, True, False),
    (torch.float16, 1, 257, 4, 256, False, True),
    (torch.bfloat16, 2, 1, 16, 2048, False, False),
])
@pytest.mark.parametrize("qk32", [False, True])
def test_fused_projection_matches_gemm_then_prepare(dtype, B, L, H, C, cos_attn, rope, qk32):
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(L + H)
    x = torch.randn(B, L, C, device=dev, generator=g).to(dtype)
    w = (torch.randn(3 * H * 128, C, device=dev, generator=g) * 0.02).to(dtype)
    sm = torch.rand(H, device=dev, generator=g) * 4 + 1 if cos_attn else None
    rp = None
    if rope:
        ang = torch.rand(L, 64, device=dev, generator=g) * 6
        rp = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
    rows = H * L + 300
    qkd = torch.float32 if qk32 else dtype
    ref_ck = torch.full((B, rows, 128), float("nan"), dtype=qkd, device=dev)
    ref_cv = torch.full((B, rows, 128), float("nan"), dtype=dtype, device=dev)
    ck, cv = ref_ck.clone(), ref_cv.clone()
    offs = torch.tensor([h * L + 7 if h % 3 != 1 else -1 for h in range(H)], dtype=torch.int64,
                        device=dev)
    qkv = torch.mm(x.view(B * L, C), w.t()).view(B, L, 3, H, 128)
    rq, rk, rv = prepare_qkv(qkv, scale_mul=sm, rope=rp, qk_dtype=qkd,
                             append=(ref_ck, ref_cv, offs))
    q, k, v = _project(x.view(B * L, C), w, B, L, H, sm, rp, (ck, cv, rows, offs), qk_dtype=qkd)
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    assert q.dtype == rq.dtype == qkd and v.dtype == rv.dtype == dtype
    for name, a, b in (("q", q, rq), ("k", k, rk), ("v", v, rv)):
        ok, info = (_close32 if a.dtype == torch.float32 else _close)(a, b)
        assert ok, (name, info)
    written = torch.zeros(rows, dtype=torch.bool, device=dev)
    for h in range(H):
        if offs[h] >= 0:
            written[offs[h]:offs[h] + L] = True
    assert torch.isnan(ck[:, ~written].float()).all() and torch.isnan(cv[:, ~written].float()).all()
    for a, b in ((ck, ref_ck), (cv, ref_cv)):
        ok, info = (_close32 if a.dtype == torch.float32 else _close)(a[:, written], b[:, written])
        assert ok, info


def test_fused_projection_flags_a_cache_offset_past_the_end():
    dev = torch.device("cuda", 0)
    B, L, H, C = 1, 64, 2, 256
    x = torch.randn(B * L, C, device=dev).bfloat16()
    w = (torch.randn(3 * H * 128, C, device=dev) * 0.02).bfloat16()
    rows = 100
    ck = torch.zeros(B, rows, 128, dtype=torch.bfloat16, device=dev)
    cv = torch.zeros_like(ck)
    offs = torch.tensor([0, rows - L + 1], dtype=torch.int64, device=dev)   # head 1 leaves
    _project(x, w, B, L, H, cache=(ck, cv, rows, offs))
    torch.cuda.synchronize()
    assert _native.device_status(dev) == _native.DEVICE_PACK_OUT_OF_RANGE
    assert (ck[:, L:] == 0).all() and (ck[:, :L] != 0).any()


def test_fused_projection_adds_the_bias():
    """``bias`` = cat(q_bias, zero_k_bias, v_bias) as the reference's F.linear adds it
    (enable_real_pruning_fast.py:2040-2043), against cuBLAS addmm then the preparation."""
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    dev = torch.device("cuda", 0)
    B, L, H, C = 2, 100, 4, 512
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(B * L, C, device=dev, generator=g).bfloat16()
    w = (torch.randn(3 * H * 128, C, device=dev, generator=g) * 0.02).bfloat16()
    qb, vb = (torch.randn(H * 128, device=dev, generator=g) * 0.5 for _ in range(2))
    bias = torch.cat((qb, torch.zeros_like(qb), vb)).bfloat16()
    sm = torch.rand(H, device=dev, generator=g) * 4 + 1
    ang = torch.rand(L, 64, device=dev, generator=g) * 6
    rp = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
    qkv = torch.addmm(bias, x, w.t()).view(B, L, 3, H, 128)
    rq, rk, rv = prepare_qkv(qkv, scale_mul=sm, rope=rp, qk_dtype=torch.bfloat16)
    q, k, v = _project(x, w, B, L, H, sm, rp, bias=bias.float().contiguous())
    torch.cuda.synchronize()
    assert _native.device_status(dev) == 0
    for name, a, b in (("q", q, rq), ("k", k, rk), ("v", v, rv)):
        ok, info = _close(a, b)
        assert ok, (name, info)
    # without the bias the v rows differ by it
    _, _, v0 = _project(x, w, B, L, H, sm, rp)
    assert not _close(v0, rv)[0]
