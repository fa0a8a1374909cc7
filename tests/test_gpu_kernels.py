"""GPU parity of the libheatkv kernels (run with ``pytest -m gpu`` on a B200).

Attention: tcgen05 (bf16/fp16, and fp32 q/k with 16-bit v through tf32 scores) and exact (every
dtype) kernels against the float64 CPU oracle on the seeded edge cases, against the outputs
recorded from the reference itself, and on larger random segment layouts against a plain PyTorch
fp32 reference on the GPU. Tolerances: bf16/fp16 and tf32 max |err| <= 2e-2 and max |err| /
max |ref| <= 1e-2; fp32 (exact kernel) 1e-5.
Pack: bit-exact against the oracle for random descriptors and mixed K/V dtypes; out-of-range
descriptors are skipped and flagged.
"""

import hashlib
import math
import os

import numpy as np
import pytest
import torch

from heatkv_b200 import _native, synthetic
from heatkv_b200.real_pruning_fused_attention import (
    fused_real_pruning_flat_segmented_attention as attn,
    pack_flat_segments_kv as pack,
)
from heatkv_b200.scheduler import build_static_slot_schedule, copy_descriptors
from oracle.attention import segmented_attention as oracle_attention
from oracle.pack import pack_flat_segments as oracle_pack

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_REL = 2e-2, 1e-2
FP32_ATOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def cuda_device():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    _native.load()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)


@pytest.fixture
def kernel(monkeypatch):
    def set_kernel(name):
        monkeypatch.setenv("HEATKV_ATTENTION_KERNEL", name)
    return set_kernel


def _to(inputs, dev):
    out = {}
    for k, v in inputs.items():
        out[k] = v.to(dev) if isinstance(v, torch.Tensor) else v
    return out


def _check_lowp(out, ref):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(out - ref).max()
    scale = max(np.abs(ref).max(), 1e-30)
    assert err <= BF16_ATOL, f"max abs err {err}"
    assert err / scale <= BF16_REL, f"relative err {err / scale}"


@pytest.mark.parametrize("case", synthetic.ATTENTION_CASES, ids=lambda c: c.name)
@pytest.mark.parametrize("which", ["auto", "exact"])
def test_attention_cases(case, which, cuda_device, kernel, golden_dir):
    kernel(which)
    inputs = synthetic.attention_case_inputs(case)
    ref = oracle_attention(**inputs)
    out = attn(**_to(inputs, cuda_device)).float().cpu().numpy()
    golden = np.load(os.path.join(golden_dir, "attention_cases.npz"))[case.name]
    if case.dtype == "bf16":
        golden = torch.from_numpy(golden).view(torch.bfloat16).float().numpy()
    if case.dtype == "f32":
        np.testing.assert_allclose(out, ref, atol=FP32_ATOL, rtol=FP32_ATOL)
        np.testing.assert_allclose(out, golden, atol=FP32_ATOL, rtol=FP32_ATOL)
    else:
        _check_lowp(out, ref)
        _check_lowp(out, golden)
    assert _native.device_status(cuda_device) == 0


def _torch_reference(q, pk, pv, starts, ends, counts, ck, cv, scale):
    """Plain PyTorch fp32 reference on the GPU (gather the head's slab rows, then softmax)."""
    B, H, L, D = q.shape
    out = torch.empty(B, L, H, D, dtype=torch.float32, device=q.device)
    st, en, ct = starts.cpu(), ends.cpu(), counts.cpu()
    for h in range(H):
        idx = [torch.arange(int(st[h, i]), int(en[h, i])) for i in range(int(ct[h]))
               if int(st[h, i]) < int(en[h, i])]
        idx = torch.cat(idx).to(q.device) if idx else torch.zeros(0, dtype=torch.long, device=q.device)
        keys = torch.cat([pk[:, idx].float(), ck[:, h].float()], dim=1)  # [B, S+L, D]
        vals = torch.cat([pv[:, idx].float(), cv[:, h].float()], dim=1)
        s = torch.einsum("bld,bsd->bls", q[:, h].float(), keys) * scale
        out[:, :, h] = torch.softmax(s, dim=-1) @ vals
    return out.reshape(B, L, H * D)


def _random_layout(rng, heads, max_segments, capacity, lengths=(1, 4, 16, 36, 64, 127, 128, 129, 300, 576)):
    starts = np.zeros((heads, max_segments), np.int32)
    ends = np.zeros((heads, max_segments), np.int32)
    counts = np.zeros((heads,), np.int32)
    for h in range(heads):
        c = int(rng.integers(0, max_segments + 1))
        counts[h] = c
        for i in range(c):
            n = min(int(rng.choice(lengths)), capacity)
            s = int(rng.integers(0, capacity - n + 1))
            starts[h, i], ends[h, i] = s, s + n
    return [torch.from_numpy(x) for x in (starts, ends, counts)]


@pytest.mark.parametrize("which", ["tcgen05_cs", "tcgen05_cs64"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,L,cap,S", [
    (1, 1, 1, 700, 3), (2, 3, 4, 400, 4), (1, 2, 127, 900, 5), (2, 2, 128, 900, 5),
    (1, 3, 129, 1200, 6), (2, 2, 255, 800, 4), (1, 2, 256, 900, 6), (2, 1, 257, 1500, 8),
    (2, 16, 576, 4000, 12), (1, 4, 1024, 3000, 12),
])
def test_tcgen05_random_layouts(which, dtype, B, H, L, cap, S, cuda_device, kernel):
    """Both 16-bit tcgen05 kernels: the 64-key one (two CTAs per SM, the default) and the
    column-split one."""
    kernel(which)
    rng = np.random.default_rng(B * 1000 + H * 100 + L)
    gen = torch.Generator().manual_seed(L)
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).to(dtype).to(cuda_device) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).to(dtype).to(cuda_device) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, cap)
    scale = 1.0 / math.sqrt(128)
    out = attn(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st.to(cuda_device),
               segment_ends=en.to(cuda_device), segment_counts=ct.to(cuda_device),
               current_k=ck, current_v=cv, softmax_scale=scale)
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(cuda_device) == 0


@pytest.mark.parametrize("which", ["tcgen05_cs", "tcgen05_cs64"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L", [5, 200, 300])
def test_tcgen05_scores_growing_tile_by_tile(which, dtype, L, cuda_device, kernel):
    """Each key tile's scores far above the previous tiles' (the running max rises by more than
    the lazy-rescale threshold again and again, so P is recomputed and O rescaled), with query
    rows of other heads in the last Q tile."""
    kernel(which)
    B, H, S, cap = 2, 3, 5, 5 * 128
    gen = torch.Generator().manual_seed(L + 7)
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen) for _ in range(2))
    growth = torch.repeat_interleave(1.0 + 2.5 * torch.arange(S, dtype=torch.float32), 128)
    pk = pk * growth[None, :, None]
    ck = ck * (1.0 + 2.5 * S)
    st = torch.tensor([[128 * i for i in range(S)]] * H, dtype=torch.int32)
    en = st + 128
    en[1, S - 1] = 128 * (S - 1) + 77   # a partial tile in the middle of head 1
    ct = torch.tensor([S, S, 2], dtype=torch.int32)
    q, ck, cv, pk, pv = (x.to(dtype).to(cuda_device) for x in (q, ck, cv, pk, pv))
    scale = 1.0 / math.sqrt(128)
    out = attn(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st.to(cuda_device),
               segment_ends=en.to(cuda_device), segment_counts=ct.to(cuda_device),
               current_k=ck, current_v=cv, softmax_scale=scale)
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(cuda_device) == 0


@pytest.mark.parametrize("L,cap,S", [(1, 300, 3), (64, 700, 6), (130, 900, 5), (300, 1500, 8)])
def test_exact_fp32_random_layouts(L, cap, S, cuda_device, kernel):
    kernel("auto")  # fp32 inputs always take the exact kernel
    rng = np.random.default_rng(L)
    gen = torch.Generator().manual_seed(L + 1)
    B, H = 2, 3
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, cap)
    scale = 1.0 / math.sqrt(128)
    ref = oracle_attention(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st, segment_ends=en,
                           segment_counts=ct, current_k=ck, current_v=cv, softmax_scale=scale)
    d = cuda_device
    out = attn(q=q.to(d), persisted_k=pk.to(d), persisted_v=pv.to(d), segment_starts=st.to(d),
               segment_ends=en.to(d), segment_counts=ct.to(d), current_k=ck.to(d),
               current_v=cv.to(d), softmax_scale=scale)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=FP32_ATOL, rtol=FP32_ATOL)


def test_exact_mixed_dtypes_real_model_layout(cuda_device, kernel):
    """q, k fp32 and v bf16: the dtypes of the real model (cos-attn under bf16 autocast), on the
    exact kernel (what REAL_PRUNING_FUSED_QK_DOT_MODE=fp32 selects)."""
    kernel("exact")
    rng = np.random.default_rng(7)
    gen = torch.Generator().manual_seed(7)
    B, H, L, cap = 2, 4, 100, 600
    q, ck = (torch.randn(B, H, L, 128, generator=gen) for _ in range(2))
    cv = torch.randn(B, H, L, 128, generator=gen).bfloat16()
    pk = torch.randn(B, cap, 128, generator=gen)
    pv = torch.randn(B, cap, 128, generator=gen).bfloat16()
    st, en, ct = _random_layout(rng, H, 5, cap)
    ref = oracle_attention(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st, segment_ends=en,
                           segment_counts=ct, current_k=ck, current_v=cv, softmax_scale=0.09)
    d = cuda_device
    out = attn(q=q.to(d), persisted_k=pk.to(d), persisted_v=pv.to(d), segment_starts=st.to(d),
               segment_ends=en.to(d), segment_counts=ct.to(d), current_k=ck.to(d),
               current_v=cv.to(d), softmax_scale=0.09)
    assert out.dtype == torch.float32
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=FP32_ATOL, rtol=FP32_ATOL)


@pytest.mark.parametrize("vdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,L,cap,S", [
    (1, 1, 1, 700, 3), (2, 3, 4, 400, 4), (1, 2, 127, 900, 5), (2, 2, 128, 900, 5),
    (1, 3, 129, 1200, 6), (2, 2, 255, 800, 4), (2, 1, 257, 1500, 8), (2, 16, 576, 4000, 12),
    (1, 4, 1024, 3000, 12), (2, 3, 64, 0, 0),
])
def test_tcgen05_tf32_mixed_dtypes(vdtype, B, H, L, cap, S, cuda_device, kernel):
    """fp32 q and k with 16-bit v on the tf32 tcgen05 kernel (the reference's default dot modes on
    these dtypes: tf32 scores, P rounded to v's dtype); the output is fp32."""
    kernel("tcgen05")
    rng = np.random.default_rng(B * 1000 + H * 100 + L + 5)
    gen = torch.Generator().manual_seed(L + 5)
    q, ck = (torch.randn(B, H, L, 128, generator=gen).to(cuda_device) for _ in range(2))
    cv = torch.randn(B, H, L, 128, generator=gen).to(vdtype).to(cuda_device)
    pk = torch.randn(B, cap, 128, generator=gen).to(cuda_device)
    pv = torch.randn(B, cap, 128, generator=gen).to(vdtype).to(cuda_device)
    if cap:
        st, en, ct = _random_layout(rng, H, S, cap)
    else:
        st = en = torch.zeros(H, 0, dtype=torch.int32)
        ct = torch.zeros(H, dtype=torch.int32)
    scale = 1.0 / math.sqrt(128)
    out = attn(q=q, persisted_k=pk if cap else None, persisted_v=pv if cap else None,
               segment_starts=st.to(cuda_device), segment_ends=en.to(cuda_device),
               segment_counts=ct.to(cuda_device), current_k=ck, current_v=cv, softmax_scale=scale)
    assert out.dtype == torch.float32
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    _check_lowp(out.cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(cuda_device) == 0


def test_64_key_kernel_rejects_fp32_queries(cuda_device, kernel):
    """The 64-key kernel asked for by name takes only all-bf16 or all-f16 inputs."""
    kernel("tcgen05_cs64")
    d = cuda_device
    q, ck = (torch.randn(1, 2, 8, 128, device=d) for _ in range(2))
    cv = torch.randn(1, 2, 8, 128, device=d).bfloat16()
    z = torch.zeros(2, 0, dtype=torch.int32, device=d)
    with pytest.raises(RuntimeError, match="64-key"):
        attn(q=q, persisted_k=None, persisted_v=None, segment_starts=z, segment_ends=z,
             segment_counts=torch.zeros(2, dtype=torch.int32, device=d), current_k=ck,
             current_v=cv, softmax_scale=0.1)


@pytest.mark.parametrize("L", [5, 200, 300])
def test_tcgen05_tf32_scores_growing_tile_by_tile(L, cuda_device, kernel):
    """The lazy-rescale path of the tf32 kernel: every key tile's scores far above the previous
    tiles', both key halves of a tile exchanged between the softmax warpgroups, a partial tile in
    the middle of a head and query rows past Lq in the last block."""
    kernel("tcgen05")
    B, H, S, cap = 2, 3, 5, 5 * 128
    gen = torch.Generator().manual_seed(L + 11)
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen) for _ in range(2))
    growth = torch.repeat_interleave(1.0 + 2.5 * torch.arange(S, dtype=torch.float32), 128)
    pk = pk * growth[None, :, None]
    ck = ck * (1.0 + 2.5 * S)
    st = torch.tensor([[128 * i for i in range(S)]] * H, dtype=torch.int32)
    en = st + 128
    en[1, S - 1] = 128 * (S - 1) + 77
    en[2, 0] = 40   # keys only in the first half of head 2's first tile
    ct = torch.tensor([S, S, 2], dtype=torch.int32)
    d = cuda_device
    q, ck, pk = (x.to(d) for x in (q, ck, pk))
    cv, pv = (x.bfloat16().to(d) for x in (cv, pv))
    scale = 1.0 / math.sqrt(128)
    out = attn(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st.to(d),
               segment_ends=en.to(d), segment_counts=ct.to(d),
               current_k=ck, current_v=cv, softmax_scale=scale)
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    _check_lowp(out.cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(cuda_device) == 0


@pytest.mark.parametrize("kd,vd", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.bfloat16),
                                   (torch.float16, torch.float32)])
def test_pack_random_descriptors(kd, vd, cuda_device):
    rng = np.random.default_rng(3)
    B, H, S, cap, D = 3, 5, 150, 2000, 128
    gen = torch.Generator().manual_seed(3)
    src_k = torch.randn(B, H * S, D, generator=gen).to(kd)
    src_v = torch.randn(B, H * S, D, generator=gen).to(vd)
    dst_k = torch.randn(B, cap, D, generator=gen).to(kd)
    dst_v = torch.randn(B, cap, D, generator=gen).to(vd)
    # non-overlapping destination runs of assorted lengths (1 .. S)
    lengths = rng.integers(1, S + 1, size=9)
    dst = np.cumsum(np.concatenate([[0], lengths[:-1] + rng.integers(0, 7, size=8)]))
    src = np.array([int(rng.integers(0, H)) * S + int(rng.integers(0, S - n + 1)) for n in lengths])
    exp_k, exp_v = dst_k.clone(), dst_v.clone()
    oracle_pack(exp_k.view(torch.int16 if kd != torch.float32 else torch.int32).numpy(),
                exp_v.view(torch.int16 if vd != torch.float32 else torch.int32).numpy(),
                src_k.view(torch.int16 if kd != torch.float32 else torch.int32).numpy(),
                src_v.view(torch.int16 if vd != torch.float32 else torch.int32).numpy(),
                dst, src, lengths)
    d = cuda_device
    gk, gv = dst_k.to(d), dst_v.to(d)
    pack(dst_k=gk, dst_v=gv, src_k=src_k.to(d), src_v=src_v.to(d),
         dst_starts=torch.from_numpy(dst).to(d), src_starts=torch.from_numpy(src).to(d),
         lengths=torch.from_numpy(lengths).to(d))
    assert torch.equal(gk.cpu(), exp_k) and torch.equal(gv.cpu(), exp_v)
    assert _native.device_status(d) == 0


def test_pack_out_of_range_item_is_skipped_and_flagged(cuda_device):
    d = cuda_device
    src = torch.arange(2 * 10 * 128, dtype=torch.float32, device=d).reshape(2, 10, 128)
    dst_k = torch.zeros(2, 20, 128, device=d)
    dst_v = torch.zeros(2, 20, 128, device=d)
    pack(dst_k=dst_k, dst_v=dst_v, src_k=src, src_v=src,
         dst_starts=torch.tensor([0, 18], device=d), src_starts=torch.tensor([2, 0], device=d),
         lengths=torch.tensor([3, 5], device=d))  # second item would end at row 23 > 20
    assert torch.equal(dst_k[:, :3], src[:, 2:5])
    assert torch.count_nonzero(dst_k[:, 3:]) == 0
    assert _native.device_status(d) & _native.DEVICE_PACK_OUT_OF_RANGE
    assert _native.device_status(d) == 0  # cleared by the previous read


def _sha(t):
    return list(hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).digest())


def test_config1_pipeline_against_reference(cuda_device, golden_dir):
    """Activation pack, per-scale appends and fused attention of config 1 on the GPU reproduce the
    reference's slab bytes (SHA-256) and attention outputs (fp32, 1e-5)."""
    from test_host_golden import config1_controller

    cfg, ctrl = config1_controller()
    sched = build_static_slot_schedule(ctrl, layer_idx=0, num_heads=cfg.num_heads)
    pk_golden = np.load(os.path.join(golden_dir, "pack_c1.npz"))["digests"].tolist()
    ga = np.load(os.path.join(golden_dir, "attention_c1.npz"))
    d = cuda_device
    qkv = [tuple(x.to(d) for x in s) for s in synthetic.config1_qkv(cfg)]
    first = synthetic.first_pruned_target(ctrl.removed_heads_by_source_for, len(qkv))
    cap = sched["capacity"]
    slab_k = torch.zeros(cfg.batch, cap, 128, device=d)
    slab_v = torch.zeros_like(slab_k)

    def run_pack(runs, k, v):
        desc = copy_descriptors(runs)
        B, H, T, D = k.shape
        pack(dst_k=slab_k, dst_v=slab_v, src_k=k.reshape(B, H * T, D), src_v=v.reshape(B, H * T, D),
             dst_starts=torch.from_numpy(desc["dst_starts"]).to(d),
             src_starts=torch.from_numpy(desc["src_starts"]).to(d),
             lengths=torch.from_numpy(desc["lengths"]).to(d), max_length=desc["max_length"])

    dense_k = torch.cat([qkv[s][1] for s in range(first)], dim=2)
    dense_v = torch.cat([qkv[s][2] for s in range(first)], dim=2)
    run_pack(sched["old_pack_runs_by_target"][first], dense_k, dense_v)
    assert [first, -1] + _sha(slab_k) + _sha(slab_v) == pk_golden[0]
    step = 1
    for t in range(first, len(qkv)):
        q, k, v = qkv[t]
        st, en, ct = (torch.from_numpy(x).to(d) for x in sched["metadata_cpu_by_target"][t])
        out = attn(q=q, persisted_k=slab_k, persisted_v=slab_v, segment_starts=st, segment_ends=en,
                   segment_counts=ct, current_k=k, current_v=v, softmax_scale=cfg.softmax_scale)
        o = out.cpu().numpy()
        np.testing.assert_allclose(o[:, :4, :], ga[f"t{t}_head_rows"], atol=FP32_ATOL, rtol=FP32_ATOL)
        np.testing.assert_allclose(synthetic.output_checksums(o), ga[f"t{t}_checksums"],
                                   rtol=1e-5, atol=1e-3)
        if t + 1 < len(qkv):
            run_pack(sched["append_runs_by_key"][(t, t + 1)], k, v)
            assert [t, t + 1] + _sha(slab_k) + _sha(slab_v) == pk_golden[step]
            step += 1
    assert _native.device_status(d) == 0


def _attention_ws(q, pk, pv, st, en, ct, ck, cv, scale, *, head_order, splits, workspace,
                  kernel=_native.ATTN_TCGEN05):
    import ctypes
    lib = _native.load()
    B, H, L, D = q.shape
    out = torch.empty(B, L, H * D, dtype=q.dtype, device=q.device)
    dt = _native.DTYPE_CODES
    status = lib.heatkv_segmented_attention_ws(
        _native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
        _native.ptr(ct), _native.ptr(ck), _native.ptr(cv), _native.ptr(out), dt[q.dtype],
        dt[ck.dtype], dt[cv.dtype], B, H, L, pk.shape[1], D, st.shape[1], ctypes.c_float(scale), 0,
        kernel, _native.ptr(head_order), splits, _native.ptr(workspace),
        0 if workspace is None else workspace.numel(), _native.stream_handle(q.device))
    _native.check(status, "heatkv_segmented_attention_ws")
    return out


SPLIT_KERNELS = {"cs": (_native.ATTN_TCGEN05_CS, 128), "cs64": (_native.ATTN_TCGEN05_CS64, 128)}


@pytest.mark.parametrize("variant", sorted(SPLIT_KERNELS))
@pytest.mark.parametrize("splits", [1, 2, 3, 4])
@pytest.mark.parametrize("B,H,L,cap,S", [(1, 3, 129, 1500, 6), (2, 4, 576, 3000, 10),
                                         (2, 16, 1600, 5000, 12), (1, 2, 20, 900, 4)])
def test_tcgen05_split_kv_and_head_order(variant, splits, B, H, L, cap, S, cuda_device):
    """Split-KV partials merged by the last CTA and a shuffled head order give the same result as
    the reference, in both tcgen05 kernels (blocks of 128 query rows); splits without key
    tiles (heads with fewer tiles than splits) contribute nothing; the workspace counters are back
    to zero after every call."""
    kern, block_rows = SPLIT_KERNELS[variant]
    rng = np.random.default_rng(splits * 7 + L)
    gen = torch.Generator().manual_seed(L + splits)
    d = cuda_device
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, cap)
    order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
    lib = _native.load()
    nbytes = int(lib.heatkv_attention_workspace_bytes(B, H, L, splits))
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=d)
    scale = 1.0 / math.sqrt(128)
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    for _ in range(2):  # second call reuses the workspace the first one left zeroed
        out = _attention_ws(q, pk, pv, st.to(d), en.to(d), ct.to(d), ck, cv, scale,
                            head_order=order, splits=splits, workspace=ws, kernel=kern)
        _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    if splits > 1:
        blocks = B * H * ((L + block_rows - 1) // block_rows)
        assert int(ws[: 4 * blocks].count_nonzero()) == 0, "split counters not reset"
    assert _native.device_status(d) == 0


@pytest.mark.parametrize("variant", sorted(SPLIT_KERNELS))
@pytest.mark.parametrize("B,H,L,cap,S,splits", [(2, 16, 1600, 5000, 12, 2), (2, 4, 576, 3000, 10, 2),
                                                (1, 8, 4096, 2000, 6, 3)])
def test_tcgen05_tail_split_schedule(variant, B, H, L, cap, S, splits, cuda_device):
    """heatkv_segmented_attention_sched: only the blocks after the first `unsplit` (schedule
    order, blocks of the kernel's 128 query rows) are split; every choice of unsplit gives
    the reference's result, and the unsplit blocks are bit-identical to an unsplit launch."""
    kern, block_rows = SPLIT_KERNELS[variant]
    import ctypes
    rng = np.random.default_rng(L + H)
    gen = torch.Generator().manual_seed(L + 3)
    d = cuda_device
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, cap)
    st, en, ct = st.to(d), en.to(d), ct.to(d)
    order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
    lib = _native.load()
    nbytes = int(lib.heatkv_attention_workspace_bytes(B, H, L, splits))
    ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=d)
    scale = 1.0 / math.sqrt(128)
    ref = _torch_reference(q, pk, pv, st.cpu(), en.cpu(), ct.cpu(), ck, cv, scale)
    whole = _attention_ws(q, pk, pv, st, en, ct, ck, cv, scale, head_order=order, splits=1,
                          workspace=None, kernel=kern)
    qpairs = (L + block_rows - 1) // block_rows
    blocks = B * H * qpairs
    dt = _native.DTYPE_CODES
    for unsplit in (0, 1, blocks // 2, blocks - 3, blocks):
        out = torch.full((B, L, H * 128), float("nan"), dtype=q.dtype, device=d)
        status = lib.heatkv_segmented_attention_sched(
            _native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
            _native.ptr(ct), _native.ptr(ck), _native.ptr(cv), _native.ptr(out), dt[q.dtype],
            dt[ck.dtype], dt[cv.dtype], B, H, L, cap, 128, S, ctypes.c_float(scale),
            kern, _native.ptr(order), splits, unsplit, _native.ptr(ws),
            ws.numel(), _native.stream_handle(d))
        _native.check(status, "heatkv_segmented_attention_sched")
        torch.cuda.synchronize()
        _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
        # blocks [0, unsplit) in schedule order = (head rank, row, query block): same bits
        for blk in range(unsplit):
            rank, qp = divmod(blk, qpairs)
            rank, b = divmod(rank, B)
            h = int(order[rank])
            rows = slice(qp * block_rows, min(L, (qp + 1) * block_rows))
            cols = slice(h * 128, (h + 1) * 128)
            assert torch.equal(out[b, rows, cols], whole[b, rows, cols]), (unsplit, blk)
        assert int(ws[: 4 * blocks].count_nonzero()) == 0, "split counters not reset"
    assert _native.device_status(d) == 0


@pytest.mark.parametrize("variant", sorted(SPLIT_KERNELS))
def test_workspace_shared_across_shapes(variant, cuda_device):
    """One workspace serves calls of different shapes in any order (the split counters sit in a
    region no partial result ever overwrites)."""
    kern = SPLIT_KERNELS[variant][0]
    d = cuda_device
    lib = _native.load()
    shapes = [(2, 4, 576, 3000, 10, 3), (2, 16, 1600, 5000, 12, 2), (1, 3, 129, 1500, 6, 5),
              (2, 16, 1024, 4000, 12, 4)]
    need = max(int(lib.heatkv_attention_workspace_bytes(B, H, L, sp)) for B, H, L, _, _, sp in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device=d)
    scale = 1.0 / math.sqrt(128)
    for rep in range(2):
        for k, (B, H, L, cap, S, sp) in enumerate(shapes):
            rng = np.random.default_rng(100 * rep + k)
            gen = torch.Generator().manual_seed(100 * rep + k)
            q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
            pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
            st, en, ct = _random_layout(rng, H, S, cap)
            order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
            out = _attention_ws(q, pk, pv, st.to(d), en.to(d), ct.to(d), ck, cv, scale,
                                head_order=order, splits=sp, workspace=ws, kernel=kern)
            ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
            _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(d) == 0


@pytest.mark.parametrize("which,dtype", [("tcgen05", torch.bfloat16), ("exact", torch.bfloat16),
                                         ("exact", torch.float32)])
def test_slab_rows_outside_segments_are_never_used(which, dtype, cuda_device, kernel):
    """Slab slots no segment covers may hold anything (the slab is uninitialised memory); rows a
    128-key tile loads past a segment's end must not reach the output even when they are NaN."""
    kernel(which)
    rng = np.random.default_rng(5)
    gen = torch.Generator().manual_seed(5)
    B, H, L, cap, S = 2, 4, 200, 1500, 6
    d = cuda_device
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).to(dtype).to(d) for _ in range(3))
    st, en, ct = _random_layout(rng, H, S, cap, lengths=(1, 5, 36, 100, 129, 250))
    pk = torch.full((B, cap, 128), float("nan"), dtype=dtype)
    pv = torch.full((B, cap, 128), float("nan"), dtype=dtype)
    for h in range(H):
        for i in range(int(ct[h])):
            s0, e0 = int(st[h, i]), int(en[h, i])
            pk[:, s0:e0] = torch.randn(B, e0 - s0, 128, generator=gen).to(dtype)
            pv[:, s0:e0] = torch.randn(B, e0 - s0, 128, generator=gen).to(dtype)
    pk, pv = pk.to(d), pv.to(d)
    scale = 1.0 / math.sqrt(128)
    out = attn(q=q, persisted_k=pk, persisted_v=pv, segment_starts=st.to(d), segment_ends=en.to(d),
               segment_counts=ct.to(d), current_k=ck, current_v=cv, softmax_scale=scale)
    assert torch.isfinite(out).all()
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, scale)
    if dtype == torch.float32:
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=FP32_ATOL, rtol=FP32_ATOL)
    else:
        _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())


def _attention_mapped(q, pk, pv, st, en, ct, ck, cv, scale, *, order, splits, unsplit, item_map,
                      grid, workspace, kernel=_native.ATTN_TCGEN05_CS):
    import ctypes
    lib = _native.load()
    B, H, L, D = q.shape
    out = torch.full((B, L, H * D), float("nan"), dtype=q.dtype, device=q.device)
    dt = _native.DTYPE_CODES
    _native.check(lib.heatkv_segmented_attention_mapped(
        _native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
        _native.ptr(ct), _native.ptr(ck), _native.ptr(cv), _native.ptr(out), dt[q.dtype],
        dt[ck.dtype], dt[cv.dtype], B, H, L, pk.shape[1], D, st.shape[1], ctypes.c_float(scale),
        kernel, _native.ptr(order), splits, unsplit, _native.ptr(item_map), item_map.numel(), grid,
        _native.ptr(workspace), 0 if workspace is None else workspace.numel(),
        _native.stream_handle(q.device)), "heatkv_segmented_attention_mapped")
    return out


@pytest.mark.parametrize("splits,unsplit_frac", [(1, 1.0), (2, 0.5), (3, 0.0)])
@pytest.mark.parametrize("B,H,L,cap,S", [(2, 16, 1600, 5000, 12), (2, 4, 576, 3000, 10),
                                         (1, 3, 129, 1500, 6)])
def test_item_map_is_a_schedule_only(splits, unsplit_frac, B, H, L, cap, S, cuda_device):
    """heatkv_segmented_attention_mapped: any assignment of the column-split kernel's items to its
    CTAs (a random one, with empty slots, on a grid of 37 CTAs) gives the same bits as the
    launch without a map; the counters are reset."""
    rng = np.random.default_rng(L + splits)
    gen = torch.Generator().manual_seed(L + 7 * splits)
    d = cuda_device
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = (x.to(d) for x in _random_layout(rng, H, S, cap))
    order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
    blocks = B * H * ((L + 127) // 128)
    unsplit = int(blocks * unsplit_frac)
    n_items = unsplit + (blocks - unsplit) * splits
    lib = _native.load()
    ws = torch.zeros(max(int(lib.heatkv_attention_workspace_bytes(B, H, L, splits)), 256),
                     dtype=torch.uint8, device=d)
    scale = 1.0 / math.sqrt(128)
    grid = 37
    per_cta = [[] for _ in range(grid)]
    for item in rng.permutation(n_items):
        per_cta[int(rng.integers(grid))].append(int(item))
    rounds = max(len(x) for x in per_cta)
    imap = np.full(rounds * grid, -1, dtype=np.int32)
    for c, items in enumerate(per_cta):
        for k, item in enumerate(items):
            imap[c + k * grid] = item
    imap = torch.from_numpy(imap).to(d)
    import ctypes
    plain = torch.full((B, L, H * 128), float("nan"), dtype=q.dtype, device=d)
    dt = _native.DTYPE_CODES
    _native.check(lib.heatkv_segmented_attention_sched(
        _native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
        _native.ptr(ct), _native.ptr(ck), _native.ptr(cv), _native.ptr(plain), dt[q.dtype],
        dt[ck.dtype], dt[cv.dtype], B, H, L, cap, 128, S, ctypes.c_float(scale),
        _native.ATTN_TCGEN05_CS, _native.ptr(order), splits, unsplit, _native.ptr(ws), ws.numel(),
        _native.stream_handle(d)), "heatkv_segmented_attention_sched")
    mapped = _attention_mapped(q, pk, pv, st, en, ct, ck, cv, scale, order=order, splits=splits,
                               unsplit=unsplit, item_map=imap, grid=grid, workspace=ws)
    torch.cuda.synchronize()
    assert not torch.isnan(mapped.float()).any()
    assert torch.equal(mapped, plain)
    ref = _torch_reference(q, pk, pv, st.cpu(), en.cpu(), ct.cpu(), ck, cv, scale)
    _check_lowp(mapped.float().cpu().numpy(), ref.cpu().numpy())
    assert int(ws[: 4 * blocks].count_nonzero()) == 0, "split counters not reset"
    assert _native.device_status(d) == 0


def test_planned_item_map_matches_the_reference(cuda_device):
    """The hot path's planner (greedy item map, tail splits of the longest blocks) on a layout
    with uneven heads."""
    from heatkv_b200.hotpath import plan_column_split
    rng = np.random.default_rng(5)
    gen = torch.Generator().manual_seed(5)
    d = cuda_device
    B, H, L, cap, S = 2, 16, 576, 6000, 12
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, cap)
    lengths = [[int(en[h, i]) - int(st[h, i]) for i in range(int(ct[h]))] for h in range(H)]
    for splits in (None, 2):
        order, ns, unsplit, imap, grid = plan_column_split(lengths, L, B, splits=splits)
        lib = _native.load()
        ws = torch.zeros(max(int(lib.heatkv_attention_workspace_bytes(B, H, L, ns)), 256),
                         dtype=torch.uint8, device=d)
        out = _attention_mapped(q, pk, pv, st.to(d), en.to(d), ct.to(d), ck, cv,
                                1.0 / math.sqrt(128), order=torch.from_numpy(order).to(d),
                                splits=ns, unsplit=unsplit,
                                item_map=torch.from_numpy(imap).to(d), grid=grid, workspace=ws)
        ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, 1.0 / math.sqrt(128))
        _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(d) == 0


def test_item_map_entry_outside_the_launch_is_skipped_and_flagged(cuda_device):
    """An entry past the item space is skipped (HEATKV_DEVICE_BAD_ITEM_MAP = 0x10); the items
    the map does hold are computed."""
    rng = np.random.default_rng(8)
    gen = torch.Generator().manual_seed(8)
    d = cuda_device
    B, H, L, cap, S = 1, 2, 256, 1000, 4
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = (x.to(d) for x in _random_layout(rng, H, S, cap))
    order = torch.arange(H, dtype=torch.int32, device=d)
    imap = torch.tensor([0, 1, 2, 3, 1000, -1], dtype=torch.int32, device=d)  # 4 items, grid 2
    out = _attention_mapped(q, pk, pv, st, en, ct, ck, cv, 1.0 / math.sqrt(128), order=order,
                            splits=1, unsplit=4, item_map=imap, grid=2, workspace=None)
    assert _native.device_status(d) == 0x10
    ref = _torch_reference(q, pk, pv, st.cpu(), en.cpu(), ct.cpu(), ck, cv, 1.0 / math.sqrt(128))
    _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())


@pytest.mark.parametrize("sel", ["cs", "exact", "cs64"])
def test_current_in_segments_flag(sel, cuda_device):
    """HEATKV_ATTN_CURRENT_IN_SEGMENTS: with every head's current keys copied into the slab right
    after its last segment (extending it), the flagged call reads no separate current tiles and
    matches the reference; a head without segments still attends the current K/V."""
    import ctypes
    rng = np.random.default_rng(21)
    gen = torch.Generator().manual_seed(21)
    d = cuda_device
    B, H, L, S = 2, 6, 96, 5
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    cap = 6000
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = _random_layout(rng, H, S, 4000)
    ct[H - 1] = 0  # no segment: the current K/V come from cur_k / cur_v
    ref = _torch_reference(q, pk, pv, st, en, ct, ck, cv, 1.0 / math.sqrt(128))
    # extended layout: each head with segments gets its current keys as a last segment of its own
    st2, en2, ct2 = (x.numpy().copy() for x in (st, en, ct))
    st2 = np.concatenate([st2, np.zeros((H, 1), np.int32)], axis=1)
    en2 = np.concatenate([en2, np.zeros((H, 1), np.int32)], axis=1)
    pk2, pv2 = pk.clone(), pv.clone()
    base = 4000
    for h in range(H):
        if ct2[h] == 0:
            continue
        # append the current keys right after the head's last non-empty segment, copied there
        i = int(ct2[h])
        st2[h, i], en2[h, i] = base, base + L
        pk2[:, base:base + L] = ck[:, h]
        pv2[:, base:base + L] = cv[:, h]
        ct2[h] = i + 1
        base += L
    st2, en2, ct2 = (torch.from_numpy(np.ascontiguousarray(x, dtype=np.int32)).to(d)
                     for x in (st2, en2, ct2))
    kern = {"cs": _native.ATTN_TCGEN05_CS, "exact": _native.ATTN_EXACT,
            "cs64": _native.ATTN_TCGEN05_CS64}[sel]
    out = torch.empty(B, L, H * 128, dtype=q.dtype, device=d)
    dt = _native.DTYPE_CODES
    order = torch.arange(H, dtype=torch.int32, device=d)
    _native.check(_native.load().heatkv_segmented_attention_sched(
        _native.ptr(q), _native.ptr(pk2), _native.ptr(pv2), _native.ptr(st2), _native.ptr(en2),
        _native.ptr(ct2), _native.ptr(ck), _native.ptr(cv), _native.ptr(out), dt[q.dtype],
        dt[ck.dtype], dt[cv.dtype], B, H, L, cap, 128, st2.shape[1],
        ctypes.c_float(1.0 / math.sqrt(128)), kern | _native.ATTN_CURRENT_IN_SEGMENTS,
        _native.ptr(order), 1, 0, None, 0, _native.stream_handle(d)),
        "heatkv_segmented_attention_sched")
    torch.cuda.synchronize()
    _check_lowp(out.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(d) == 0


def test_cs64_item_map_and_kernel_choice(cuda_device):
    """The 64-key kernel (two CTAs per SM) runs when named (heatkv_attention_kernel_for), a random
    item map over its 128-row items on 296 CTAs gives the same bits as its launch without one,
    and both match the reference."""
    import ctypes
    lib = _native.load()
    dt = _native.DTYPE_CODES
    B, H, L, cap, S = 2, 16, 576, 4000, 12
    assert lib.heatkv_attention_kernel_for(dt[torch.bfloat16], dt[torch.bfloat16],
                                           dt[torch.bfloat16], B, H, L,
                                           _native.ATTN_TCGEN05_CS64, 1, 0, 0) == \
        _native.RUN_TCGEN05_CS64
    rng = np.random.default_rng(31)
    gen = torch.Generator().manual_seed(31)
    d = cuda_device
    q, ck, cv = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st, en, ct = (x.to(d) for x in _random_layout(rng, H, S, cap))
    order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
    n_items = B * H * ((L + 127) // 128)
    grid = 296
    per_cta = [[] for _ in range(grid)]
    for item in rng.permutation(n_items):
        per_cta[int(rng.integers(grid))].append(int(item))
    rounds = max(len(x) for x in per_cta)
    imap = np.full(rounds * grid, -1, dtype=np.int32)
    for c, items in enumerate(per_cta):
        for k, item in enumerate(items):
            imap[c + k * grid] = item
    imap = torch.from_numpy(imap).to(d)
    scale = 1.0 / math.sqrt(128)
    plain = torch.full((B, L, H * 128), float("nan"), dtype=q.dtype, device=d)
    _native.check(lib.heatkv_segmented_attention_sched(
        _native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
        _native.ptr(ct), _native.ptr(ck), _native.ptr(cv), _native.ptr(plain), dt[q.dtype],
        dt[ck.dtype], dt[cv.dtype], B, H, L, cap, 128, S, ctypes.c_float(scale),
        _native.ATTN_TCGEN05_CS64, _native.ptr(order), 1, 0, None, 0,
        _native.stream_handle(d)), "heatkv_segmented_attention_sched")
    mapped = _attention_mapped(q, pk, pv, st, en, ct, ck, cv, scale, order=order, splits=1,
                               unsplit=0, item_map=imap, grid=grid, workspace=None,
                               kernel=_native.ATTN_TCGEN05_CS64)
    torch.cuda.synchronize()
    assert torch.equal(mapped, plain)
    ref = _torch_reference(q, pk, pv, st.cpu(), en.cpu(), ct.cpu(), ck, cv, scale)
    _check_lowp(mapped.float().cpu().numpy(), ref.cpu().numpy())
    assert _native.device_status(d) == 0
