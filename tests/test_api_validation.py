"""The drop-in wrappers validate like the reference (same order, exception types and messages),
without needing a GPU: every check below fires before the CUDA requirement."""

import pytest
import torch

from heatkv_b200.real_pruning_fused_attention import (
    fused_real_pruning_flat_segmented_attention as attn,
    pack_flat_segments_kv as pack,
)


def _inputs(B=2, H=3, L=5, D=128, cap=16, S=2):
    q = torch.randn(B, H, L, D)
    return dict(q=q, persisted_k=torch.randn(B, cap, D), persisted_v=torch.randn(B, cap, D),
                segment_starts=torch.zeros(H, S, dtype=torch.int32),
                segment_ends=torch.zeros(H, S, dtype=torch.int32),
                segment_counts=torch.zeros(H, dtype=torch.int32),
                current_k=torch.randn(B, H, L, D), current_v=torch.randn(B, H, L, D),
                softmax_scale=0.1)


@pytest.mark.parametrize("mutate,exc,msg", [
    (lambda a: a.update(q=a["q"][0]), ValueError, r"must have shape \[B, H, L, D\]"),
    (lambda a: a.update(current_k=a["current_k"][:, :, :2]), ValueError, "identical"),
    (lambda a: a.update(persisted_k=a["persisted_k"][0]), ValueError, r"shape \[B, S, D\]"),
    (lambda a: a.update(persisted_v=a["persisted_v"][:, :3]), ValueError, "identical shapes"),
    (lambda a: a.update(persisted_k=a["persisted_k"][:1], persisted_v=a["persisted_v"][:1]),
     ValueError, "batch dimension"),
    (lambda a: a.update(persisted_k=a["persisted_k"].half()), ValueError, "persisted_k dtype"),
    (lambda a: a.update(persisted_v=a["persisted_v"].half()), ValueError, "persisted_v dtype"),
    (lambda a: a.update(segment_ends=a["segment_ends"][:, :1]), ValueError, "identical shapes"),
    (lambda a: a.update(segment_starts=a["segment_starts"][:2], segment_ends=a["segment_ends"][:2]),
     ValueError, r"shape \[H, S\]"),
    (lambda a: a.update(segment_counts=a["segment_counts"][:1]), ValueError, r"shape \[H\]"),
    (lambda a: a.update(softmax_mode="exp3"), ValueError, "unsupported softmax_mode"),
    (lambda a: None, RuntimeError, "requires CUDA tensors"),
    (lambda a: a.update(allow_cpu_fallback=True), RuntimeError, "no CPU fallback"),
])
def test_attention_validation(mutate, exc, msg):
    a = _inputs()
    mutate(a)
    with pytest.raises(exc, match=msg):
        attn(**a)


def test_attention_none_slab_is_accepted_until_device_check():
    a = _inputs()
    a.update(persisted_k=None, persisted_v=None)
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        attn(**a)


def test_bad_dot_mode_env(monkeypatch):
    from heatkv_b200 import real_pruning_fused_attention as m
    monkeypatch.setenv("REAL_PRUNING_FUSED_QK_DOT_MODE", "int8")
    with pytest.raises(ValueError, match="QK_DOT_MODE"):
        m._kernel_selector()
    monkeypatch.setenv("REAL_PRUNING_FUSED_QK_DOT_MODE", "fp32")
    assert m._kernel_selector() == m._native.ATTN_EXACT
    # tf32 scores are what the tensor-core kernels compute on fp32 q/k (and exact on 16-bit ones)
    monkeypatch.setenv("REAL_PRUNING_FUSED_QK_DOT_MODE", "tf32")
    assert m._kernel_selector() == m._native.ATTN_AUTO
    monkeypatch.setenv("REAL_PRUNING_FUSED_VALUE_DOT_MODE", "fp32")
    assert m._kernel_selector() == m._native.ATTN_EXACT
    monkeypatch.setenv("HEATKV_ATTENTION_KERNEL", "tcgen05")
    assert m._kernel_selector() == m._native.ATTN_TCGEN05
    monkeypatch.setenv("HEATKV_ATTENTION_KERNEL", "tcgen05_pair")   # retired
    with pytest.raises(ValueError, match="HEATKV_ATTENTION_KERNEL"):
        m._kernel_selector()
    monkeypatch.setenv("HEATKV_ATTENTION_KERNEL", "tcgen05_cs")
    assert m._kernel_selector() == m._native.ATTN_TCGEN05_CS
    monkeypatch.setenv("HEATKV_ATTENTION_KERNEL", "fast")
    with pytest.raises(ValueError, match="HEATKV_ATTENTION_KERNEL"):
        m._kernel_selector()


def _pack_inputs():
    return dict(dst_k=torch.zeros(2, 10, 128), dst_v=torch.zeros(2, 10, 128),
                src_k=torch.randn(2, 6, 128), src_v=torch.randn(2, 6, 128),
                dst_starts=torch.tensor([0]), src_starts=torch.tensor([1]),
                lengths=torch.tensor([3]))


@pytest.mark.parametrize("mutate,exc,msg", [
    (lambda a: a.update(dst_k=a["dst_k"][0]), ValueError, r"dst_k shaped \[B, S, D\]"),
    (lambda a: a.update(dst_v=a["dst_v"][:, :5]), ValueError, "destination shapes"),
    (lambda a: a.update(src_v=a["src_v"][:, :5]), ValueError, "source shapes"),
    (lambda a: a.update(src_k=a["src_k"][:1], src_v=a["src_v"][:1]), ValueError, "batch and head_dim"),
    (lambda a: None, RuntimeError, "requires CUDA tensors"),
])
def test_pack_validation(mutate, exc, msg):
    a = _pack_inputs()
    mutate(a)
    with pytest.raises(exc, match=msg):
        pack(**a)
