"""The attention entry point that allocates nothing, against the workspace entry point (GPU).

``heatkv_segmented_attention_noalloc`` serves callers that cannot allocate device memory when
they call attention (a serving step running inside a memory pool that must not grow, or a host
without its own CUDA allocator): its split-KV scratch is a fixed 32 MiB array inside the library.
This file is named to be collected last, so a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from heatkv_b200 import _native

pytestmark = pytest.mark.gpu

ATOL, REL = 2e-2, 1e-2   # the bf16 tolerances of the other attention tests


def _inputs(B, H, L, cap, S, seed):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    d = torch.device("cuda", 0)
    q, k, v = (torch.randn(B, H, L, 128, generator=gen).bfloat16().to(d) for _ in range(3))
    pk, pv = (torch.randn(B, cap, 128, generator=gen).bfloat16().to(d) for _ in range(2))
    st = np.zeros((H, S), np.int32)
    en = np.zeros((H, S), np.int32)
    ct = np.zeros(H, np.int32)
    for h in range(H):
        ct[h] = rng.integers(1, S + 1)
        for i in range(ct[h]):
            n = int(rng.choice([1, 16, 64, 129, 400]))
            s0 = int(rng.integers(0, cap - n + 1))
            st[h, i], en[h, i] = s0, s0 + n
    meta = [torch.from_numpy(x).to(d) for x in (st, en, ct)]
    order = torch.from_numpy(rng.permutation(H).astype(np.int32)).to(d)
    return q, k, v, pk, pv, meta, order


def _call(lib, fn_name, q, k, v, pk, pv, meta, order, splits, extra):
    B, H, L, D = q.shape
    out = torch.full((B, L, H * D), float("nan"), dtype=q.dtype, device=q.device)
    st, en, ct = meta
    args = [_native.ptr(q), _native.ptr(pk), _native.ptr(pv), _native.ptr(st), _native.ptr(en),
            _native.ptr(ct), _native.ptr(k), _native.ptr(v), _native.ptr(out),
            _native.DTYPE_CODES[q.dtype], _native.DTYPE_CODES[k.dtype], _native.DTYPE_CODES[v.dtype],
            B, H, L, pk.shape[1], D, st.shape[1], ctypes.c_float(1 / math.sqrt(128)), 0,
            _native.ATTN_TCGEN05, _native.ptr(order), splits] + extra
    status = getattr(lib, fn_name)(*args, _native.stream_handle(q.device))
    return status, out


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _native.load()
    q, k, v, pk, pv, meta, order = _inputs(2, 16, 576, 4000, 10, seed=21)
    splits = 2
    nbytes = int(lib.heatkv_attention_workspace_bytes(2, 16, 576, splits))
    assert 0 < nbytes <= 32 << 20
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=q.device)
    status, ref = _call(lib, "heatkv_segmented_attention_ws", q, k, v, pk, pv, meta, order, splits,
                        [_native.ptr(ws), nbytes])
    _native.check(status, "workspace entry point")
    for _ in range(2):  # the second call finds the scratch left by the first
        status, out = _call(lib, "heatkv_segmented_attention_noalloc", q, k, v, pk, pv, meta,
                            order, splits, [])
        _native.check(status, "noalloc entry point")
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= ATOL and err / ref.float().abs().max().item() <= REL, err
    assert _native.device_status(q.device) == 0


def test_noalloc_rejects_scratch_beyond_its_fixed_size():
    lib = _native.load()
    q, k, v, pk, pv, meta, order = _inputs(2, 16, 4096, 2000, 4, seed=22)
    assert int(lib.heatkv_attention_workspace_bytes(2, 16, 4096, 4)) > 32 << 20
    status, out = _call(lib, "heatkv_segmented_attention_noalloc", q, k, v, pk, pv, meta, order,
                        4, [])
    assert status == _native.HEATKV_ERR_UNSUPPORTED
    assert b"scratch" in lib.heatkv_last_error_string()
    torch.cuda.synchronize()
    assert torch.isnan(out).all()  # nothing was launched
