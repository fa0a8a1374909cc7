"""Which attention kernel a call runs (heatkv_attention_kernel_for, no GPU needed): dtype routing
as the reference's dot modes imply it, the kernel selectors, and the 64-key kernel as the default
for 16-bit calls, with or without key-range splits."""

import pytest

from heatkv_b200 import _native

F32, F16, BF16 = 0, 1, 2
AUTO, EXACT, TC, CS, CS64 = (_native.ATTN_AUTO, _native.ATTN_EXACT, _native.ATTN_TCGEN05,
                             _native.ATTN_TCGEN05_CS, _native.ATTN_TCGEN05_CS64)


def run(dt=(BF16, BF16, BF16), batch=2, heads=16, q_len=4096, kernel=AUTO, splits=1, ws=0,
        unsplit=0):
    return _native.load().heatkv_attention_kernel_for(*dt, batch, heads, q_len, kernel, splits, ws,
                                                      unsplit)


def test_sixteen_bit_calls_take_the_64_key_kernel():
    for batch in (2, 8, 16):
        for lq in (1, 4, 16, 36, 64, 144, 256, 400, 576, 1024, 1600, 2304, 4096):
            assert run(batch=batch, q_len=lq) == _native.RUN_TCGEN05_CS64, (batch, lq)
    assert run(kernel=TC) == _native.RUN_TCGEN05_CS64
    # splits without a workspace cannot run split: the 64-key kernel runs them whole
    assert run(splits=2, ws=0) == _native.RUN_TCGEN05_CS64


def test_split_calls_take_the_64_key_kernel():
    """The 64-key kernel takes key-range splits too (unsplit_blocks counts its 128-row blocks),
    so splits, the workspace and unsplit_blocks leave 16-bit calls on it at every size.
    (Scattering calls run it unsplit; the GPU scatter tests cover those.)"""
    for splits, unsplit in ((2, 0), (4, 100), (3, 2 * 16 * 32)):
        assert run(splits=splits, ws=1, unsplit=unsplit) == _native.RUN_TCGEN05_CS64
        assert run(batch=16, splits=splits, ws=1, unsplit=unsplit) == _native.RUN_TCGEN05_CS64
    assert run(batch=8, heads=28, q_len=2304, splits=2, ws=1) == _native.RUN_TCGEN05_CS64
    # a named variant keeps its own kernel with splits
    assert run(kernel=CS, splits=2, ws=1) == _native.RUN_TCGEN05_CS


def test_named_variants_and_the_flags():
    assert run(batch=16, kernel=CS) == _native.RUN_TCGEN05_CS
    assert run(kernel=CS64) == _native.RUN_TCGEN05_CS64
    assert run(kernel=CS64, splits=2, ws=1) == _native.RUN_TCGEN05_CS64
    assert run(kernel=AUTO | _native.ATTN_STATIC_META) == _native.RUN_TCGEN05_CS64
    assert run(kernel=AUTO | _native.ATTN_CURRENT_IN_SEGMENTS) == _native.RUN_TCGEN05_CS64
    assert run(kernel=EXACT) == _native.RUN_EXACT


def test_dtype_routing():
    # fp32 q/k with 16-bit v (the real model under autocast): tf32 scores on tensor cores
    assert run(dt=(F32, F32, BF16)) == _native.RUN_TCGEN05_TF32
    assert run(dt=(F32, F32, F16), kernel=TC) == _native.RUN_TCGEN05_TF32
    assert run(dt=(F32, F32, BF16), kernel=EXACT) == _native.RUN_EXACT
    # every other mix, and all-fp32, on the exact kernel
    assert run(dt=(F32, F32, F32)) == _native.RUN_EXACT
    assert run(dt=(F16, BF16, BF16)) == _native.RUN_EXACT
    assert run(dt=(F16, F16, F16)) == _native.RUN_TCGEN05_CS64


@pytest.mark.parametrize("dt,kernel", [((F32, F32, F32), TC), ((F16, BF16, BF16), TC),
                                       ((F32, F32, BF16), CS64)])
def test_tensor_core_selectors_reject_other_dtypes(dt, kernel):
    assert run(dt=dt, kernel=kernel) == _native.HEATKV_ERR_UNSUPPORTED


def test_invalid_arguments():
    assert run(kernel=7) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert run(kernel=6) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert run(kernel=3) == _native.HEATKV_ERR_INVALID_ARGUMENT  # the retired two-tile selector
    assert run(q_len=0) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert run(dt=(5, BF16, BF16)) == _native.HEATKV_ERR_UNSUPPORTED
