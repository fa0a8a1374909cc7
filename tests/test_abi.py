"""The C-ABI library loads, exports every symbol include/heatkv.h declares, and rejects bad
arguments with the documented status codes before touching the GPU (no device needed)."""

import ctypes
import os
import re

import pytest

from heatkv_b200 import _native
from heatkv_b200.build import build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _native.load()


def declared_symbols():
    text = open(os.path.join(REPO, "include", "heatkv.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(heatkv_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    assert "heatkv_pack_kv" in syms and "heatkv_segmented_attention" in syms
    assert set(syms) == set(_native.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = os.popen(f"nm -D {_native.library_path()}").read()
    exported = set(re.findall(r" T (heatkv_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_library_targets_sm100a(lib):
    out = os.popen(f"cuobjdump --list-elf {_native.library_path()} 2>/dev/null").read()
    if not out:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out


def test_version_and_error_string(lib):
    assert b"sm_100a" in lib.heatkv_version()
    assert lib.heatkv_last_error_string() is not None


def _attn(lib, **over):
    args = dict(q=1, sk=None, sv=None, st=1, en=1, ct=1, ck=1, cv=1, out=1, qd=2, kd=2, vd=2,
                b=2, h=4, lq=8, cap=0, d=128, s=1, scale=0.1, exp2=0, kern=0)
    args.update(over)
    p = lambda x: None if x is None else ctypes.c_void_p(x)  # noqa: E731
    return lib.heatkv_segmented_attention(
        p(args["q"]), p(args["sk"]), p(args["sv"]), p(args["st"]), p(args["en"]), p(args["ct"]),
        p(args["ck"]), p(args["cv"]), p(args["out"]), args["qd"], args["kd"], args["vd"],
        args["b"], args["h"], args["lq"], args["cap"], args["d"], args["s"],
        args["scale"], args["exp2"], args["kern"], None)


def test_attention_argument_errors(lib):
    assert _attn(lib, d=64) == _native.HEATKV_ERR_UNSUPPORTED
    assert b"head_dim=128" in lib.heatkv_last_error_string()
    assert _attn(lib, lq=0) == _native.HEATKV_ERR_UNSUPPORTED
    assert b"current_len > 0" in lib.heatkv_last_error_string()
    assert _attn(lib, qd=7) == _native.HEATKV_ERR_UNSUPPORTED
    assert _attn(lib, q=None) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert _attn(lib, cap=10) == _native.HEATKV_ERR_INVALID_ARGUMENT  # null slab, capacity > 0
    assert _attn(lib, s=300) == _native.HEATKV_ERR_UNSUPPORTED
    assert _attn(lib, kern=9) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert _attn(lib, kern=2, qd=0) == _native.HEATKV_ERR_UNSUPPORTED  # tcgen05 needs 16-bit
    assert _attn(lib, b=0) == _native.HEATKV_OK  # nothing to do


def test_pack_argument_errors(lib):
    p = ctypes.c_void_p
    call = lambda **o: lib.heatkv_pack_kv(  # noqa: E731
        p(1), p(1), p(1), p(1), o.get("kd", 2), o.get("vd", 2), o.get("b", 2), 100, 100,
        o.get("d", 128), p(1), p(1), p(1), o.get("n", 3), o.get("ml", 5), None)
    assert call(kd=5) == _native.HEATKV_ERR_UNSUPPORTED
    assert call(b=-1) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert call(n=0) == _native.HEATKV_OK
    assert call(ml=0) == _native.HEATKV_OK
    assert call(n=70000) == _native.HEATKV_ERR_UNSUPPORTED


def test_scatter_argument_errors(lib):
    """Both scatter entry points check their destinations, full-output sizes and (mapped) item
    map before any device work."""
    p = ctypes.c_void_p

    def scatter(mapped=False, **o):
        args = (p(16), p(16), p(16), p(16), p(16), p(16), p(16), p(16),
                None if o.get("no_ptrs") else p(16), o.get("n_out", 2), p(16), p(16),
                o.get("out_batch", 4), o.get("out_heads", 16), 2, 2, 2, 2, 8, 64, 100, 128, 4,
                ctypes.c_float(0.088), None)
        if mapped:
            return lib.heatkv_segmented_attention_scatter_mapped(
                *args, None if o.get("no_map") else p(16), o.get("map_len", 296),
                o.get("grid", 148), None)
        return lib.heatkv_segmented_attention_scatter(*args, None)

    for mapped in (False, True):
        name = b"heatkv_segmented_attention_scatter" + (b"_mapped" if mapped else b"")
        assert scatter(mapped, n_out=0) == _native.HEATKV_ERR_INVALID_ARGUMENT
        assert name + b": 1..64 destinations" in lib.heatkv_last_error_string()
        assert scatter(mapped, n_out=65) == _native.HEATKV_ERR_INVALID_ARGUMENT
        assert scatter(mapped, no_ptrs=True) == _native.HEATKV_ERR_INVALID_ARGUMENT
        assert scatter(mapped, out_batch=1) == _native.HEATKV_ERR_INVALID_ARGUMENT
        assert b"smaller than this shard" in lib.heatkv_last_error_string()
        assert scatter(mapped, out_heads=4) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert scatter(True, no_map=True) == _native.HEATKV_ERR_INVALID_ARGUMENT
    assert b"item_map of rounds x map_grid" in lib.heatkv_last_error_string()
    assert scatter(True, map_len=300) == _native.HEATKV_ERR_INVALID_ARGUMENT   # not rounds x grid
    assert scatter(True, grid=0) == _native.HEATKV_ERR_INVALID_ARGUMENT
