"""ctypes binding of libheatkv.so (the C ABI declared in include/heatkv.h).

The library is loaded from the package directory (it is built in-tree by ``heatkv_b200.build``).
There is no fallback: when the library is missing or cannot be loaded every entry point raises
``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libheatkv.so")

HEATKV_OK = 0
HEATKV_ERR_INVALID_ARGUMENT = -1
HEATKV_ERR_UNSUPPORTED = -2
HEATKV_ERR_CUDA = -3

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

ATTN_AUTO, ATTN_EXACT, ATTN_TCGEN05, ATTN_TCGEN05_CS = 0, 1, 2, 4  # 3: retired
ATTN_TCGEN05_CS64 = 5
ATTN_STATIC_META = 0x100  # OR into a selector: metadata not written by preceding work
ATTN_CURRENT_IN_SEGMENTS = 0x200  # OR into a selector: current keys end every head's segments
RUN_EXACT, RUN_TCGEN05_CS, RUN_TCGEN05_TF32 = 1, 3, 4  # heatkv_attn_run (2: retired)
RUN_TCGEN05_CS64 = 5

DEVICE_PACK_OUT_OF_RANGE = 0x1
DEVICE_WAIT_TIMEOUT = 0x2
DEVICE_BAD_SEGMENT = 0x4
DEVICE_GATHER_OUT_OF_RANGE = 0x8

# every symbol include/heatkv.h declares, with its ctypes signature
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_i = ctypes.c_int
SIGNATURES = {
    "heatkv_last_error_string": (ctypes.c_char_p, []),
    "heatkv_version": (ctypes.c_char_p, []),
    "heatkv_pack_kv": (_i, [_p, _p, _p, _p, _i, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _i64,
                            _i64, _p]),
    "heatkv_pack_kv_batched": (_i, [_p, _i64, _p, _p, _p, _p, _i64, _i, _i, _i64, _i64, _i64, _i,
                                    _p]),
    "heatkv_segmented_attention": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i64, _i64,
                                        _i64, _i64, _i64, _i64, ctypes.c_float, _i, _i, _p]),
    "heatkv_segmented_attention_ws": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i64,
                                           _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i, _i,
                                           _p, _i, _p, ctypes.c_size_t, _p]),
    "heatkv_attention_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i]),
    "heatkv_segmented_attention_sched": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i,
                                              _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                              _i, _p, _i, _i64, _p, ctypes.c_size_t, _p]),
    "heatkv_segmented_attention_mapped": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i,
                                               _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                               _i, _p, _i, _i64, _p, _i64, _i, _p, ctypes.c_size_t,
                                               _p]),
    "heatkv_segmented_attention_scatter": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _p, _p,
                                                _i64, _i64, _i, _i, _i, _i64, _i64, _i64, _i64,
                                                _i64, _i64, ctypes.c_float, _p, _p]),
    "heatkv_segmented_attention_scatter_mapped": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _p,
                                                       _p, _i64, _i64, _i, _i, _i, _i64, _i64,
                                                       _i64, _i64, _i64, _i64, ctypes.c_float,
                                                       _p, _p, _i64, _i, _p]),
    "heatkv_peer_barrier": (_i, [_p, _p, _i, _i, _p]),
    "heatkv_peer_alloc": (_i, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _p]),
    "heatkv_peer_open": (_i, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "heatkv_peer_close": (_i, [_p]),
    "heatkv_peer_free": (_i, [_p]),
    "heatkv_enable_peer_access": (_i, [_i]),
    "heatkv_segmented_attention_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i,
                                                _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                                _i, _i, _p, _i, _p]),
    "heatkv_gather_head_shards": (_i, [_p, _p, _i, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _p, _p, _p]),
    "heatkv_attention_kernel_for": (_i, [_i, _i, _i, _i64, _i64, _i64, _i, _i, _i, _i64]),
    "heatkv_slot_schedule": (_i, [_p, _i, _i, _p, _p, _p, _p, _p, _p]),
    "heatkv_scas_mass": (_i, [_p, _p, _i, _i64, _i64, _i64, _i64, ctypes.c_float, _p, _i, _p,
                              _i64, _p]),
    "heatkv_qkv_prepare": (_i, [_p, _p, _p, _p, _i, _i, _i64, _i64, _i64, _i64, _p,
                                ctypes.c_float, _p, _p, _i64, _p]),
    "heatkv_qkv_prepare_append": (_i, [_p, _p, _p, _p, _i, _i, _i64, _i64, _i64, _i64, _p,
                                       ctypes.c_float, _p, _p, _i64, _p, _p, _i64, _p, _p]),
    "heatkv_qkv_project": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _i64, _i64, _i64, _i64, _p,
                                ctypes.c_float, _p, _p, _i64, _p, _p, _i64, _p, _p]),
    "heatkv_slot_tables": (_i, [_i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "heatkv_strict_budget": (_i, [_p, _i, _i, _i, _i, _p, _i, _i, _i, ctypes.c_double, _p, _p,
                                  _p, _i64, _p, _p]),
    "heatkv_device_status": (_i, [ctypes.POINTER(ctypes.c_uint32), _i, _p]),
}

_lock = threading.Lock()
_lib = None
_load_error = None


def library_path() -> str:
    return _LIB_PATH


def load():
    """Load (once) and return the ctypes library; RuntimeError if it is not available."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                _load_error = (f"libheatkv.so not found at {_LIB_PATH}; build it with "
                               "`python -m heatkv_b200.build`")
                raise RuntimeError(_load_error)
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Map a heatkv_status to the reference's exception types."""
    if status == HEATKV_OK:
        return
    msg = load().heatkv_last_error_string().decode(errors="replace") or what
    if status == HEATKV_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(msg)


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device):
    """The current CUDA stream of ``device`` as the ``cudaStream_t`` the C ABI takes (the raw
    handle is read without building a ``torch.cuda.Stream``: this runs on every launch)."""
    if not isinstance(device, torch.device):
        device = torch.device(device)
    if _RAW_STREAM is not None:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return _RAW_STREAM(index)
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t):
    """Device address of a tensor (or None) for a ``void*`` argument."""
    return None if t is None else t.data_ptr()


def device_status(device=None, clear: bool = True) -> int:
    """Sticky HEATKV_DEVICE_* flags of ``device`` (synchronises its current stream)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flags = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        check(load().heatkv_device_status(ctypes.byref(flags), int(clear), stream_handle(device)),
              "heatkv_device_status")
    return int(flags.value)
