"""ctypes binding of libaoh.so (the C ABI declared in include/aoh.h).

The library is built in-tree by ``python -m aoh_b200.build``.  Loading never
falls back to anything else: a missing or stale library is an ImportError at
first use, and every non-zero status becomes a Python exception carrying the
library's own message (the reference's error types: ValueError for bad
arguments, torch.OutOfMemoryError for an exhausted page pool, RuntimeError for
state and CUDA errors).
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaoh.so"
ABI_VERSION = 1

OK, INVALID, OUT_OF_PAGES, CUDA, UNSUPPORTED, STATE, DEVICE_CHECK = range(7)
F32, BF16 = 0, 1
PAST_LEN_DEVICE = -1


class KVConfig(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("batch", C.c_int32),
        ("num_q_heads", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("page_size", C.c_int32),
        ("dtype", C.c_int32),
        ("sink_size", C.c_int32),
        ("recent_size", C.c_int32),
        ("max_context", C.c_int32),
        ("num_pages", C.c_int32),
        ("labels", C.POINTER(C.c_uint8)),
        ("owned", C.POINTER(C.c_uint8)),
    ]


_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_SIGNATURES = {
    "aoh_abi_version": (C.c_int, []),
    "aoh_last_error": (C.c_char_p, []),
    "aoh_kv_create": (C.c_int, [C.POINTER(KVConfig), C.POINTER(_vp)]),
    "aoh_kv_destroy": (None, [_vp]),
    "aoh_kv_buffer_sizes": (C.c_int, [_vp, C.POINTER(_i64), C.POINTER(_i64)]),
    "aoh_kv_bind": (C.c_int, [_vp, _vp, _vp, _vp]),
    "aoh_kv_reserve": (C.c_int, [_vp, _i32, _i32]),
    "aoh_kv_release": (C.c_int, [_vp, _i32]),
    "aoh_kv_sync": (C.c_int, [_vp, _vp]),
    "aoh_kv_free_pages": (_i32, [_vp]),
    "aoh_kv_unit_pages": (C.c_int, [_vp, _i32, _i32, _i32, C.POINTER(_i32), _i32, C.POINTER(_i32)]),
    "aoh_kv_locate": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, C.POINTER(_i32), C.POINTER(_i32)]),
    "aoh_kv_device_status": (C.c_int, [_vp, C.POINTER(_i32), _vp]),
    "aoh_decode_workspace_bytes": (C.c_size_t, [_vp]),
    "aoh_kv_set_length": (C.c_int, [_vp, _i32, _vp]),
    "aoh_kv_advance": (C.c_int, [_vp, _i32, _vp]),
    "aoh_kv_set_decode_append": (C.c_int, [_vp, _i32]),
    "aoh_attn_decode": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, C.c_size_t, _vp]),
    "aoh_attn_decode_noalloc": (C.c_int, [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "aoh_attn_prefill": (C.c_int, [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "aoh_attn_prefill_flash": (C.c_int, [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "aoh_kv_append": (C.c_int, [_vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    "aoh_classify_workspace_bytes": (C.c_size_t, [_i32, _i32, _i32, _i32]),
    "aoh_classify_eff_ranks": (C.c_int, [_vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                                         C.c_size_t, _vp]),
    "aoh_partition": (C.c_int, [C.POINTER(C.c_uint8), _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                C.POINTER(_i32)]),
    "aoh_shared_alloc": (C.c_int, [C.c_size_t, C.POINTER(_vp), _vp]),
    "aoh_shared_free": (C.c_int, [_vp]),
    "aoh_shared_open": (C.c_int, [_vp, C.POINTER(_vp)]),
    "aoh_shared_close": (C.c_int, [_vp]),
    "aoh_kv_set_peers": (C.c_int, [_vp, _i32, _i32, C.POINTER(_vp), C.c_size_t, C.POINTER(_vp)]),
    "aoh_gather_wait": (C.c_int, [_vp, _i32, _i32, _vp]),
    "aoh_diag_exp2_poly": (C.c_int, [_vp, _vp, _i32, _vp]),
    "aoh_rope_qk": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, C.c_float, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                              _vp]),
}
IPC_HANDLE_BYTES = 64

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loads it on first use)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(f"{LIB_PATH} is missing: build it with `python -m aoh_b200.build`")
            h = C.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            if h.aoh_abi_version() != ABI_VERSION:
                raise ImportError(f"{LIB_PATH} has ABI {h.aoh_abi_version()}, expected {ABI_VERSION}")
            _lib = h
    return _lib


def exported_symbols():
    return list(_SIGNATURES)


def check(rc: int, what: str = "") -> None:
    """Raise the exception matching an aoh_status."""
    if rc == OK:
        return
    msg = lib().aoh_last_error().decode(errors="replace")
    if what:
        msg = f"{what}: {msg}"
    if rc == INVALID:
        raise ValueError(msg)
    if rc == OUT_OF_PAGES:
        import torch
        raise torch.OutOfMemoryError(msg)
    if rc == UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"[aoh status {rc}] {msg}")


def stream_handle(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
