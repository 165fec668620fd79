"""ctypes binding of the C ABI declared in ``include/paged_serve.h``.

This is the whole Python↔native boundary: every call passes raw device
pointers, sizes and the current CUDA stream handle. Loading fails loudly —
there is no CPU or PyTorch fallback for any operation in this package.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_int64, c_void_p
from pathlib import Path

from paged_serve_b200.build import LIB_PATH

PS_OK = 0
PS_ERR_INVALID = 1
PS_ERR_UNSUPPORTED = 2
PS_ERR_CUDA = 3

PS_DTYPE_F16 = 1
PS_DTYPE_BF16 = 2

PS_DEVERR_BLOCK_ID = 1
PS_DEVERR_SLOT = 2
PS_DEVERR_POSITION = 4
PS_DEVERR_TIMEOUT = 8
PS_DEVERR_LENGTH = 16
PS_DEVERR_BLOCK_PAIRS = 32

PS_STREAM_BULK = 0
PS_STREAM_LOADS = 1

ABI_VERSION = 1

_p = c_void_p
_i = c_int
_l = c_int64

# name -> (restype, argtypes); mirrors include/paged_serve.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ps_abi_version": (c_int, []),
    "ps_last_error_string": (ctypes.c_char_p, []),
    "ps_cache_append": (c_int, [_p, _p, _p, _p, _p, _l, _l, _l, _i, _i, _i, _l, _i, _p, _p]),
    "ps_cache_append_rope": (
        c_int,
        [_p, _p, _p, _p, _p, _p, _l, _l, _l, _i, _i, _i, _l, _p, _l, _i, _i, _p, _p],
    ),
    "ps_copy_blocks": (c_int, [_p, _p, _p, _l, _i, _l, _l, _l, _p, _p]),
    "ps_build_slot_mapping": (c_int, [_p, _p, _p, _l, _p, _p, _i, _i, _i, _i, _l, _p, _p]),
    "ps_swap_blocks": (c_int, [_p, _p, _l, _l, _p, _p, _l, _l, _p, _l, _i, _l, _i, _p, _p]),
    "ps_paged_decode_workspace_bytes": (c_int64, [_i, _i, _i, _i, _i, _i]),
    "ps_paged_decode": (
        c_int,
        [_p, _l, _p, _l, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _i, _i, c_float, _i, _p, _l, _i,
         _p, _p],
    ),
    "ps_paged_decode_order": (c_int, [_p, _i, _p, _p]),
    "ps_selftest_wait_timeout": (c_int, [_p, _p]),
    "ps_paged_decode_ordered": (
        c_int,
        [_p, _l, _p, _l, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _i, _i, c_float, _i, _p, _l, _i,
         _p, _p, _p],
    ),
    "ps_paged_decode_append": (
        c_int,
        [_p, _l, _p, _l, _p, _l, _p, _l, _p, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _i, _i,
         c_float, _i, _p, _l, _i, _p, _p, _p],
    ),
    "ps_paged_decode_plan": (c_int, [_p, _i, _p, _i, _i, _i, _i, _i, _p, _l, _p]),
    "ps_paged_decode_append_planned": (
        c_int,
        [_p, _l, _p, _l, _p, _l, _p, _l, _p, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _i, _i,
         c_float, _i, _p, _l, _i, _p, _p, _p],
    ),
    "ps_paged_decode_listed": (
        c_int,
        [_p, _l, _p, _l, _p, _p, _l, _p, _l, _p, _i, _p, _i, _i, _i, _i, _i, _i, c_float, _i, _p,
         _l, _i, _p, _p],
    ),
    "ps_paged_decode_noalloc": (
        c_int,
        [_p, _l, _p, _l, _p, _p, _l, _p, _l, _p, _i, _i, _i, _i, _i, _i, c_float, _i, _i, _p,
         _p],
    ),
    "ps_stream_read": (c_int, [_p, _l, _p, _i, _p, _p]),
    "ps_paged_prefill": (
        c_int,
        [_p, _l, _p, _l, _l, _p, _p, _l, _p, _l, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, c_float,
         _i, _p, _p],
    ),
    "ps_paged_prefill_split": (
        c_int,
        [_p, _l, _p, _l, _l, _p, _p, _l, _p, _l, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, c_float,
         _i, _p, _l, _i, _p, _p],
    ),
    "ps_paged_prefill_workspace_bytes": (c_int64, [_i, _i, _i, _i, _i, _i, _i, _i]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A C-ABI call returned PS_ERR_CUDA."""


def library_path() -> Path:
    override = os.environ.get("PAGED_SERVE_B200_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared library once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise ImportError(
                f"paged_serve_b200 native library not found at {path}; build it with "
                "`python -m paged_serve_b200.build` (nvcc, sm_100a)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        got = lib.ps_abi_version()
        if got != ABI_VERSION:
            raise ImportError(f"{path} has ABI version {got}, expected {ABI_VERSION}")
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Map a C-ABI status to the reference's exception types."""
    if status == PS_OK:
        return
    msg = load().ps_last_error_string().decode(errors="replace")
    if status in (PS_ERR_INVALID, PS_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise NativeError(f"{what}: {msg}")
