"""ctypes binding of ``libnie_b200.so`` (the C ABI declared in ``include/nie_b200.h``).

The library is loaded once per process.  There is no fallback: if the
shared object is missing the import fails with instructions to build it.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnie_b200.so"

NIE_DTYPE_F32 = 0
NIE_DTYPE_BF16 = 1
NIE_DTYPE_F16 = 2

NIE_OK = 0
NIE_ERR_INVALID = 1
NIE_ERR_UNSUPPORTED = 2
NIE_ERR_CUDA = 3

NIE_DEV_ERR_BLOCK_RANGE = 1
NIE_DEV_ERR_SLOT_RANGE = 2
NIE_DEV_ERR_TIMEOUT = 4
NIE_DEV_ERR_CAPACITY = 8
NIE_DEV_ERR_INDEX_RANGE = 16

# name -> (restype, argtypes); mirrors include/nie_b200.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "nie_version": (c_int, []),
    "nie_last_error": (ctypes.c_char_p, []),
    "nie_device_sm_count": (c_int, [c_int]),
    "nie_pack_ragged": (
        c_int,
        [c_void_p, c_int32, c_int64, c_void_p, c_int64, c_int32, c_int64]
        + [c_void_p] * 10
        + [c_void_p],
    ),
    "nie_write_kv": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int64, c_int64]
        + [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "nie_gather_kv": (
        c_int,
        [c_void_p, c_void_p, c_int32, c_int32, c_int64, c_int64, c_int32, c_int32, c_int32]
        + [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "nie_copy_blocks": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]
        + [c_int64, c_int32, c_int32, c_int64, c_int32, c_int32, c_int32, c_void_p, c_void_p],
    ),
    "nie_enable_peer_access": (c_int, [c_int, c_int]),
    "nie_ipc_export": (c_int, [c_void_p, c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "nie_ipc_import": (c_int, [c_void_p, ctypes.c_uint64, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p)]),
    "nie_ipc_close": (c_int, [c_void_p]),
    "nie_paged_decode_workspace_size": (c_size_t, [c_int, c_int32, c_int32, c_int32]),
    "nie_paged_decode": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int64]
        + [c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p]
        + [c_void_p, c_void_p, c_int32, c_float, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "nie_paged_decode_overlapped": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int64]
        + [c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p]
        + [c_void_p, c_void_p, c_int32, c_float, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "nie_paged_decode_noalloc_capacity": (c_size_t, []),
    "nie_paged_decode_noalloc": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int64]
        + [c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p]
        + [c_void_p, c_void_p, c_int32, c_float, c_void_p, c_void_p],
    ),
    "nie_add_rmsnorm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_float, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "nie_rope_write_kv": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64]
        + [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int64, c_int64]
        + [c_int32, c_void_p, c_void_p, c_void_p],
    ),
    "nie_silu_mul": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "nie_embed_rows": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "nie_argmax_workspace_size": (c_size_t, []),
    "nie_argmax_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_size_t, c_void_p]),
    "nie_linear": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int32, c_void_p, c_void_p],
    ),
    "nie_linear_overlapped": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int32, c_void_p, c_void_p],
    ),
    "nie_linear_timeout_test": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int32, c_void_p, c_void_p]
        + [ctypes.c_uint32],
    ),
    "nie_varlen_workspace_size": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "nie_varlen_attention": (
        c_int,
        [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int32, c_int32, c_int64, c_int64]
        + [c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]
        + [c_void_p, c_int32, c_int32, c_int32, c_float, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
}


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "or `python -m nano_infer_engine_b200._build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


def check(status: int, what: str) -> None:
    if status != NIE_OK:
        message = lib.nie_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed (status {status}): {message}")
