"""The C-ABI library loads and exports every entry point of include/nie_b200.h (no GPU needed)."""

import ctypes
import re
from pathlib import Path

from nano_infer_engine_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "nie_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(nie_\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("nie_pack_ragged", "nie_write_kv", "nie_paged_decode", "nie_varlen_attention", "nie_copy_blocks"):
        assert required in names


def test_every_declared_symbol_is_exported_and_bound():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string():
    assert _native.lib.nie_version() >= 100
    assert isinstance(_native.lib.nie_last_error(), bytes)


def test_invalid_arguments_fail_before_any_launch():
    lib = _native.lib
    # null pointers are rejected on the host with NIE_ERR_INVALID
    rc = lib.nie_write_kv(None, None, 4, None, None, 1, 0, 1, 8, 16, 8, 64, None, None, None)
    assert rc == _native.NIE_ERR_INVALID
    assert b"null pointer" in lib.nie_last_error()
    rc = lib.nie_pack_ragged(None, 0, 1, None, 1, 16, 1, *([None] * 9), None, None)
    assert rc == _native.NIE_ERR_INVALID
    rc = lib.nie_copy_blocks(None, None, 1, None, None, None, 1, None, 1, 0, 1, 1, 16, 8, 64, None, None)
    assert rc == _native.NIE_ERR_INVALID
    rc = lib.nie_write_kv(1, 1, 4, 1, 1, 7, 0, 1, 8, 16, 8, 64, 1, None, None)
    assert rc == _native.NIE_ERR_INVALID and b"dtype" in lib.nie_last_error()


def test_new_entry_points_validate_before_any_launch():
    """nie_linear(_overlapped) and nie_paged_decode_overlapped reject bad arguments on the host."""
    lib = _native.lib
    for fn in (lib.nie_linear, lib.nie_linear_overlapped):
        assert fn(None, 64, None, 128, 64, 1, None, 128, _native.NIE_DTYPE_BF16, None, None) == _native.NIE_ERR_INVALID
        # shapes the weight-streaming kernel does not take come back as UNSUPPORTED, so
        # a caller can fall back to a library GEMM (no pointer is dereferenced)
        fake = 1 << 20
        assert fn(fake, 64, fake, 128, 64, 17, fake, 128, _native.NIE_DTYPE_BF16, None, None) == \
            _native.NIE_ERR_UNSUPPORTED  # 17 rows
        assert fn(fake, 64, fake, 128, 64, 4, fake, 128, _native.NIE_DTYPE_F32, None, None) == \
            _native.NIE_ERR_UNSUPPORTED  # fp32
        assert fn(fake, 64, fake, 100, 64, 4, fake, 100, _native.NIE_DTYPE_BF16, None, None) == \
            _native.NIE_ERR_UNSUPPORTED  # n not a multiple of 64
        assert fn(fake + 2, 64, fake, 128, 64, 4, fake, 128, _native.NIE_DTYPE_BF16, None, None) == \
            _native.NIE_ERR_UNSUPPORTED  # x not 16-byte aligned
        # an empty batch is done before any device call
        assert fn(fake, 64, fake, 128, 64, 0, fake, 128, _native.NIE_DTYPE_BF16, None, None) == _native.NIE_OK
    rc = lib.nie_paged_decode_overlapped(None, 0, None, 0, None, None, 1, 0, 1, 8, 16, 8, 64, 32, None, 1,
                                         None, None, None, None, 1, 0.125, None, 0, None, None)
    assert rc == _native.NIE_ERR_INVALID and b"null pointer" in lib.nie_last_error()
