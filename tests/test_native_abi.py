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
