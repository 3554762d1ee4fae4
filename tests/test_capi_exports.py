"""The C-ABI library loads and exports every entry point include/omni_b200.h declares.

No compute call is made here (CPU-only test); only symbol presence and the
pure-host entry points.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    return sorted(set(re.findall(r"OMNI_API\s+[\w\s\*]+?\b(omni_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "omni_sample_topk_topp" in names and "omni_version" in names


def test_library_exports_every_declared_symbol():
    from omni_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string():
    from omni_b200 import _lib

    lib = _lib.load()
    assert b"sm_100a" in lib.omni_version()
    assert isinstance(lib.omni_last_error(), bytes)


def test_unsupported_contract_is_reported_without_launch():
    """An off-ladder width is rejected on the host before any device work."""
    from omni_b200 import _lib

    lib = _lib.load()
    rc = lib.omni_sample_topk_topp(None, 4, 2048, 2048, None, None, None, None, None, 7, 0, None, None)
    assert rc == _lib.OMNI_ERR_UNSUPPORTED
    assert "ladder" in _lib.last_error()
    assert lib.omni_sample_sorted_seeded(None, None, 1, 0, None, None, None, None) == _lib.OMNI_ERR_UNSUPPORTED
    assert ctypes.sizeof(ctypes.c_void_p) == 8
