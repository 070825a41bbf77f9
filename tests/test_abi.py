"""The C ABI: the in-tree library loads without a GPU and exports every entry
point that include/skcq_b200.h declares (no device work is done here)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "skcq_b200.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|size_t)\s+(skcq_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "skcq_assign" in names and "skcq_reconstruct" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol():
    from skcq_b200 import _lib

    lib = _lib.load()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding types every declared entry point
    untyped = [n for n in declared() if n not in _lib.exported_symbols()]
    assert not untyped, untyped


def test_host_helpers_without_gpu():
    from skcq_b200 import _lib

    lib = _lib.load()
    assert lib.skcq_abi_version() >= 1
    assert lib.skcq_packed_width(1, 4) == 16  # 3*4 + 2 bias -> 16
    assert lib.skcq_packed_width(0, 8) == 24
    assert lib.skcq_packed_width(1, 16) == 56
    assert lib.skcq_packed_width(0, 0) < 0
    assert "block size" in _lib.last_error()
    assert lib.skcq_reseed_scratch_bytes(4, 128) == 4 * (128 * 4 + 128 * 8)


def test_null_pointers_are_rejected_without_touching_the_device():
    from skcq_b200 import _lib

    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("skcq_assign", 0, None, None, None, None, None, 1, 256, 128, 4, None, None, None, None, None)
    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("skcq_reconstruct", None, 1, 1, 1, None, 0, None, 0, None)
