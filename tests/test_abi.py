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


def test_exchange_layout_and_argument_checks_without_gpu():
    """Host-side checks of the expert-parallel and incremental-assignment
    entry points: sizes and null pointers are rejected before any device
    work."""
    import ctypes as C

    from skcq_b200 import _lib

    offs = (C.c_int64 * 6)()
    assert _lib.call("skcq_ep_layout", 2, 16, 8, 64, offs) == 0
    rows, ids, wts, cnt, ret, total = list(offs)
    assert rows == 0 and ids >= 2 * 16 * 64 * 4 and wts >= ids + 2 * 16 * 8 * 4 and cnt > wts
    assert ret > cnt and total >= ret + 2 * 16 * 64 * 4
    assert all(v % 256 == 0 for v in offs)
    with pytest.raises(RuntimeError, match="bad sizes"):
        _lib.call("skcq_ep_layout", 9, 16, 8, 64, offs)  # more ranks than one node has
    with pytest.raises(RuntimeError, match="bad sizes"):
        _lib.call("skcq_ep_layout", 2, 16, 32, 64, offs)  # top-k above 31
    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("skcq_moved_lists", None, None, 1, 256, 128, None, None, None, None, None, None, None, None, 0,
                  None)
    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("skcq_assign_merge", 1, None, None, None, 1, 256, 128, 4, None, None, None, None, None, None, None,
                  None, 0, None, None, None, None, None, None)
    with pytest.raises(RuntimeError, match="null pointer"):
        _lib.call("skcq_list_points", None, 1, 256, None, None, None, None, None, 0, None)
    assert _lib.load().skcq_moved_lists_scratch_bytes(3, 8192, 4096) == 3 * (2 + 1) * 4


def test_grid_cell_counts_stay_within_the_kernel_limits():
    """The engine's cells-per-coordinate choice for the centroid grid
    (about one centroid per cell) is accepted by the library for every block
    size and centroid count it can be given, and the library rejects shapes
    outside its limits (bs in 2..4, 2 <= G <= 256, bs (G - 1) <= 1024,
    G^bs <= 2^20)."""
    from skcq_b200 import _engine, _lib

    lib = _lib.load()
    for bs in (2, 3, 4):
        for k in (_engine.GRID_MIN_K, 16384, 65536, 1 << 20):
            G = _engine.grid_cells(bs, k)
            assert 2 <= G <= 256 and bs * (G - 1) <= 1024 and G ** bs <= (1 << 20), (bs, k, G)
            assert lib.skcq_assign_grid_scratch_bytes(4, 98304, k, bs, G) > 0, (bs, k, G)
    assert _engine.grid_cells(4, 65536) == 16  # one centroid per cell at the layer's second residual
    assert lib.skcq_assign_grid_scratch_bytes(4, 1024, 8192, 5, 8) == 0  # block size 5
    assert lib.skcq_assign_grid_scratch_bytes(4, 1024, 8192, 4, 33) == 0  # 33^4 cells > 2^20
    assert lib.skcq_assign_grid_scratch_bytes(4, 1024, 8192, 2, 257) == 0
    assert lib.skcq_assign_grid_scratch_bytes(4, 1024, 8192, 4, 1) == 0
    # the layout grows with every dimension it holds
    a = lib.skcq_assign_grid_scratch_bytes(2, 98304, 65536, 4, 16)
    assert lib.skcq_assign_grid_scratch_bytes(4, 98304, 65536, 4, 16) > a
    assert lib.skcq_assign_grid_scratch_bytes(2, 2 * 98304, 65536, 4, 16) > a
