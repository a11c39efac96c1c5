"""The C-ABI library: it loads without a GPU and exports every declared entry point."""

from __future__ import annotations

import ctypes
import re

from .conftest import ROOT

HEADER = ROOT / "include" / "microserve_b200.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"MS_API\s+[\w\s\*]+?\b(ms_\w+)\s*\(", text)))


def test_header_declares_the_boundary() -> None:
    names = declared()
    for must in ("ms_forward", "ms_sample", "ms_spec_accept", "ms_verify_probs",
                 "ms_kv_write", "ms_kv_gather", "ms_paged_attention", "ms_gemm"):
        assert must in names


def test_library_loads_and_exports_every_declared_symbol() -> None:
    from microserve_b200 import _lib

    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared()) == set(_lib.exported_names())
    assert lib.ms_version() >= 1
    assert isinstance(lib.ms_launch_count(), int)


def test_invalid_arguments_fail_on_the_host() -> None:
    """Argument validation happens before any CUDA call, so it works without a GPU."""
    from microserve_b200 import _lib

    lib = _lib.load()
    rc = lib.ms_gemm(None, None, None, None, 4, 4, 4, 0, 0, 0, 0, None)
    assert rc == _lib.MS_ERR_INVALID
    assert b"null pointer" in lib.ms_last_error()
    rc = lib.ms_spec_accept(None, 0, None, 0, None, 0, None, None, 4, 0, 10, None, None, None)
    assert rc == _lib.MS_ERR_INVALID


def test_struct_layouts_match_the_header() -> None:
    from microserve_b200 import _lib

    assert ctypes.sizeof(_lib.MsKVCache) == 6 * 4 + 2 * 8
    assert ctypes.sizeof(_lib.MsBatch) == 6 * 4 + 6 * 8
    assert _lib.SAMPLING_PARAMS_DTYPE.itemsize == 32
    assert _lib.ROW_STATS_DTYPE.itemsize == 16


def test_host_table_helpers_check_before_changing_anything() -> None:
    """ms_host_append / ms_host_truncate refuse a bad batch as a whole."""
    import numpy as np

    from microserve_b200 import _lib

    lib = _lib.load()

    def a(x: np.ndarray) -> int:
        return x.__array_interface__["data"][0]

    bs, stride = 4, 3
    rows = np.array([0, 1], np.int64)
    ntok = np.array([3, 8], np.int64)
    nblk = np.array([1, 2], np.int32)
    table = np.array([[5, 0, 0], [6, 7, 0]], np.int32)
    before = (ntok.copy(), nblk.copy(), table.copy())
    slots = np.zeros(16, np.int64)
    widest = ctypes.c_int64(0)
    counts = np.array([2, 1], np.int64)
    assert lib.ms_host_blocks_needed(a(rows), a(counts), 2, a(ntok), a(nblk), bs,
                                     ctypes.addressof(widest)) == 2
    assert widest.value == 3
    blocks = np.array([9], np.int32)  # one block short
    assert lib.ms_host_append(a(rows), a(counts), 2, a(ntok), a(nblk), a(table), stride, bs,
                              a(blocks), 1, a(slots)) == _lib.MS_ERR_INVALID
    too_wide = np.array([0, 5], np.int64)  # row 1 would need 4 blocks of 3
    assert lib.ms_host_append(a(rows), a(too_wide), 2, a(ntok), a(nblk), a(table), stride, bs,
                              a(blocks), 1, a(slots)) == _lib.MS_ERR_INVALID
    out = np.zeros(8, np.int32)
    grow = np.array([2, 9], np.int64)
    assert lib.ms_host_truncate(a(rows), a(grow), 2, a(ntok), a(nblk), a(table), stride, bs,
                                a(out), out.size) == -1
    assert all(np.array_equal(x, y) for x, y in zip((ntok, nblk, table), before))
    # the good batch: row 0 fills its block 5 (slot 23), then takes block 9
    # (slot 36); row 1's ninth token opens new block 11 (slot 44)
    blocks = np.array([9, 11], np.int32)
    assert lib.ms_host_append(a(rows), a(counts), 2, a(ntok), a(nblk), a(table), stride, bs,
                              a(blocks), 2, a(slots)) == 0
    assert slots[:3].tolist() == [23, 36, 44]
    assert ntok.tolist() == [5, 9] and nblk.tolist() == [2, 3]
    assert table.tolist() == [[5, 9, 0], [6, 7, 11]]
    shrink = np.array([1, 4], np.int64)
    assert lib.ms_host_truncate(a(rows), a(shrink), 2, a(ntok), a(nblk), a(table), stride, bs,
                                a(out), out.size) == 3
    # blocks past each new end, row by row in table order
    assert out[:3].tolist() == [9, 7, 11] and nblk.tolist() == [1, 1] and ntok.tolist() == [1, 4]
