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
