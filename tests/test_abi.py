"""The C ABI (include/trispconv_b200.h) without a GPU: the library builds,
loads, exports every declared symbol, and rejects bad arguments on the host
before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from trispconv_b200 import _lib as L

HEADER = Path(__file__).resolve().parent.parent / "include" / "trispconv_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^TSC_API\s+[\w\s\*]+?\b(tsc_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not L.LIB_PATH.exists():
        from trispconv_b200.build import build

        build()
    return L.load()


def test_header_declares_the_bound_symbols():
    decl = declared_symbols()
    assert len(decl) >= 17
    assert set(decl) == set(L.EXPORTED), set(decl) ^ set(L.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(L.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_abi_version_and_introspection(lib):
    assert lib.tsc_abi_version() == 1
    assert isinstance(L.launch_count(), int)
    assert isinstance(L.last_error(), str)


def test_workspace_sizes(lib):
    # 12 bytes per slot (a 64-bit key + a row, for grids above 2^32 - 2 cells),
    # 2^ceil(log2 8n) slots (at least 2^10)
    assert lib.tsc_subm_kmap_workspace(0) == 12 << 10
    assert lib.tsc_subm_kmap_workspace(1000) == 12 << 13         # 8n rounded up to 2^13
    assert lib.tsc_subm_kmap_workspace(160000) == 12 << 21
    g = L.make_geometry(4, (41, 1600, 1408), (21, 800, 704), (3, 3, 3), (2, 2, 2), (1, 1, 1))
    ws = lib.tsc_strided_kmap_workspace(ctypes.byref(g))
    bits = 4 * 21 * 800 * 704
    assert ws >= 2 * (bits // 8)                                  # bitmap + word prefix
    assert lib.tsc_pairs_workspace(27, 1000) > 0
    assert lib.tsc_inverse_kmap_workspace(1000) > 0


def test_host_side_argument_checks(lib):
    """Rejected before any CUDA call, so this runs without a GPU."""
    meta = ctypes.c_int64 * 64
    m, s = meta(), meta()
    bad = L.make_geometry(0, (4, 4, 4), (4, 4, 4), (3, 3, 3))
    rc = lib.tsc_subm_kmap(None, 10, ctypes.byref(bad), None, 0, None, ctypes.addressof(m),
                           ctypes.addressof(s), None)
    assert rc == L.TSC_ERR_INVALID_ARG and "batch" in L.last_error()
    g = L.make_geometry(1, (4, 4, 4), (4, 4, 4), (3, 3, 3))
    rc = lib.tsc_subm_kmap(None, -1, ctypes.byref(g), None, 0, None, ctypes.addressof(m),
                           ctypes.addressof(s), None)
    assert rc == L.TSC_ERR_INVALID_ARG
    # 2^63 cells: beyond the 64-bit key range (2^62)
    big = L.make_geometry(1 << 30, (1 << 11, 1 << 11, 1 << 11), (4, 4, 4), (3, 3, 3))
    rc = lib.tsc_subm_kmap(None, 1, ctypes.byref(big), None, 0, None, ctypes.addressof(m),
                           ctypes.addressof(s), None)
    assert rc == L.TSC_ERR_GRID_TOO_LARGE and "2^62" in L.last_error()
    # 2^50 cells: accepted (64-bit keys); the call then stops at its undersized
    # workspace, before any CUDA call (the pointers are never dereferenced)
    wide = L.make_geometry(1 << 20, (1 << 10, 1 << 10, 1 << 10), (1 << 10, 1 << 10, 1 << 10), (3, 3, 3))
    rc = lib.tsc_subm_kmap(1 << 20, 1, ctypes.byref(wide), 1 << 20, 16, 1 << 20, ctypes.addressof(m),
                           ctypes.addressof(s), None)
    # the message names the smallest workspace the call takes: 12 bytes x 2^8 slots
    assert rc == L.TSC_ERR_WORKSPACE and str(12 << 8) in L.last_error()
    assert lib.tsc_subm_kmap_workspace(1) == 12 << 10
    rc = lib.tsc_conv_forward(None, 0, 10, 0, None, 0, None, None, None, 27, 10, 8, None, 0, None, None, 0,
                              ctypes.addressof(s), None, None)
    assert rc == L.TSC_ERR_INVALID_ARG
    rc = lib.tsc_conv_forward(None, 0, 10, 4, None, 0, None, None, None, 27, 10, 8, None, 0, None, None, 0,
                              ctypes.addressof(s), None, None)
    assert rc == L.TSC_ERR_INVALID_ARG and "identity" in L.last_error()
    rc = lib.tsc_pairs_materialize(None, 27, 10, 7, None, None, None, 5, None, 0, None, None)
    assert rc == L.TSC_ERR_INVALID_ARG


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(L.LibraryMissing):
        L.load(tmp_path / "nope.so")
