"""The C-ABI library loads on a machine without a GPU, exports every symbol that
include/sparseconv_b200.h declares, and its host-side sizing and argument validation
behave as documented (none of these calls reach the device)."""
import ctypes
import os
import re

import pytest

from sparseconv import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def _declared_functions():
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(spconv_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    return _native.load_library()


def test_header_declares_entry_points():
    names = _declared_functions()
    assert "spconv_build_submanifold_neighbor_map" in names
    assert "spconv_submanifold_conv_forward" in names


def test_every_declared_symbol_is_exported(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version(lib):
    assert lib.spconv_abi_version() == 1


def test_hashmap_capacity(lib):
    assert lib.spconv_hashmap_capacity(0) == 1024
    assert lib.spconv_hashmap_capacity(256) == 1024
    assert lib.spconv_hashmap_capacity(257) == 2048
    for m in (1000, 168546, 2_000_000, 1_342_011):       # load <= 0.25 while the table is <= 64 MB
        cap = lib.spconv_hashmap_capacity(m)
        assert cap >= 4 * m and cap & (cap - 1) == 0 and cap * 8 <= 64 << 20
    for m in (3_000_000, 5_000_000):                      # larger tables: load <= 0.5
        cap = lib.spconv_hashmap_capacity(m)
        assert 2 * m <= cap < 4 * m and cap & (cap - 1) == 0


def test_mask_words(lib):
    assert [lib.spconv_mask_words(v) for v in (1, 27, 32, 33, 125, 343)] == [1, 1, 1, 2, 4, 11]


def test_workspace_bytes(lib):
    cap = lib.spconv_hashmap_capacity(1000)
    # <= 2^30 cells: table + a one-bit-per-cell occupancy bitmap
    small_grid = lib.spconv_neighbor_map_workspace_bytes(1000, 4, 128, 128, 128)
    assert small_grid >= 8 * cap + 4 * 128 ** 3 // 8
    # 2^30 < cells < 2^32: table only, plus the sorted-input path's column ranges (8 bytes per
    # (b, x, y) column, at most 2^23 columns) and flat keys (4 bytes per voxel)
    mid_grid = lib.spconv_neighbor_map_workspace_bytes(1000, 16, 512, 512, 512)
    sorted_regions = 16 * 512 * 512 * 8 + (1000 * 4 + 255) // 256 * 256
    assert 8 * cap <= mid_grid - sorted_regions < 8 * cap + 64 * 1024
    # more than 2^23 columns: no sorted-input regions
    many_cols = lib.spconv_neighbor_map_workspace_bytes(1000, 64, 2048, 128, 128)
    assert 8 * cap <= many_cols < 8 * cap + 64 * 1024
    # >= 2^32 cells: 64-bit keys add a row array
    big_grid = lib.spconv_neighbor_map_workspace_bytes(1000, 2, 2048, 2048, 1024)
    assert big_grid >= 12 * cap and big_grid > mid_grid - sorted_regions
    assert lib.spconv_neighbor_map_workspace_bytes(-1, 1, 1, 1, 1) == -1


def test_argument_validation_before_any_launch(lib):
    nb = lib.spconv_build_submanifold_neighbor_map
    # bad kernel size / dilation / shape / count: SPCONV_ERR_ARG with a message
    assert nb(None, 10, 1, 4, 4, 4, 0, 3, 3, 1, 1, 1, None, 0, None, None, None, None, None) == 1
    assert b"kernel size" in lib.spconv_last_error()
    assert nb(None, 10, 1, 4, 4, 4, 3, 3, 3, 0, 1, 1, None, 0, None, None, None, None, None) == 1
    assert nb(None, -1, 1, 4, 4, 4, 3, 3, 3, 1, 1, 1, None, 0, None, None, None, None, None) == 1
    assert nb(None, 10, 0, 4, 4, 4, 3, 3, 3, 1, 1, 1, None, 0, None, None, None, None, None) == 1
    assert nb(None, 10, 1, 4, 4, 4, 11, 11, 11, 1, 1, 1, None, 0, None, None, None, None, None) == 1
    # null buffers for a non-empty input
    assert nb(None, 10, 1, 4, 4, 4, 3, 3, 3, 1, 1, 1, None, 0, None, None, None, None, None) == 1
    # empty input: nothing to do
    assert nb(None, 0, 1, 4, 4, 4, 3, 3, 3, 1, 1, 1, None, 0, None, None, None, None, None) == 0
    cf = lib.spconv_submanifold_conv_forward
    assert cf(None, 7, 10, 3, None, None, 3, 27, None, None, None, None, None, None) == 1   # dtype
    assert cf(None, 0, 10, 0, None, None, 3, 27, None, None, None, None, None, None) == 1   # Ci
    assert cf(None, 0, 10, 3, None, None, 3, 2000, None, None, None, None, None, None) == 1  # V
    assert cf(None, 0, 0, 3, None, None, 3, 27, None, None, None, None, None, None) == 0    # M=0
    ex = lib.spconv_submanifold_conv_forward_ex
    assert ex(None, 0, 10, 3, None, None, 3, 27, None, None, None, None, None, None, 9) == 1
    assert ex(ctypes.c_void_p(16), 0, 10, 3, ctypes.c_void_p(16), None, 3, 27, ctypes.c_void_p(16),
              None, None, ctypes.c_void_p(16), None, None, 2) == 3        # tcgen05: no fp32 path


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _native.load_library(str(tmp_path / "absent.so"))


def test_wait_limit_setter_round_trip(lib):
    default = _native.set_wait_limit_ns(0)            # 0 restores the default
    assert default == 2_000_000_000
    assert _native.set_wait_limit_ns(12345) == default
    assert _native.set_wait_limit_ns(0) == 12345
    assert _native.set_wait_limit_ns(0) == default
