"""The C-ABI library: it loads, exports every symbol include/shoehorn_cuda.h
declares, and answers the host-only queries without a GPU."""
import ctypes
import os
import re

import pytest

import shoehorn_b200 as sh

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "shoehorn_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(shc_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(sh.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), n


def test_row_bytes_matches_reference_layout():
    for ty in sh.GgmlType:
        bs, tb = ty.block_layout()
        assert sh.row_bytes(ty, bs * 7) == tb * 7
        if bs > 1:
            assert sh.row_bytes(ty, bs * 7 + 1) == -1
    assert sh.row_bytes(99, 256) == -1


def test_supported_types():
    for ty in (sh.GgmlType.Q8_0, sh.GgmlType.Q4_K, sh.GgmlType.Q5_K, sh.GgmlType.Q6_K, sh.GgmlType.F16):
        assert sh.type_supported(ty)
    assert not sh.type_supported(99)


def test_status_strings():
    L = sh.lib()
    assert L.shc_status_string(0) == b"ok"
    assert L.shc_status_string(-3) == b"IQ point off the lattice"


def test_invalid_arguments_rejected_without_gpu():
    L = sh.lib()
    assert L.shc_free(None) == -1
    assert L.shc_encode_rows(None, 12, 30, None, 0, 256, None, 0, 0, 0, None, None) == -1
    out = ctypes.c_void_p()
    rc = L.shc_init(0, ctypes.byref(out))
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        assert rc == -7  # SHC_ENODEV
    elif rc == 0:
        L.shc_free(out)


def test_grid_info_host_only():
    gs, kmap, nb = sh.grid_info(0)
    assert gs == 256 and kmap.size == 6561
    assert int((kmap >= 0).sum()) == 256
    gs, kmap, nb = sh.grid_info(4)
    assert gs == 512 and kmap.size == 4096 and int((kmap >= 0).sum()) == 512


def test_negative_row_indices_rejected_before_any_launch():
    """Global row indices and matrix heights are unsigned in the reference
    (imatrix.rs:124 row_slice takes usize): negative ones are refused before
    anything touches a device."""
    L = sh.lib()
    f = L.shc_encode_rows_noalloc
    f.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    assert f(12, 30, 256, 4, 256, 256, 512, 2, -1, 256, None) == -1   # row0 < 0
    assert f(12, 30, 256, 4, 256, 256, 512, -2, 0, 256, None) == -1   # rows_per_mat < 0
    assert L.shc_encode_tensor_host(None, 12, 30, None, 1, 256, None, 0, 0, -1, None, 0) == -1
