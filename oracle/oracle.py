"""ctypes front-end of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker or the timed CPU restatement of the reference.
The shipped library (shoehorn_b200) never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)
_c_f64p = ctypes.POINTER(ctypes.c_double)
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_i64p = ctypes.POINTER(ctypes.c_int64)


def build(force=False):
    """Compile liboracle.so with the strict-FP flags of oracle/Makefile."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oq_row_bytes.restype = ctypes.c_int64
        L.oq_row_bytes.argtypes = [ctypes.c_uint32, ctypes.c_int64]
        L.oq_encode_row.argtypes = [ctypes.c_uint32, _c_f32p, ctypes.c_int64, _c_f32p, _c_u8p]
        L.oq_decode_row.argtypes = [ctypes.c_uint32, _c_u8p, ctypes.c_int64, _c_f32p]
        L.oq_row_error.argtypes = [ctypes.c_uint32, _c_f32p, ctypes.c_int64, _c_f32p, _c_f64p]
        L.oq_encode_tensor_bf16.argtypes = [ctypes.c_uint32, _c_u16p, ctypes.c_int64, ctypes.c_int64, _c_f32p,
                                            ctypes.c_int64, ctypes.c_int64, _c_u8p, ctypes.c_int]
        L.oq_row_errors_bf16.argtypes = [ctypes.c_uint32, _c_u16p, ctypes.c_int64, ctypes.c_int64, _c_f32p,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _c_f64p, ctypes.c_int]
        L.oq_grid_info.argtypes = [ctypes.c_int, _c_i32p, _c_i32p, _c_i64p, _c_i32p, _c_u16p]
        L.oq_f32_to_f16.restype = ctypes.c_uint16
        L.oq_f32_to_f16.argtypes = [ctypes.c_float]
        L.oq_f16_to_f32.restype = ctypes.c_float
        L.oq_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oq_nearest_int.restype = ctypes.c_int32
        L.oq_nearest_int.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


class OracleError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise OracleError(f"{what} failed with status {rc}")


def row_bytes(ty, n):
    return int(lib().oq_row_bytes(ty, n))


def encode_row(ty, x, im=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    im = None if im is None else np.ascontiguousarray(im, dtype=np.float32)
    rb = row_bytes(ty, x.size)
    if rb < 0:
        raise OracleError(f"type {ty} cannot encode a row of {x.size}")
    out = np.zeros(rb, dtype=np.uint8)
    _check(lib().oq_encode_row(ty, _p(x, _c_f32p), x.size, _p(im, _c_f32p), _p(out, _c_u8p)), "encode_row")
    return out


def decode_row(ty, data, n):
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    _check(lib().oq_decode_row(ty, _p(data, _c_u8p), n, _p(out, _c_f32p)), "decode_row")
    return out


def row_error(ty, x, im=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    im = None if im is None else np.ascontiguousarray(im, dtype=np.float32)
    e = ctypes.c_double(0.0)
    _check(lib().oq_row_error(ty, _p(x, _c_f32p), x.size, _p(im, _c_f32p), ctypes.byref(e)), "row_error")
    return e.value


def encode_tensor_bf16(ty, src_u16, im=None, rows_per_mat=0, n_threads=None):
    """src_u16: [n_rows, ne0] uint16 BF16 bits. Returns [n_rows, row_bytes] uint8."""
    src = np.ascontiguousarray(src_u16, dtype=np.uint16)
    n_rows, ne0 = src.shape
    im = None if im is None else np.ascontiguousarray(im, dtype=np.float32)
    rb = row_bytes(ty, ne0)
    out = np.zeros((n_rows, rb), dtype=np.uint8)
    nt = n_threads or os.cpu_count() or 1
    _check(lib().oq_encode_tensor_bf16(ty, _p(src, _c_u16p), n_rows, ne0, _p(im, _c_f32p),
                                       0 if im is None else im.size, rows_per_mat or n_rows,
                                       _p(out, _c_u8p), nt), "encode_tensor_bf16")
    return out


def row_errors_bf16(ty, src_u16, im=None, row_step=1, rows_per_mat=0, n_threads=None):
    src = np.ascontiguousarray(src_u16, dtype=np.uint16)
    n_rows, ne0 = src.shape
    im = None if im is None else np.ascontiguousarray(im, dtype=np.float32)
    n_s = (n_rows + row_step - 1) // row_step
    out = np.zeros(n_s, dtype=np.float64)
    nt = n_threads or os.cpu_count() or 1
    _check(lib().oq_row_errors_bf16(ty, _p(src, _c_u16p), n_rows, ne0, _p(im, _c_f32p),
                                    0 if im is None else im.size, rows_per_mat or n_rows, row_step,
                                    _p(out, _c_f64p), nt), "row_errors_bf16")
    return out


def grid_info(which):
    """(grid_size, kmap int32[kmap_size], neighbours uint16[n]) of quant_iq.rs build_grid."""
    gs, ks, nn = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
    _check(lib().oq_grid_info(which, ctypes.byref(gs), ctypes.byref(ks), ctypes.byref(nn), None, None), "grid_info")
    kmap = np.zeros(ks.value, dtype=np.int32)
    nb = np.zeros(nn.value, dtype=np.uint16)
    _check(lib().oq_grid_info(which, None, None, None, _p(kmap, _c_i32p), _p(nb, _c_u16p)), "grid_info")
    return gs.value, kmap, nb


def f32_to_f16_bits(x):
    return int(lib().oq_f32_to_f16(float(x)))


def nearest_int(x):
    return int(lib().oq_nearest_int(float(x)))
