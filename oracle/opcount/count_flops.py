"""Executed f32 operations per element of the reference encoders — TEST
INFRASTRUCTURE.

Runs the op-counting build of the oracle (opcount.hpp) on rows sampled from
the benchmark workloads and prints, per type, the executed operations per
input element by category.  The totals are the algorithmic FLOP figures the
benchmark's roofline uses.

  python oracle/opcount/count_flops.py [--rows 32]
"""
import argparse
import ctypes
import os
import subprocess
import sys

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE = os.path.dirname(_HERE)
_LIB_PATH = os.path.join(_HERE, "libopcount.so")
CATEGORIES = ("arith", "cmp", "sqrt", "round", "minmax", "f64")
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-s", "-C", _ORACLE, "opcount/libopcount.so"], check=True)
        L = ctypes.CDLL(_LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        L.oc_encode_rows.argtypes = [ctypes.c_uint32, f32p, ctypes.c_int64, ctypes.c_int64, f32p,
                                     ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_uint64)]
        _lib = L
    return _lib


def encode_counted(ty, x, im, row_bytes):
    """Encodes f32 rows x (n_rows, ne0); returns (codes, {category: count})."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_rows, ne0 = x.shape
    out = np.zeros((n_rows, row_bytes), np.uint8)
    cnt = np.zeros(6, np.uint64)
    imp = None if im is None else np.ascontiguousarray(im, np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    rc = lib().oc_encode_rows(ty, x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n_rows, ne0, imp,
                              out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                              cnt.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)))
    if rc != 0:
        raise RuntimeError(f"oc_encode_rows failed: {rc}")
    return out, dict(zip(CATEGORIES, (int(c) for c in cnt)))


def f32_ops(counts):
    """Total f32 operations (f64 work is reported apart)."""
    return sum(v for k, v in counts.items() if k != "f64")


def main():
    sys.path.insert(0, os.path.dirname(_ORACLE))
    import bench
    from oracle import oracle as O

    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32, help="rows sampled (evenly spaced) from each tensor")
    a = ap.parse_args()

    bits, im = bench.make_workload()
    sweep = [("4096x14336", bits, im)]
    iq = bench.make_iq_workload()
    print(f"{'type':8s} {'tensor':11s} " + " ".join(f"{c:>7s}" for c in CATEGORIES) + "   f32/elt")
    for types, tensors in ((bench.SWEEP, sweep), (bench.IQ_TYPES, iq)):
        for name in types:
            ty = bench.TYPE_IDS[name]
            tot, elts = 0, 0
            for tname, b, imt in tensors:
                rows = np.linspace(0, b.shape[0] - 1, a.rows).astype(np.int64)
                x = (b[rows].astype(np.uint32) << 16).view(np.float32)
                codes, c = encode_counted(ty, x, imt, O.row_bytes(ty, b.shape[1]))
                want = O.encode_tensor_bf16(ty, b[rows], imt)
                if not np.array_equal(codes, want):
                    raise SystemExit(f"{name}: counting build disagrees with the oracle")
                per = {k: v / x.size for k, v in c.items()}
                print(f"{name:8s} {tname:11s} " + " ".join(f"{per[k]:7.1f}" for k in CATEGORIES)
                      + f"   {f32_ops(c) / x.size:7.1f}")
                tot += f32_ops(c)
                elts += x.size
            print(f"{name:8s} {'(all)':11s} {'':63s}   {tot / elts:7.1f}")


if __name__ == "__main__":
    main()
