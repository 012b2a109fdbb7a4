"""Python front-end of the host pipeline library (libshoehorn_host.so): the
plan / quantize flow of the reference (src/main.rs:454-751) over the CUDA
library, for synthetic models of the benchmark configurations, on one rank
of a job that runs one process per GPU.

The ranks exchange only the measured per-row errors (an all-gather of f64
rows, src/main.rs:546-560 then sums them in row order) through callbacks
into this process's torch.distributed group; encoding needs no exchange.
"""
import ctypes
import json
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
HOST_LIB_PATH = os.path.join(_HERE, "libshoehorn_host.so")

ALLGATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                ctypes.c_int64, ctypes.c_void_p)
BARRIER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(HOST_LIB_PATH):
            raise ImportError(f"{HOST_LIB_PATH} is missing: run `python -m shoehorn_b200.build`")
        L = ctypes.CDLL(HOST_LIB_PATH)
        L.shh_shard_exchange_check.restype = ctypes.c_int
        L.shh_shard_exchange_check.argtypes = [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                               ctypes.c_int, ctypes.c_int, ALLGATHER_FN, ctypes.c_void_p,
                                               ctypes.c_void_p]
        L.shh_bench_model.restype = ctypes.c_int
        L.shh_bench_model.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p,
                                      ctypes.c_uint64, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ALLGATHER_FN, BARRIER_FN, ctypes.c_void_p, ctypes.c_char_p,
                                      ctypes.c_char_p, ctypes.c_int64]
        _lib = L
    return _lib


class Comm:
    """The two callbacks a sharded run needs, over torch.distributed's default
    group (or, with world == 1, over nothing).  Keeps the ctypes callback
    objects alive for as long as it lives."""

    def __init__(self, rank=0, world=1):
        self.rank, self.world = rank, world
        self._blobs = None

        def allgather(_user, mine, n, out, cap, sizes):
            try:
                if not out:
                    data = ctypes.string_at(mine, n) if n else b""
                    if self.world == 1:
                        self._blobs = [data]
                    else:
                        import torch.distributed as dist
                        blobs = [None] * self.world
                        dist.all_gather_object(blobs, data)
                        self._blobs = blobs
                    return sum(len(b) for b in self._blobs)
                total = sum(len(b) for b in self._blobs)
                if total > cap:
                    return -1
                buf = (ctypes.c_uint8 * cap).from_address(out)
                sz = (ctypes.c_int64 * self.world).from_address(sizes)
                at = 0
                for r, b in enumerate(self._blobs):
                    buf[at:at + len(b)] = b
                    sz[r] = len(b)
                    at += len(b)
                self._blobs = None
                return total
            except Exception:
                return -1

        def barrier(_user):
            try:
                if self.world > 1:
                    import torch.distributed as dist
                    dist.barrier()
                return 0
            except Exception:
                return -1

        self.allgather = ALLGATHER_FN(allgather)
        self.barrier = BARRIER_FN(barrier)


def shard_exchange_check(n_rows, n_cands, sample_rows=128, comm=None):
    """Error-table exchange on made-up errors (no GPU): [n_tensors, max_cands]
    per-(tensor, candidate) errors after the exchange and the row-order sums."""
    comm = comm or Comm()
    n_rows = np.ascontiguousarray(n_rows, dtype=np.uint64)
    n_cands = np.ascontiguousarray(n_cands, dtype=np.int32)
    sums = np.zeros((len(n_rows), int(n_cands.max())), dtype=np.float64)
    rc = lib().shh_shard_exchange_check(len(n_rows), n_rows.ctypes.data, n_cands.ctypes.data, sample_rows, comm.rank,
                                        comm.world, comm.allgather, None, sums.ctypes.data)
    if rc != 0:
        raise RuntimeError("shard exchange failed")
    return sums


def bench_model(name, device=0, exact_errors=False, budget=None, reserve="0", ctx=8192, uniform="",
                workers_per_gpu=3, seed=20261201, out_path="", comm=None):
    """Error table + solve + encode of a synthetic model on this rank's rows.
    Returns the timing record (dict)."""
    comm = comm or Comm()
    buf = ctypes.create_string_buffer(1 << 16)
    rc = lib().shh_bench_model(name.encode(), seed, int(exact_errors), (budget or "").encode() or None,
                               reserve.encode() if reserve is not None else None, ctx, uniform.encode(),
                               workers_per_gpu, device, comm.rank, comm.world, comm.allgather, comm.barrier, None,
                               out_path.encode(), buf, len(buf))
    if rc != 0:
        raise RuntimeError(f"bench_model {name}: {buf.value.decode(errors='replace')}")
    return json.loads(buf.value.decode())
