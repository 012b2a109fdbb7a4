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
        L.shh_bench_model.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                      ctypes.c_char_p,
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
                    self._blobs = self._gather(mine, n)
                    return int(sum(b.size for b in self._blobs))
                total = int(sum(b.size for b in self._blobs))
                if total > cap:
                    return -1
                sz = (ctypes.c_int64 * self.world).from_address(sizes)
                at = 0
                for r, b in enumerate(self._blobs):
                    if b.size:
                        ctypes.memmove(out + at, b.ctypes.data, b.size)
                    sz[r] = b.size
                    at += b.size
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

    def _gather(self, mine, n):
        """Every rank's bytes (numpy uint8 arrays, rank order): sizes first,
        then one all-gather of the blobs padded to the largest (on the GPU
        under NCCL, in host memory under gloo)."""
        data = np.frombuffer(ctypes.string_at(mine, n), dtype=np.uint8) if n else np.zeros(0, np.uint8)
        if self.world == 1:
            return [data]
        import torch
        import torch.distributed as dist
        dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
        size = torch.tensor([data.size], dtype=torch.int64, device=dev)
        sizes = [torch.zeros_like(size) for _ in range(self.world)]
        dist.all_gather(sizes, size)
        sizes = [int(x.item()) for x in sizes]
        mx = max(sizes)
        buf = torch.zeros(mx, dtype=torch.uint8, device=dev)
        if data.size:
            buf[:data.size] = torch.from_numpy(data.copy()).to(dev)
        outs = [torch.empty(mx, dtype=torch.uint8, device=dev) for _ in range(self.world)]
        dist.all_gather(outs, buf)
        return [o[:sz].cpu().numpy() for o, sz in zip(outs, sizes)]


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


def bench_model(name, device=0, modes=("sampled",), budget=None, reserve="0", ctx=8192, uniform="",
                workers_per_gpu=4, seed=20261201, out_path="", streaming=False, comm=None):
    """Error table + solve + encode of a synthetic model on this rank's rows,
    once per mode ("sampled": the reference's 128-row error table, "exact":
    every row).  streaming: rows are generated as the pipeline asks for them
    (no weight storage); out_path "-" discards the encoded bytes after their
    copy to the host.  Returns the timing records (list of dicts)."""
    comm = comm or Comm()
    bits = (1 if "sampled" in modes else 0) | (2 if "exact" in modes else 0)
    buf = ctypes.create_string_buffer(1 << 16)
    rc = lib().shh_bench_model(name.encode(), seed, bits, int(streaming), (budget or "").encode() or None,
                               reserve.encode() if reserve is not None else None, ctx, uniform.encode(),
                               workers_per_gpu, device, comm.rank, comm.world, comm.allgather, comm.barrier, None,
                               out_path.encode(), buf, len(buf))
    if rc != 0:
        raise RuntimeError(f"bench_model {name}: {buf.value.decode(errors='replace')}")
    return json.loads(buf.value.decode())
