"""Row-range sharding of the error table across ranks (one process per GPU):
the only exchange is an all-gather of the per-row f64 errors each rank
measured, after which every rank sums each tensor's rows in row order
(main.rs:553-555).  On CPU with gloo ranks and made-up errors: the sums after
the exchange must equal the single-rank sums bit for bit, for uneven splits,
sampled and exact tables."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from shoehorn_b200 import host  # noqa: E402

# tensor heights of the benchmark models (q/k/v/o, FFN, vocabularies), plus
# heights below and just above the 128-row sample and a single row
N_ROWS = [4096, 1024, 1024, 4096, 14336, 14336, 4096, 128256, 151936, 2048, 3072, 100, 129, 128, 1, 7]
N_CANDS = [11, 11, 11, 11, 11, 11, 11, 6, 6, 11, 11, 7, 7, 7, 1, 3]
EXACT = 2 ** 64 - 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, sample_rows, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sums = host.shard_exchange_check(N_ROWS, N_CANDS, sample_rows, host.Comm(rank, world))
        q.put((rank, sums.tobytes()))
    finally:
        dist.destroy_process_group()


def _run_ranks(world, sample_rows):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, sample_rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("sample_rows", [128, EXACT], ids=["sampled", "exact"])
def test_exchanged_error_table_equals_single_rank(world, sample_rows):
    want = host.shard_exchange_check(N_ROWS, N_CANDS, sample_rows).tobytes()
    got = _run_ranks(world, sample_rows)
    for r in range(world):
        assert got[r] == want, f"rank {r} of {world}"


def test_every_sampled_row_is_owned_by_exactly_one_rank():
    """The row ranges partition each tensor, so each sampled row is measured
    once: without the exchange a rank's sums cover only its own rows."""
    ones = host.shard_exchange_check(N_ROWS, N_CANDS)
    assert np.all(ones[np.arange(len(N_ROWS)), 0] > 0)


def _rows(name, tensor, r0, n, mode, rank=0, world=1, ne0=256):
    import ctypes
    L = host.lib()
    L.shh_synthetic_rows.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    out = np.zeros(n * ne0, dtype=np.uint16)
    assert L.shh_synthetic_rows(name.encode(), 20261201, tensor, r0, n, mode, rank, world, out.ctypes.data) == 0
    return out


def test_streamed_and_sharded_synthetic_rows_equal_the_whole_model():
    """The synthetic weights are a function of (tensor, element), so a rank's
    shard and the streaming source (rows generated on demand, the 70B
    shape's way) give the same bytes as the model held whole."""
    # tiny: tensor 1 is token_embd-adjacent attn_q [256 x 256]; tensor 0 token_embd [256 x 256]
    for tensor in (0, 2):
        whole = _rows("tiny", tensor, 0, 256, 0)
        assert np.array_equal(_rows("tiny", tensor, 0, 256, 2), whole)
        assert np.array_equal(_rows("tiny", tensor, 128, 128, 1, rank=1, world=2), whole[128 * 256:])
        assert np.array_equal(_rows("tiny", tensor, 37, 5, 2), whole[37 * 256:42 * 256])
    x = (whole.astype(np.uint32) << 16).view(np.float32)
    assert abs(float(x.std()) - 0.02) < 0.002 and abs(float(x.mean())) < 0.002
