"""bench.py's multi-rank plumbing on CPU: two gloo ranks (the GPU run uses
the same code over NCCL, one rank per GPU)."""
import os
import socket
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r, lr, w = bench.dist_env()
        step_ms = 10.0 + 5.0 * rank  # the slower rank sets the job's time
        got = bench.max_over_ranks(step_ms, torch.device("cpu"))
        value = bench.aggregate_gbs(1_000_000_000, 4, got * 1e-3)
        dist.barrier()
        q.put((r, lr, w, got, value))
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_strong_scaling_aggregate():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for r, (rank, lrank, w, got, value) in enumerate(res):
        assert (rank, lrank, w) == (r, r, 2)
        assert got == 15.0  # max over ranks, identical on every rank
        assert abs(value - 4 * 1.0 / 0.015) < 1e-9  # GB/s of the whole tensor, shared by the ranks


def test_max_over_ranks_without_a_process_group():
    assert bench.max_over_ranks(3.5, torch.device("cpu")) == 3.5


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and r.stdout.strip() == ""
