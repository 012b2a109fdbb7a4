"""bench.py pieces that run without a GPU: workload generation and the
JSON contract of the reference (CPU) arm on a tiny sample."""
import json
import subprocess
import sys

import numpy as np

import bench


def test_workloads_have_the_named_shapes():
    bits, im = bench.workloads.sweep_tensor()
    assert bits.shape == (4096, 14336) and bits.dtype == np.uint16 and im.shape == (14336,)
    iq = bench.workloads.iq_tensors()
    assert [t[1].shape for t in iq] == [(4096, 4096), (14336, 4096)]


def test_row_shards_partition_every_tensor():
    for n in (1, 7, 1024, 4096, 14336, 128256):
        for world in (1, 2, 3, 4, 8):
            ranges = [bench.shard_rows(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


def test_model_cpu_baseline_extrapolates_from_a_sample():
    """The CPU restatement timed on a small sample of the Llama-3-8B shape's
    error table and encode, extrapolated by rows and elements per type."""
    cb = bench.cpu_model_baseline({"Q4_K": 4096 * 4096, "F16": 100})
    assert cb["measure_s"] > 0 and cb["encode_s"] > 0 and cb["measure_exact_s"] > cb["measure_s"]
    assert cb["kind"] == "port" and "extrapolated" in cb["sample"]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--types", "Q8_0", "--ref-budget", "0.2"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"


def test_model_budgets_leave_the_configured_weight_budget():
    """--budget = weights + f16 KV at ctx 8192 + the compute estimate
    (main.rs:294-337 with --reserve 0): 5.5 GiB for the 8B shape, 40 GiB for
    the 70B shape."""
    for name, gib in (("llama3-8b", 5.5), ("llama3-70b", 40.0)):
        m = bench.MODELS[name]
        kv = m["layers"] * 8192 * 8 * 256 * 2
        compute = 512 * m["vocab"] * 4 + 512 * m["hidden"] * 32
        assert int(bench.model_budget_arg(name)) - kv - compute == int(gib * (1 << 30))
    assert bench.model_budget_arg("llama3-8b") == "7309099008"
    names = [s[0] for s in bench.model_shapes("llama3-70b")]
    assert names[-2:] == ["token_embd", "output"] and sum(s[4] for s in bench.model_shapes("llama3-70b")) == 562
