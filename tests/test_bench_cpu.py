"""bench.py pieces that run without a GPU: workload generation and the
JSON contract of the reference (CPU) arm on a tiny sample."""
import json
import subprocess
import sys

import numpy as np

import bench


def test_workloads_have_the_named_shapes():
    bits, im = bench.make_workload()
    assert bits.shape == (4096, 14336) and bits.dtype == np.uint16 and im.shape == (14336,)
    iq = bench.make_iq_workload()
    assert [t[1].shape for t in iq] == [(4096, 4096), (14336, 4096)]


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
