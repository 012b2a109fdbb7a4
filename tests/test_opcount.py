"""The op-counting build of the oracle (oracle/opcount): same bytes as the
plain oracle, and per-element counts consistent with the figures the
benchmark's roofline uses."""
import numpy as np
import pytest

import bench
from oracle import oracle as O
from oracle.opcount import count_flops as C
from tests.helpers import IQ, KQUANT, KQUANT_EXTRA, NAMES, bf16_bits_to_f32, edge_rows, student_rows, sweep_rows

ALL = KQUANT + KQUANT_EXTRA + IQ


@pytest.mark.parametrize("ty", ALL, ids=lambda t: NAMES[t])
def test_counting_build_matches_oracle_bytes(ty):
    bits, im = sweep_rows(6, 512, seed=40 + ty)
    x = bf16_bits_to_f32(bits)
    codes, counts = C.encode_counted(ty, x, im, O.row_bytes(ty, 512))
    assert np.array_equal(codes, O.encode_tensor_bf16(ty, bits, im))
    assert C.f32_ops(counts) > 0
    e = edge_rows(512)
    codes, _ = C.encode_counted(ty, e, None, O.row_bytes(ty, 512))
    assert np.array_equal(codes, np.stack([O.encode_row(ty, r, None) for r in e]))


@pytest.mark.parametrize("name", list(bench.FLOPS_PER_ELT), ids=str)
def test_bench_flop_table_matches_counter(name):
    ty = bench.TYPE_IDS[name]
    if name in bench.SWEEP or name in ("Q2_K", "Q3_K"):
        bits, im = sweep_rows(8, 14336, seed=7)
    else:
        bits, im = student_rows(8, 4096, seed=7)
    x = bf16_bits_to_f32(bits)
    _, counts = C.encode_counted(ty, x, im, O.row_bytes(ty, x.shape[1]))
    per_elt = C.f32_ops(counts) / x.size
    assert abs(per_elt - bench.FLOPS_PER_ELT[name]) <= 0.1 * bench.FLOPS_PER_ELT[name], (name, per_elt)
