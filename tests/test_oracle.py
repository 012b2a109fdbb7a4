"""CPU oracle checks: the reference's own tests (ported) plus independent pins
from gguf-py (decode layouts, Q8_0 bytes, IEEE f16 rounding).

The oracle is the checker for the CUDA kernels, so it is pinned first."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import (BF16, F16, IQ2_S, IQ2_XS, IQ2_XXS, IQ3_S, IQ3_XXS, IQ4_NL, IQ4_XS, NAMES, Q2_K, Q3_K,
                           Q4_0, Q4_1, Q4_K, Q5_0, Q5_1, Q5_K, Q6_K, Q8_0, edge_rows, lcg_vec, student_rows, sweep_rows,
                           bf16_bits_to_f32)

gguf = pytest.importorskip("gguf")
GQT = gguf.GGMLQuantizationType


# ---- quant.rs:659-671 roundtrips ----
@pytest.mark.parametrize("ty,tol", [(F16, 1e-3), (BF16, 1e-2), (Q8_0, 0.02), (Q6_K, 0.05), (Q5_K, 0.08),
                                    (Q5_0, 0.1), (Q5_1, 0.1), (Q4_K, 0.15), (Q4_0, 0.25), (Q4_1, 0.2)])
def test_roundtrips(ty, tol):
    x = lcg_vec(512)
    enc = O.encode_row(ty, x)
    assert enc.size == O.row_bytes(ty, 512)
    dec = O.decode_row(ty, enc, 512)
    assert dec.size == 512
    d = (x - dec).astype(np.float32)
    rmse = np.sqrt(np.float32(np.sum(d * d, dtype=np.float32)) / np.float32(512))
    assert rmse < tol, f"{NAMES[ty]} rmse {rmse}"


# ---- Q2_K / Q3_K: no reference counterpart; the reference's search routines
# in ggml's block layouts (decoder layouts pinned through gguf-py below) ----
@pytest.mark.parametrize("ty,bpb,tol", [(Q3_K, 110, 0.2), (Q2_K, 84, 0.35)])
def test_extra_kquant_roundtrips(ty, bpb, tol):
    x = lcg_vec(512)
    enc = O.encode_row(ty, x)
    assert enc.size == 2 * bpb == O.row_bytes(ty, 512)
    d = (x - O.decode_row(ty, enc, 512)).astype(np.float32)
    assert np.sqrt(np.sum(d * d, dtype=np.float32) / np.float32(512)) < tol


def test_extra_kquant_error_ladder():
    """More bits, less weighted error: Q2_K > Q3_K > Q4_K on the same rows."""
    bits, im = student_rows(8, 1024, seed=5)
    x = bf16_bits_to_f32(bits)
    for r in range(8):
        e2, e3, e4 = (O.row_error(t, x[r], im) for t in (Q2_K, Q3_K, Q4_K))
        assert e2 > e3 > e4 > 0.0


def test_extra_kquant_zero_and_scale_codes():
    z = np.zeros(256, np.float32)
    assert not O.encode_row(Q3_K, z).any()  # zero block: every byte 0
    e2 = O.encode_row(Q2_K, z)
    assert not e2.any()
    # one large positive element per 16-element sub-block: the largest scale
    # code is 15 (Q2_K) and the largest |signed scale code| is 32 (Q3_K)
    x = lcg_vec(256) * np.float32(0.01)
    x[::16] = np.float32(3.0)
    e2 = O.encode_row(Q2_K, x)
    assert max(b & 0xF for b in e2[:16]) == 15
    e3 = O.encode_row(Q3_K, x).astype(np.int64)
    u = [((e3[96 + sb % 8] >> (4 * (sb // 8))) & 0xF) | (((e3[104 + sb % 4] >> (2 * (sb // 4))) & 3) << 4)
         for sb in range(16)]
    assert max(abs(c - 32) for c in u) == 32


# ---- quant.rs:673-695 imatrix weighting ----
def test_imatrix_weighting_prioritizes_important_columns():
    x = lcg_vec(256)
    im = np.ones(256, np.float32)
    im[:32] = 100.0
    err_weighted = O.row_error(Q4_K, x, im)
    err_uniform = O.row_error(Q4_K, x, None)
    dec = O.decode_row(Q4_K, O.encode_row(Q4_K, x, None), 256)
    d = (x - dec).astype(np.float32).astype(np.float64)
    err_uniform_enc_weighted_metric = float(np.sum(im.astype(np.float64) * d * d))
    assert err_weighted <= err_uniform_enc_weighted_metric * 1.05
    assert err_uniform > 0.0


# ---- quant_iq.rs:1219-1227 iq_roundtrips ----
@pytest.mark.parametrize("ty,bpb,tol", [(IQ4_XS, 136, 0.08), (IQ3_S, 110, 0.25), (IQ3_XXS, 98, 0.35),
                                        (IQ2_S, 82, 0.62), (IQ2_XS, 74, 0.65), (IQ2_XXS, 66, 0.75)])
def test_iq_roundtrips(ty, bpb, tol):
    x = lcg_vec(512, 0x12345678)
    im = np.ones(512, np.float32)
    e = O.encode_row(ty, x, im)
    assert e.size == 2 * bpb
    d = O.decode_row(ty, e, 512)
    diff = (x - d).astype(np.float32)
    rmse = np.sqrt(np.sum(diff * diff, dtype=np.float32) / np.float32(512))
    xrms = np.sqrt(np.sum(x * x, dtype=np.float32) / np.float32(512))
    assert rmse / xrms < tol


# ---- quant_iq.rs:1229-1241 ----
def test_iq4_nl_roundtrip():
    x = lcg_vec(64, 0xDEADBEEF)
    e = O.encode_row(IQ4_NL, x, np.ones(64, np.float32))
    assert e.size == 36
    d = O.decode_row(IQ4_NL, e, 64)
    diff = (x - d).astype(np.float32)
    assert np.sqrt(np.sum(diff * diff, dtype=np.float32) / np.float32(64)) < 0.1


# ---- quant_iq.rs:1243-1254 grids_build ----
def test_grids_build():
    sizes = [O.grid_info(w)[0] for w in range(5)]
    assert sizes == [256, 512, 1024, 256, 512]
    _, kmap, _ = O.grid_info(0)
    assert int((kmap >= 0).sum()) == 256


# ---- scalar semantics ----
def test_f16_round_to_nearest_even_matches_numpy():
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.normal(0, 1, 20000).astype(np.float32),
        (rng.normal(0, 1, 5000) * 1e-5).astype(np.float32),     # f16 subnormal range
        (rng.normal(0, 1, 2000) * 7e4).astype(np.float32),      # overflow region
        np.array([0.0, -0.0, 65504.0, 65520.0, 65519.99, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                  2.9802326e-08, np.inf, -np.inf], np.float32),
    ])
    # exact ties between f16 neighbours
    h = rng.integers(0, 0x7BFF, 3000).astype(np.uint16)
    lo = h.view(np.float16).astype(np.float32)
    hi = (h + 1).view(np.float16).astype(np.float32)
    vals = np.concatenate([vals, ((lo.astype(np.float64) + hi) / 2).astype(np.float32)])
    ours = np.array([O.f32_to_f16_bits(v) for v in vals], dtype=np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_nearest_int_is_half_away_and_saturating():
    assert [O.nearest_int(v) for v in (0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 0.49999997)] == [1, 2, 3, -1, -2, -3, 0]
    assert O.nearest_int(float("nan")) == 0
    assert O.nearest_int(3e9) == 2**31 - 1
    assert O.nearest_int(-3e9) == -(2**31)


# ---- independent layout pins through gguf-py ----
_GQ = {Q8_0: GQT.Q8_0, Q2_K: GQT.Q2_K, Q3_K: GQT.Q3_K, Q4_0: GQT.Q4_0, Q4_1: GQT.Q4_1, Q5_0: GQT.Q5_0, Q5_1: GQT.Q5_1, Q4_K: GQT.Q4_K,
       Q5_K: GQT.Q5_K, Q6_K: GQT.Q6_K, IQ2_XXS: GQT.IQ2_XXS, IQ2_XS: GQT.IQ2_XS, IQ2_S: GQT.IQ2_S,
       IQ3_XXS: GQT.IQ3_XXS, IQ3_S: GQT.IQ3_S, IQ4_NL: GQT.IQ4_NL, IQ4_XS: GQT.IQ4_XS}


@pytest.mark.parametrize("ty", sorted(_GQ))
def test_oracle_decoder_matches_gguf_py(ty):
    bits, im = student_rows(4, 1024, seed=7)
    x = bf16_bits_to_f32(bits)
    for r in range(4):
        enc = O.encode_row(ty, x[r], im)
        ours = O.decode_row(ty, enc, 1024)
        theirs = gguf.quants.dequantize(enc.reshape(1, -1), _GQ[ty]).reshape(-1).astype(np.float32)
        # gguf-py keeps ggml's operand order, so the values are the same bits
        assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32)), NAMES[ty]


def test_q8_0_bytes_match_gguf_py_quantizer():
    bits, _ = sweep_rows(64, 2048, seed=3)
    x = bf16_bits_to_f32(bits)
    ours = np.stack([O.encode_row(Q8_0, r) for r in x])
    theirs = gguf.quants.quantize(x, GQT.Q8_0)
    assert np.array_equal(ours, theirs.reshape(ours.shape))


@pytest.mark.parametrize("ty", [Q8_0, Q6_K, Q4_K, Q5_K, Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL, IQ4_XS, IQ3_S, IQ3_XXS,
                                IQ2_S, IQ2_XS, IQ2_XXS, Q2_K, Q3_K])
def test_edge_rows_encode_and_decode(ty):
    rows = edge_rows(512)
    for r in rows:
        enc = O.encode_row(ty, r, np.ones(512, np.float32))
        dec = O.decode_row(ty, enc, 512)
        assert np.all(np.isfinite(dec))


def test_tensor_driver_matches_row_api():
    bits, im = sweep_rows(40, 512, seed=11)
    x = bf16_bits_to_f32(bits)
    for ty in (Q4_K, Q6_K, IQ4_XS):
        t = O.encode_tensor_bf16(ty, bits, im, n_threads=4)
        rows = np.stack([O.encode_row(ty, r, im) for r in x])
        assert np.array_equal(t, rows)
        e = O.row_errors_bf16(ty, bits, im, row_step=3, n_threads=4)
        assert np.array_equal(e, np.array([O.row_error(ty, x[r], im) for r in range(0, 40, 3)]))
