"""GPU parity: the CUDA encoders, decoders and fused error pass against the
CPU oracle, byte for byte (codes), bit for bit (decoded f32, f64 errors).

All calls go through the C ABI (libshoehorn_cuda.so via shoehorn_b200)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import (BF16, F16, F32, IQ, KQUANT, KQUANT_EXTRA, NAMES, PLAIN, bf16_bits_to_f32, edge_rows,
                           f32_to_bf16_bits, student_rows, sweep_rows)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import shoehorn_b200 as sh  # noqa: E402


def supported(types):
    return [t for t in types if sh.type_supported(t)]


# the reference's K-quants and the two ggml K-quants it lacks (Q2_K, Q3_K)
KQ = KQUANT + KQUANT_EXTRA
ENC_TYPES = supported(KQ + IQ) + PLAIN


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_encode(ctx, ty, bits, im=None, rows_per_mat=0, row0=0):
    src = dev(bits.view(np.int16))
    imt = None if im is None else dev(im)
    out = ctx.encode_rows(ty, src, imt, rows_per_mat=rows_per_mat, row0=row0, sync=True)
    return out.cpu().numpy()


def oracle_encode(ty, bits, im=None, rows_per_mat=0, row0=0):
    if row0 == 0:
        return O.encode_tensor_bf16(ty, bits, im, rows_per_mat=rows_per_mat)
    # shift the imatrix matrix selection by row0 (imatrix.rs:124 with global rows)
    x = bf16_bits_to_f32(bits)
    ne0 = bits.shape[1]
    rows = []
    for r in range(bits.shape[0]):
        g = row0 + r
        ims = None
        if im is not None:
            if im.size == ne0:
                ims = im
            elif rows_per_mat > 0 and im.size % ne0 == 0:
                m = min(g // rows_per_mat, im.size // ne0 - 1)
                ims = im[m * ne0:(m + 1) * ne0]
        rows.append(O.encode_row(ty, x[r], ims))
    return np.stack(rows)


def assert_bytes_equal(got, want, ty):
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        raise AssertionError(f"{NAMES[ty]}: {len(bad)} bytes differ; first at row {r} byte {c}: "
                             f"gpu {got[r, c]} oracle {want[r, c]}")


@pytest.mark.parametrize("ty", ENC_TYPES, ids=lambda t: NAMES[t])
def test_encode_matches_oracle_sweep_rows(ctx, ty):
    bits, im = sweep_rows(48, 2048, seed=100 + ty)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, im), oracle_encode(ty, bits, im), ty)


@pytest.mark.parametrize("ty", supported(KQ + IQ), ids=lambda t: NAMES[t])
def test_encode_matches_oracle_many_rows(ctx, ty):
    """4096 rows x 1024 (16384 super-blocks): enough near-ties between grid
    errors that a single contracted multiply-add in a search shows up."""
    bits, im = sweep_rows(4096, 1024, seed=5)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, im), oracle_encode(ty, bits, im), ty)


@pytest.fixture(scope="module")
def iq_config():
    """The IQ codebook configuration's tensors ([4096 x 4096] and
    [14336 x 4096] Student-t, nu = 5, with the log-normal imatrix)."""
    from shoehorn_b200 import workloads
    return workloads.iq_tensors()


@pytest.mark.parametrize("ty", supported(IQ), ids=lambda t: NAMES[t])
def test_iq_configuration_rows_match_oracle(ctx, iq_config, ty):
    """quant_iq.rs:275-1157 on the IQ configuration as configured (Student-t
    weights AND the imatrix): 1024 rows spread over each of the two tensors,
    32768 super-blocks per type, byte for byte."""
    for name, bits, im in iq_config:
        rows = np.linspace(0, bits.shape[0] - 1, 1024).astype(np.int64)
        sub = np.ascontiguousarray(bits[rows])
        assert_bytes_equal(gpu_encode(ctx, ty, sub, im), oracle_encode(ty, sub, im), ty)


def test_negative_row0_is_rejected(ctx):
    bits, im = sweep_rows(4, 256, seed=1)
    with pytest.raises(sh.ShoehornError):
        gpu_encode(ctx, 12, bits, np.concatenate([im, im]), rows_per_mat=2, row0=-1)


@pytest.mark.parametrize("ty", ENC_TYPES, ids=lambda t: NAMES[t])
def test_encode_matches_oracle_student_rows_no_imatrix(ctx, ty):
    bits, _ = student_rows(32, 4096, seed=200 + ty)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, None), oracle_encode(ty, bits, None), ty)


@pytest.mark.parametrize("ty", ENC_TYPES, ids=lambda t: NAMES[t])
def test_encode_matches_oracle_edge_rows(ctx, ty):
    x = edge_rows(1024)
    bits = f32_to_bf16_bits(x)
    im = np.ones(1024, np.float32)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, im), oracle_encode(ty, bits, im), ty)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, None), oracle_encode(ty, bits, None), ty)


def q8_0_special_rows():
    """Blocks with NaN, +-inf, a subnormal d with finite 1/d, a d whose
    reciprocal overflows, and exact .5 ties after scaling (Q8_0's general
    rounding path and the edges of its fast path)."""
    rng = np.random.default_rng(17)
    x = rng.normal(0, 0.02, (4, 1024)).astype(np.float32)
    x[0, 3] = np.nan
    x[0, 40] = np.inf
    x[0, 70] = -np.inf
    x[0, 96:128] = np.nan
    x[1, 0:32] = rng.uniform(-1, 1, 32).astype(np.float32) * np.float32(5.3e-37)   # d in [2^-128, 2^-126)
    x[1, 32:64] = rng.uniform(-1, 1, 32).astype(np.float32) * np.float32(1e-38)    # 1/d overflows
    x[1, 64:96] = np.float32(3e-39)
    x[2, 0:32] = (np.arange(32) - 16).astype(np.float32) * np.float32(127.0 / 16.0) / np.float32(254.0)
    x[2, 32:64] = np.float32(-0.0)
    x[3, :] = np.float32(-1.5)
    return f32_to_bf16_bits(x)


@pytest.mark.parametrize("ty", [2, 6, 3, 7], ids=lambda t: NAMES[t])
def test_legacy_blocks_without_an_accepted_grid_keep_earlier_levels(ctx, ty):
    """quant.rs:171-198: make_qx_quants writes no levels when no grid is
    accepted (zero or NaN weighted level energy for all 19 grids), and the
    row's level buffer keeps the nearest earlier block's levels, or zeros.
    Zero imatrix windows over whole blocks, a NaN (its row's sigma^2 and so
    every weight turns NaN) and a sub-epsilon block (which writes nmax)."""
    bits, im = sweep_rows(6, 1024, seed=77)
    im = im.copy()
    im[0:32] = 0.0        # block 0: nothing accepted, nothing earlier -> zeros
    im[64:128] = 0.0      # blocks 2, 3 carry block 1's levels
    im[500:540] = 0.0     # partial windows: still accepted
    x = bf16_bits_to_f32(bits)
    x[3, 200] = np.nan    # row 3: every block rejects -> zeros... or an earlier block
    x[4, 0:32] = 0.0      # row 4: block 0 is below GROUP_MAX_EPS and writes nmax,
    x[4, 40] = np.nan     #        every later block carries those levels
    bits = f32_to_bf16_bits(x)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, im), oracle_encode(ty, bits, im), ty)
    assert_bytes_equal(gpu_encode(ctx, ty, bits, None), oracle_encode(ty, bits, None), ty)


def test_q8_0_special_values(ctx):
    bits = q8_0_special_rows()
    assert_bytes_equal(gpu_encode(ctx, 8, bits), oracle_encode(8, bits), 8)


@pytest.mark.parametrize("ty", supported(KQ + IQ), ids=lambda t: NAMES[t])
def test_expert_imatrix_slicing_and_row0(ctx, ty):
    """imatrix.rs:124-141: an imatrix of n_mats*ne0 selects matrix row/rows_per_mat."""
    bits, _ = sweep_rows(24, 512, seed=300 + ty)
    rng = np.random.default_rng(ty)
    im3 = np.exp(rng.normal(0, 1, 3 * 512)).astype(np.float32)
    got = gpu_encode(ctx, ty, bits, im3, rows_per_mat=8, row0=5)
    want = oracle_encode(ty, bits, im3, rows_per_mat=8, row0=5)
    assert_bytes_equal(got, want, ty)
    # an imatrix whose length is not a multiple of ne0 means "no imatrix"
    got = gpu_encode(ctx, ty, bits, im3[:700], rows_per_mat=8)
    assert_bytes_equal(got, oracle_encode(ty, bits, None), ty)


@pytest.mark.parametrize("src_dtype", ["f32", "f16"])
def test_f32_and_f16_sources(ctx, src_dtype):
    bits, im = sweep_rows(16, 1024, seed=7)
    x = bf16_bits_to_f32(bits)
    if src_dtype == "f16":
        x = x.astype(np.float16).astype(np.float32)
    src = dev(x if src_dtype == "f32" else x.astype(np.float16))
    for ty in supported(KQ + IQ):
        got = ctx.encode_rows(ty, src, dev(im), sync=True).cpu().numpy()
        want = np.stack([O.encode_row(ty, r, im) for r in x])
        assert_bytes_equal(got, want, ty)


@pytest.mark.parametrize("ty", supported(KQ + IQ) + [F16, BF16, F32], ids=lambda t: NAMES[t])
def test_decode_matches_oracle(ctx, ty):
    bits, im = student_rows(8, 1024, seed=400 + ty)
    x = bf16_bits_to_f32(bits)
    codes = np.stack([O.encode_row(ty, r, im) for r in x])
    got = ctx.decode_rows(ty, dev(codes), 1024, sync=True).cpu().numpy()
    want = np.stack([O.decode_row(ty, c, 1024) for c in codes])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("row_step", [1, 3])
def test_row_errors_match_oracle(ctx, row_step):
    bits, im = sweep_rows(20, 1024, seed=500)
    types = supported(KQ + IQ) + [F16]
    got = ctx.row_errors(types, dev(bits.view(np.int16)), dev(im), row_step=row_step).cpu().numpy()
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, im, row_step=row_step)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


# The error table is one fused launch per candidate: rows are handed out in
# groups (1 to 32 rows, one fold lane per row), a group's 256-element units in
# column order over its rows, groups grid-strided over the resident CTAs.
# These shapes give groups of one row (few rows, long rows), groups with a
# short last group, many groups per CTA, and a sampled view of a 3-D tensor
# whose imatrix slice changes with the matrix.
@pytest.mark.parametrize("n_rows,ne0,row_step,rows_per_mat", [
    (1, 4096, 1, 0), (3, 2048, 1, 0), (45, 512, 1, 0), (2400, 256, 1, 0), (9000, 256, 1, 0), (600, 512, 7, 100)])
def test_row_errors_fused_groups(ctx, n_rows, ne0, row_step, rows_per_mat):
    bits, im1 = sweep_rows(n_rows, ne0, seed=n_rows + ne0)
    im = im1
    if rows_per_mat:
        n_mats = (n_rows + rows_per_mat - 1) // rows_per_mat
        im = np.exp(np.random.default_rng(3).normal(0, 1.0, size=n_mats * ne0)).astype(np.float32)
    types = supported(KQ + IQ) + [F16, BF16, F32]
    got = ctx.row_errors(types, dev(bits.view(np.int16)), dev(im), row_step=row_step,
                         rows_per_mat=rows_per_mat).cpu().numpy()
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, im, row_step=row_step, rows_per_mat=rows_per_mat)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


# Rows whose last 256-element unit is short (32-element block types only).
@pytest.mark.parametrize("n_rows,ne0", [(1, 96), (9, 800), (300, 288)])
def test_row_errors_fused_short_units(ctx, n_rows, ne0):
    bits, im = sweep_rows(n_rows, ne0, seed=ne0)
    types = [t for t in supported(KQ + IQ) if sh.GgmlType(t).block_layout()[0] == 32]
    assert len(types) >= 6
    got = ctx.row_errors(types, dev(bits.view(np.int16)), dev(im)).cpu().numpy()
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, im)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


@pytest.mark.parametrize("n_rows,ne0", [(3, 8), (40, 200), (130, 1032)])
def test_row_errors_fused_elementwise(ctx, n_rows, ne0):
    """F32/F16/BF16 candidates: the round trip in place of an encoder, rows of
    any multiple-of-8 width (the last 256-element unit short)."""
    bits, im = sweep_rows(n_rows, ne0, seed=ne0 + 1)
    types = [F32, F16, BF16]
    for imv in (im, None):
        got = ctx.row_errors(types, dev(bits.view(np.int16)), None if imv is None else dev(imv)).cpu().numpy()
        for t, ty in enumerate(types):
            want = O.row_errors_bf16(ty, bits, imv)
            assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


def test_row_errors_fused_legacy_carried_levels(ctx):
    """The fused table on legacy blocks that re-emit an earlier block's levels
    (quant.rs:171-198) and on NaN rows."""
    bits, im = sweep_rows(40, 1024, seed=78)
    im = im.copy()
    im[64:128] = 0.0
    x = bf16_bits_to_f32(bits)
    x[3, 200] = np.nan
    bits = f32_to_bf16_bits(x)
    types = [2, 6, 3, 7]
    for imv in (im, None):
        got = ctx.row_errors(types, dev(bits.view(np.int16)), None if imv is None else dev(imv)).cpu().numpy()
        for t, ty in enumerate(types):
            want = O.row_errors_bf16(ty, bits, imv)
            assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


def test_row_errors_fused_iq_configuration(ctx):
    """The IQ configuration's distribution (Student-t, log-normal imatrix)."""
    bits, im = student_rows(160, 4096, seed=77)
    types = supported(IQ) + supported(KQ)
    got = ctx.row_errors(types, dev(bits.view(np.int16)), dev(im), row_step=1).cpu().numpy()
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, im)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


def test_row_errors_without_imatrix_and_edges(ctx):
    x = edge_rows(512)
    bits = f32_to_bf16_bits(x)
    types = supported(KQ + IQ) + [F16, BF16]
    got = ctx.row_errors(types, dev(bits.view(np.int16)), None).cpu().numpy()
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, None)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


def test_row_api_mirrors_reference(ctx):
    x = bf16_bits_to_f32(sweep_rows(1, 512, seed=9)[0])[0]
    for ty in supported(KQ):
        enc = sh.encode_row(ty, x)
        assert np.array_equal(enc, O.encode_row(ty, x))
        assert np.array_equal(sh.decode_row(ty, enc, 512).view(np.uint32), O.decode_row(ty, enc, 512).view(np.uint32))
        assert sh.row_error(ty, x) == O.row_error(ty, x)
    with pytest.raises(ValueError):
        sh.encode_row(sh.GgmlType.Q4_K, np.zeros(100, np.float32))  # ragged row, like the reference's assert


@pytest.mark.parametrize("pinned", [False, True])
def test_host_entry_point_matches_device(ctx, pinned):
    bits, im = sweep_rows(300, 1024, seed=21)
    for ty in supported(KQ + IQ):
        want = oracle_encode(ty, bits, im)
        if pinned:
            src = torch.from_numpy(bits.view(np.int16)).pin_memory()
            out = torch.empty(want.shape, dtype=torch.uint8).pin_memory()
            ctx.encode_tensor_host(ty, src, im, out=out)
            got = out.numpy()
        else:
            got = ctx.encode_tensor_host(ty, bits, im)
        assert_bytes_equal(got, want, ty)


def test_host_row_errors_match_oracle(ctx):
    bits, im = sweep_rows(37, 1024, seed=31)
    types = supported(KQ + IQ) + [F16]
    got = ctx.row_errors_host(types, bits, im, row_step=4)
    for t, ty in enumerate(types):
        want = O.row_errors_bf16(ty, bits, im, row_step=4)
        assert np.array_equal(got[t].view(np.uint64), want.view(np.uint64)), NAMES[ty]


def test_sync_reports_clean_status(ctx):
    ctx.sync()
    assert ctx.launch_count() > 0


# ---- full encoder-sweep size (4096 x 14336): sampled rows vs the oracle, plus
# size-independent properties over every row ----
@pytest.fixture(scope="module")
def big_tensor():
    bits, im = sweep_rows(4096, 14336, seed=20261201)
    return bits, im


@pytest.mark.parametrize("ty", supported(KQ + IQ), ids=lambda t: NAMES[t])
def test_full_size_encode(ctx, big_tensor, ty):
    bits, im = big_tensor
    src = dev(bits.view(np.int16))
    imt = dev(im)
    a = ctx.encode_rows(ty, src, imt, sync=True)
    b = ctx.encode_rows(ty, src, imt, sync=True)
    assert torch.equal(a, b)  # deterministic
    codes = a.cpu().numpy()
    rng = np.random.default_rng(ty)
    rows = np.sort(rng.choice(np.arange(1, 4095), size=62, replace=False))
    rows = np.concatenate([[0], rows, [4095]])  # 64 rows, first and last included
    want = O.encode_tensor_bf16(ty, bits[rows], im)
    assert_bytes_equal(codes[rows], want, ty)
    # decode of every row stays within the reference's round-trip tolerance band
    dec = ctx.decode_rows(ty, a, 14336, sync=True)
    x = src.view(torch.bfloat16).float()
    rel = ((dec - x).pow(2).mean() / x.pow(2).mean()).sqrt().item()
    assert np.isfinite(rel) and rel < 0.8
