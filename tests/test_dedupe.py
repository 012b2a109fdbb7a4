"""The grid-skipping rule of the make_qkx3_quants kernels (Q4_K, Q5_K, Q2_K),
checked on the CPU: for x - vmin >= 0 a grid's level vector can differ from
the previous grid's only where some element crosses a rounding threshold,
and every such grid lies in the one or two grids the kernels mark from the
estimate j ~ 20 (thr (vmax - vmin)/u - (nmax - 0.9)) with a 0.004 window.
The kernels evaluate only marked grids (plus grid 0 and the initial grid),
so this is the property their byte parity rests on; the GPU parity tests
check the bytes themselves."""
import numpy as np
import pytest

from tests.helpers import bf16_bits_to_f32, edge_rows, student_rows, sweep_rows

f32 = np.float32


def level_changes_and_marks(x, nmax):
    """x: (n_sub, n) f32 sub-blocks. Returns boolean (n_sub, 37) arrays of the
    grids whose levels differ from the previous grid's, and of marked grids."""
    vmin = np.minimum(x.min(1), f32(0))
    vmax = x.max(1)
    keep = vmax > vmin
    x, vmin, vmax = x[keep], vmin[keep], vmax[keep]
    rng = (vmax - vmin).astype(f32)
    u = (x - vmin[:, None]).astype(f32)
    fn = f32(nmax)
    j = np.arange(37, dtype=f32)
    # iscale_j = (rmin + rdelta*j + nmax) / (vmax - vmin), rounded as the reference does
    with np.errstate(over="ignore", divide="ignore"):
        isc = (((f32(-0.9) + (f32(0.05) * j).astype(f32)).astype(f32) + fn).astype(f32)[None, :] /
               rng[:, None]).astype(f32)
    # sub-blocks with a non-finite range or scale evaluate every grid
    clean = np.isfinite(rng) & np.isfinite(isc[:, 36])
    isc, u, rng = isc[clean], u[clean], rng[clean]
    y = (isc[:, :, None] * u[:, None, :]).astype(f32)              # (n_sub, 37, n)
    lev = np.minimum(np.floor(y.astype(np.float64) + 0.5), nmax)    # round half up of y >= 0, clamped
    changed = np.zeros(lev.shape[:2], bool)
    changed[:, 1:] = (lev[:, 1:] != lev[:, :-1]).any(2)
    marks = np.zeros_like(changed)
    marks[:, 0] = True
    l0, l36 = lev[:, 0, :], lev[:, 36, :]
    with np.errstate(divide="ignore", invalid="ignore"):
        ru = (rng[:, None] / u).astype(f32)
    for c in (1, 2):
        thr = (l0 + (c - 0.5)).astype(f32)
        active = thr < l36
        z = (f32(20.0) * ((thr * ru).astype(f32) - (fn - f32(0.9))).astype(f32)).astype(f32)
        for eps in (-0.004, 0.004):
            jj = np.ceil(np.clip(np.where(active, z + f32(eps), 0.5), 0.5, 36.0)).astype(int)
            rows, cols = np.nonzero(active)
            marks[rows, jj[rows, cols]] = True
    assert (l36 - l0).max() <= 2  # at most two crossings per element
    return changed, marks


@pytest.mark.parametrize("n,nmax", [(32, 15), (32, 31), (16, 3)], ids=["Q4_K", "Q5_K", "Q2_K"])
def test_marked_grids_cover_every_level_change(n, nmax):
    subs = []
    bits, _ = sweep_rows(8, 14336, seed=21)
    subs.append(bf16_bits_to_f32(bits).reshape(-1, n))
    bits, _ = student_rows(16, 4096, seed=22)
    subs.append(bf16_bits_to_f32(bits).reshape(-1, n))
    subs.append(edge_rows(512).astype(np.float32).reshape(-1, n))
    x = np.concatenate(subs)
    changed, marks = level_changes_and_marks(x, nmax)
    missed = changed & ~marks
    assert not missed.any(), f"{missed.sum()} level changes outside the marked grids"
    # the marks stay a small superset: most grids are still skipped
    assert marks.sum(1).mean() < 0.7 * 37


# ---- IQ4_NL / IQ4_XS: the 15 scale trials of quant_iq.rs:1078-1095 ----
KV = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], f32)
_CNT = np.array([sum(1 for k in range(1, 15) if KV[k] <= f - 128) for f in range(256)])


def iq4_index(y):
    """best_index_int8 (quant_iq.rs:1002-1024) as the kernel's final pass
    evaluates it: clamp to [-128, 127] (NaN to the top), neighbouring pair
    from floor(x), rounded distances compared."""
    xc = np.maximum(np.minimum(y, f32(127)), f32(-128)).astype(f32)
    xc = np.where(np.isnan(y), f32(127), xc)
    mu = 1 + _CNT[np.floor(xc.astype(np.float64)).astype(int) + 128]
    lower = (xc - KV[mu - 1]).astype(f32) < (KV[mu] - xc).astype(f32)
    return np.where(lower, mu - 1, mu)


# The trial loop's form (iq.cu best_value_iq4_bounded / best_index_iq4_bounded):
# no float clamp, a table over floor(y) in [-136, 135], the slot read from the
# bits of RD(y + 1.5 * 2^23) and clamped as an unsigned integer at 271.
_CNT272 = np.array([sum(1 for k in range(1, 15) if KV[k] <= f - 136) for f in range(272)])


def iq4_slot_bounded(y):
    """Slot of the clamp-free lookup for f32 y (finite in [-136, 136), or NaN
    as the device add produces it: the canonical 0x7FFFFFFF)."""
    y = np.asarray(y, f32)
    fin = np.isfinite(y)
    bits = np.where(fin, np.uint32(0x4B400000) + np.floor(np.where(fin, y, 0).astype(np.float64)).astype(np.int64)
                    .astype(np.uint32), np.uint32(0x7FFFFFFF)).astype(np.uint32)
    return np.minimum(bits - np.uint32(0x4B400000 - 136), np.uint32(271)).astype(np.int64)


def iq4_index_bounded(y):
    y = np.asarray(y, f32)
    mu = 1 + _CNT272[iq4_slot_bounded(y)]
    with np.errstate(invalid="ignore"):
        lower = (y - KV[mu - 1]).astype(f32) < (KV[mu] - y).astype(f32)
    return np.where(lower, mu - 1, mu)


def test_iq4_clamp_free_lookup_matches_the_clamped_search():
    """Trial products are bounded by 134 (1 + 2^-22) in magnitude (|id| <=
    134/|max|, |x| <= |max|), or NaN: over that domain the clamp-free lookup
    picks the codebook index the clamped binary-search form picks."""
    mids = (KV[:-1] + KV[1:]) / 2
    near = [mids[:, None] + np.arange(-64, 65)[None, :] * np.spacing(np.abs(mids))[:, None]]
    grid = np.arange(-136.0, 136.0, 1 / 64)
    rng = np.random.default_rng(31)
    y = np.concatenate([np.concatenate(near).ravel(), grid, KV, KV - np.spacing(np.abs(KV)), KV + np.spacing(np.abs(KV)),
                        rng.uniform(-136, 136, 200_000), rng.standard_normal(100_000) * 20,
                        np.array([-135.99998, 135.99998, -0.0, 0.0, 1e-30, -1e-30, np.nan])]).astype(f32)
    y = y[(np.abs(y) < 136) | np.isnan(y)]
    np.testing.assert_array_equal(iq4_index_bounded(y), iq4_index(y))
    # every NaN bit pattern, either sign, lands above the table and is clamped
    # onto the last pair, where the false comparison picks v15 as the clamped
    # form (NaN sent to 127) does
    for b in (0x7F800001, 0x7FC00000, 0x7FFFFFFF, 0xFF800001, 0xFFC00000, 0xFFFFFFFF):
        assert (b - (0x4B400000 - 136)) % 2**32 > 271


def iq4_changes_and_marks(x):
    ax = np.abs(x)
    mx = x[np.arange(len(x)), ax.argmax(1)]
    keep = ax.max(1) >= 1e-15
    x, mx = x[keep], mx[keep]
    ids = np.stack([((f32(j - 8) + f32(-127)) / mx).astype(f32) for j in range(1, 16)], 1)
    idx = iq4_index((ids[:, :, None] * x[:, None, :]).astype(f32))     # trials 1..15
    changed = np.zeros((len(x), 16), bool)
    changed[:, 2:] = (idx[:, 1:] != idx[:, :-1]).any(2)
    marks = np.zeros_like(changed)
    marks[:, :2] = True
    lo, hi = np.minimum(idx[:, 0], idx[:, 14]), np.maximum(idx[:, 0], idx[:, 14])
    assert (hi - lo).max() <= 2
    with np.errstate(divide="ignore", invalid="ignore"):
        r = (mx[:, None] / x).astype(f32)
    for c in (0, 1):
        k = lo + c
        active = k < hi
        t = ((KV[np.clip(k, 0, 14)] + KV[np.clip(k + 1, 0, 15)]) * f32(0.5)).astype(f32)
        js = (f32(135) + (t * r).astype(f32)).astype(f32)
        for eps in (-0.01, 0.01):
            jj = np.ceil(np.clip(np.where(active, js + f32(eps), 2.0), 2.0, 15.0)).astype(int)
            rows, cols = np.nonzero(active)
            marks[rows, jj[rows, cols]] = True
    return changed, marks


def test_iq4_marked_trials_cover_every_code_change():
    x = np.concatenate([bf16_bits_to_f32(student_rows(32, 4096, seed=23)[0]).reshape(-1, 32),
                        bf16_bits_to_f32(sweep_rows(8, 14336, seed=24)[0]).reshape(-1, 32),
                        edge_rows(512).astype(np.float32).reshape(-1, 32)])
    changed, marks = iq4_changes_and_marks(x)
    assert not (changed & ~marks).any()
    assert marks.sum(1).mean() < 0.6 * 16


# ---- make_qx_quants (Q6_K nmax 32, Q3_K nmax 4): 19 grids is = -9..9 ----
def qx_changes_and_marks(x, nmax):
    ax = np.abs(x)
    mx = x[np.arange(len(x)), ax.argmax(1)]
    keep = (ax.max(1) >= 1e-15) & np.isfinite(x).all(1)
    x, mx = x[keep], mx[keep]
    fn = f32(nmax)
    t = np.arange(19)
    a = ((fn + (f32(0.1) * (t - 9).astype(f32)).astype(f32)).astype(f32))
    tab = np.abs((-a[None, :] / mx[:, None]).astype(f32))                # |iscale_t|
    axv = np.abs(x)
    y = (tab[:, :, None] * axv[:, None, :]).astype(f32)                   # |iscale_t x|
    positive = (x != 0) & (np.signbit(x) != np.signbit(mx)[:, None])      # iscale*x > 0
    cap = np.where(positive, nmax - 1, nmax)
    lev = np.minimum(np.floor(y.astype(np.float64) + 0.5), cap[:, None, :])
    changed = np.zeros((len(x), 19), bool)
    changed[:, 1:] = (lev[:, 1:] != lev[:, :-1]).any(2)
    marks = np.zeros_like(changed)
    marks[:, 0] = True
    m0, m18 = lev[:, 0], lev[:, 18]
    assert (m18 - m0).max() <= 2
    with np.errstate(divide="ignore", invalid="ignore"):
        ru = (np.abs(mx)[:, None] / axv).astype(f32)
    for c in (1, 2):
        thr = (m0 + (c - 0.5)).astype(f32)
        active = thr < m18
        z = ((f32(10) * ((thr * ru).astype(f32) - fn).astype(f32)).astype(f32) + f32(9)).astype(f32)
        for eps in (-0.01, 0.01):
            jj = np.ceil(np.clip(np.where(active, z + f32(eps), 0.5), 0.5, 18.0)).astype(int)
            rows, cols = np.nonzero(active)
            marks[rows, jj[rows, cols]] = True
    return changed, marks


@pytest.mark.parametrize("nmax", [32, 4], ids=["Q6_K", "Q3_K"])
def test_qx_marked_grids_cover_every_level_change(nmax):
    x = np.concatenate([bf16_bits_to_f32(sweep_rows(8, 14336, seed=25)[0]).reshape(-1, 16),
                        bf16_bits_to_f32(student_rows(16, 4096, seed=26)[0]).reshape(-1, 16),
                        edge_rows(512).astype(np.float32).reshape(-1, 16)])
    changed, marks = qx_changes_and_marks(x, nmax)
    assert not (changed & ~marks).any()
    assert marks.sum(1).mean() < 0.6 * 19
