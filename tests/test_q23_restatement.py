"""Q2_K and Q3_K have no encoder in the reference, so the C oracle's
restatement of them (the reference's make_qkx3_quants / make_qx_quants at
16-element sub-blocks, ggml's block layouts) cannot be pinned to reference
output. This test pins it to a second, independent restatement written
here in scalar Python with explicit binary32 rounding of every operation,
on a few super-blocks of each test distribution."""
import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import Q2_K, Q3_K, bf16_bits_to_f32, edge_rows, student_rows, sweep_rows

F = np.float32


def rnd(v):
    """nearest_int (quant.rs:16): f32 round half away from zero, saturating cast."""
    v = float(v)
    if math.isnan(v):
        return 0
    if math.isinf(v):
        return 2**31 - 1 if v > 0 else -2**31
    r = math.floor(abs(v) + 0.5) * (1 if v >= 0 else -1)
    return int(max(min(r, 2**31 - 1), -2**31))


def f16_bytes(v):
    return np.array([v], np.float32).astype(np.float16).view(np.uint8).tolist()


def weights(xs, im, sig):
    return [F(F(1.0) if im is None else im[i]) * F(np.sqrt(F(sig + F(xs[i] * xs[i])))) for i in range(len(xs))]


def qx(xs, nmax, w):
    """make_qx_quants (quant.rs:34-73): returns the chosen scale."""
    amax, mx = F(0), F(0)
    for v in xs:
        if abs(v) > amax:
            amax, mx = F(abs(v)), v
    if amax < F(1e-15):
        return F(0)
    best_scale, best, first = F(0), F(0), True
    for is_ in range(-9, 10):
        iscale = F(F(-F(F(nmax) + F(F(0.1) * F(is_)))) / mx)
        sumlx, suml2 = F(0), F(0)
        for v, wi in zip(xs, w):
            l = max(-nmax, min(nmax - 1, rnd(F(iscale * v))))
            sumlx = F(sumlx + F(F(wi * v) * F(l)))
            suml2 = F(suml2 + F(wi * F(l * l)))
        if suml2 > 0 and (first or F(sumlx * sumlx) > F(best * suml2)):
            best_scale = F(sumlx / suml2)
            best = F(best_scale * sumlx)
            first = False
    return best_scale


def qkx3(xs, nmax, w):
    """make_qkx3_quants (quant.rs:77-141), rmin -0.9, rdelta 0.05, 36 steps: (scale, min)."""
    vals = [v for v in xs if not math.isnan(v)]
    vmin = F(min(min(vals), F(0))) if vals else F(0)
    vmax = F(max(vals)) if vals else F(-np.inf)
    if vmax <= vmin:
        return F(0), vmin
    rng = F(vmax - vmin)
    iscale = F(F(nmax) / rng)
    scale = F(F(1) / iscale)
    err = F(0)
    for v, wi in zip(xs, w):
        l = max(0, min(nmax, rnd(F(iscale * F(v - vmin)))))
        d = F(F(F(scale * F(l)) + vmin) - v)
        err = F(err + F(F(wi * d) * d))
    best_err, best_min = err, vmin
    sw = sx = F(0)
    for is_ in range(37):
        isc = F(F(F(F(-0.9) + F(F(0.05) * F(is_))) + F(nmax)) / rng)
        ls, sl, sl2, sxl = [], F(0), F(0), F(0)
        sw, sx = F(0), F(0)
        for v, wi in zip(xs, w):
            l = max(0, min(nmax, rnd(F(isc * F(v - vmin)))))
            ls.append(l)
            sw = F(sw + wi)
            sx = F(sx + F(wi * v))
            sl = F(sl + F(wi * F(l)))
            sl2 = F(sl2 + F(wi * F(l * l)))
            sxl = F(sxl + F(F(wi * F(l)) * v))
        D = F(F(sw * sl2) - F(sl * sl))
        if D > 0:
            ts = F(F(F(sw * sxl) - F(sx * sl)) / D)
            tm = F(F(F(sl2 * sx) - F(sl * sxl)) / D)
            if tm > 0:
                tm = F(0)
                ts = F(sxl / sl2) if sl2 > 0 else F(0)
            e = F(0)
            for v, wi, l in zip(xs, w, ls):
                d = F(F(F(ts * F(l)) + tm) - v)
                e = F(e + F(F(wi * d) * d))
            if e < best_err:
                best_err, scale, best_min = e, ts, tm
    return scale, best_min


def enc_q3_k(blk, im, sig):
    scales = []
    for sb in range(16):
        xs = blk[16 * sb:16 * sb + 16]
        scales.append(qx(xs, 4, weights(xs, None if im is None else im[16 * sb:16 * sb + 16], sig)))
    amax, ms = F(0), F(0)
    for s in scales:
        if abs(s) > amax:
            amax, ms = F(abs(s)), s
    out = [0] * 110
    if amax < F(1e-15):
        return out
    iscale = F(F(-32) / ms)
    d = F(F(1) / iscale)
    levels = []
    for sb in range(16):
        q = max(-32, min(31, rnd(F(iscale * scales[sb]))))
        u = q + 32
        out[96 + sb % 8] |= (u & 0xF) << (4 * (sb // 8))
        out[104 + sb % 4] |= (u >> 4) << (2 * (sb // 4))
        dd = F(d * F(q))
        for v in blk[16 * sb:16 * sb + 16]:
            levels.append(4 if dd == 0 else max(-4, min(3, rnd(F(v / dd)))) + 4)
    for e, l in enumerate(levels):
        out[32 + (e // 128) * 32 + e % 32] |= (l & 3) << (2 * ((e % 128) // 32))
        if l & 4:
            out[e % 32] |= 1 << (e // 32)
    out[108:110] = f16_bytes(d)
    return out


def enc_q2_k(blk, im, sig):
    scales, mins = [], []
    for sb in range(16):
        xs = blk[16 * sb:16 * sb + 16]
        s, m = qkx3(xs, 3, weights(xs, None if im is None else im[16 * sb:16 * sb + 16], sig))
        scales.append(s)
        mins.append(F(-m))
    max_s = max([F(0)] + [s for s in scales if not math.isnan(s)])
    max_m = max([F(0)] + [m for m in mins if not math.isnan(m)])
    inv_s = F(F(15) / max_s) if max_s > 0 else F(0)
    inv_m = F(F(15) / max_m) if max_m > 0 else F(0)
    d, dmin = F(max_s / F(15)), F(max_m / F(15))
    out = [0] * 84
    levels = []
    for sb in range(16):
        ls = max(0, min(15, rnd(F(inv_s * scales[sb]))))
        lm = max(0, min(15, rnd(F(inv_m * mins[sb]))))
        out[sb] = ls | (lm << 4)
        dsub, msub = F(d * F(ls)), F(dmin * F(lm))
        for v in blk[16 * sb:16 * sb + 16]:
            levels.append(0 if dsub == 0 else max(0, min(3, rnd(F(F(v + msub) / dsub)))))
    for e, l in enumerate(levels):
        out[16 + (e // 128) * 32 + e % 32] |= l << (2 * ((e % 128) // 32))
    out[80:82] = f16_bytes(d)
    out[82:84] = f16_bytes(dmin)
    return out


def rows_under_test():
    bits, im = sweep_rows(2, 512, seed=61)
    yield bf16_bits_to_f32(bits), im
    bits, im = student_rows(2, 512, seed=62)
    yield bf16_bits_to_f32(bits), None
    yield edge_rows(256).astype(np.float32), np.ones(256, np.float32)


@pytest.mark.parametrize("ty,enc,bb", [(Q3_K, enc_q3_k, 110), (Q2_K, enc_q2_k, 84)], ids=["Q3_K", "Q2_K"])
@pytest.mark.filterwarnings("ignore::RuntimeWarning")  # the edge rows overflow some scales, as in f32
def test_oracle_matches_independent_restatement(ty, enc, bb):
    for x, im in rows_under_test():
        for row in x:
            want = O.encode_row(ty, row, im)
            # sigma^2: sequential f32 fold of x^2 over the row, / ne0 (quant.rs:153-155)
            s = F(0)
            for v in row:
                s = F(s + F(v * v))
            sig = F(s / F(len(row)))
            got = []
            for b in range(len(row) // 256):
                got += enc([F(v) for v in row[256 * b:256 * b + 256]], None if im is None else im[256 * b:256 * b + 256], sig)
            assert np.array_equal(np.array(got, np.uint8), want), np.nonzero(np.array(got, np.uint8) != want)
