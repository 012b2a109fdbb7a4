"""The IQ tables: generated header vs gguf-py's independent copy of the
decode grids, the encoder lattice tables vs the decode grids, and the
library's compacted search structures vs the oracle's full ones."""
import os
import re

import numpy as np
import pytest

from oracle import oracle as O

gguf = pytest.importorskip("gguf")
HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "shoehorn_b200", "csrc", "iq_tables.h")


def table(name):
    s = open(HDR).read()
    m = re.search(r"#define SH_%s_DATA \{(.*?)\n\}" % name, s, re.S)
    vals = [v.strip().rstrip("ULL") for v in m.group(1).replace("\\", " ").split(",") if v.strip()]
    return [int(v, 0) for v in vals]


def gguf_grid(cls):
    cls.init_grid()
    return np.asarray(cls.grid, dtype=np.float32).reshape(cls.grid_shape)


@pytest.mark.parametrize("name,cls,dim", [("IQ2XXS_GRID", "IQ2_XXS", 8), ("IQ2XS_GRID", "IQ2_XS", 8),
                                          ("IQ2S_GRID", "IQ2_S", 8), ("IQ3XXS_GRID", "IQ3_XXS", 4),
                                          ("IQ3S_GRID", "IQ3_S", 4)])
def test_decode_grids_match_gguf_py(name, cls, dim):
    ours = np.array([[(v >> (8 * k)) & 0xFF for k in range(dim)] for v in table(name)], dtype=np.float32)
    theirs = gguf_grid(getattr(gguf.quants, cls))
    assert np.array_equal(ours, theirs)


def test_small_tables():
    assert table("KMASK_IQ2XS") == [1 << i for i in range(8)]
    # ksigns: 7 stored bits + the parity bit that makes the popcount even
    ks = table("KSIGNS_IQ2XS")
    assert ks == [i | ((bin(i).count("1") & 1) << 7) for i in range(128)]
    vals = table("KVALUES_IQ4NL")
    vals = [v - 256 if v > 127 else v for v in vals]
    assert vals == list(gguf.quants.IQ4_NL.kvalues)


@pytest.mark.parametrize("kgrid,grid,levels,bits,dim", [
    ("KGRID_2BIT_256", "IQ2XXS_GRID", (0x08, 0x19, 0x2b), 2, 8),
    ("KGRID_2BIT_512", "IQ2XS_GRID", (0x08, 0x19, 0x2b), 2, 8),
    ("KGRID_2BIT_1024", "IQ2S_GRID", (0x08, 0x19, 0x2b), 2, 8),
    ("KGRID_256", "IQ3XXS_GRID", (0x04, 0x0c, 0x14, 0x1c, 0x24, 0x2c, 0x34, 0x3e), 3, 4),
    ("KGRID_512", "IQ3S_GRID", (0x01, 0x03, 0x05, 0x07, 0x09, 0x0b, 0x0d, 0x0f), 3, 4)])
def test_encoder_lattice_matches_decode_grid(kgrid, grid, levels, bits, dim):
    """Point i of the encoder lattice is the level index of decode-grid entry i."""
    for k_packed, g in zip(table(kgrid), table(grid)):
        for k in range(dim):
            assert levels[(k_packed >> (bits * k)) & ((1 << bits) - 1)] == (g >> (8 * k)) & 0xFF


@pytest.mark.parametrize("which", range(5))
def test_library_compact_tables_match_oracle(which):
    import shoehorn_b200 as sh
    gs, kmap, nb = O.grid_info(which)
    gs2, cmap, cnb = sh.grid_info(which)
    assert gs == gs2
    dim, bits, levels = (8, 2, 3) if which < 3 else (4, 3, 8)
    grid_packed = table(["KGRID_2BIT_256", "KGRID_2BIT_512", "KGRID_2BIT_1024", "KGRID_256", "KGRID_512"][which])
    for c in range(levels ** dim):
        rem, u = c, 0
        for k in range(dim):
            u |= (rem % levels) << (bits * k)
            rem //= levels
        m, cm = int(kmap[u]), int(cmap[c])
        if m >= 0:
            assert cm == m
            continue
        assert cm < 0
        off, coff = -m - 1, -cm - 1
        n = int(nb[off])
        assert int(cnb[coff]) == n
        for t in range(n):
            e = int(cnb[coff + 1 + t])
            j = int(nb[off + 1 + t])
            assert (e & 0xFFFF) == j and (e >> 16) == grid_packed[j]
