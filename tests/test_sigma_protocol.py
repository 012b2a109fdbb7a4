"""The row sigma^2 kernel's stage hand-off, replayed on the CPU.

row_sigma2_kernel (shoehorn_b200/csrc/kquant.cu) has three loader warps and a
folding warp that pass ring stages to each other through hardware named
barriers: FULL(s) (loaders arrive, folder syncs) and EMPTY(s) (folder arrives,
loaders sync), each completing once all four warps reached it.  A mistake in
the order of these calls hangs the kernel (a barrier that never completes) or
lets two tiles' arrivals meet in one barrier instance.  These tests replay the
exact sequence of barrier calls each warp makes, under many interleavings, for
every tile count a row can have up to 300 tiles (153,600 BF16 columns), and
check that every warp finishes and that every barrier instance collects the
arrivals of one tile only.
"""
import random

import pytest

STAGES = 6   # kSigStages
LOADERS = 3  # kSigLoaders


def loader_calls(ntiles):
    """Barrier calls of one loader warp, in program order."""
    ops = []
    for t in range(ntiles):
        if t >= STAGES - 1:
            ops.append(("arrive", "F", t - (STAGES - 1)))
        if t >= STAGES:
            ops.append(("sync", "E", t - STAGES))
    first = ntiles - (STAGES - 1) if ntiles > STAGES - 1 else 0
    for t in range(first, ntiles):
        ops.append(("arrive", "F", t))
    return ops


def folder_calls(ntiles, full_tiles):
    """Barrier calls of the folding warp: FULL of the next tile is synced
    before the current tile's stage is released."""
    ops = []
    if full_tiles > 0:
        ops.append(("sync", "F", 0))
    for t in range(full_tiles):
        if t + 1 < ntiles:
            ops.append(("sync", "F", t + 1))
        if t + STAGES < ntiles:
            ops.append(("arrive", "E", t))
    if full_tiles < ntiles:
        t = full_tiles
        if t == 0:
            ops.append(("sync", "F", 0))
        if t + STAGES < ntiles:
            ops.append(("arrive", "E", t))
    return ops


def replay(ntiles, full_tiles, rng):
    warps = [loader_calls(ntiles) for _ in range(LOADERS)] + [folder_calls(ntiles, full_tiles)]
    pc = [0] * len(warps)
    bars = {}      # (kind, stage) -> {"tile", "arrived", "gen"}
    waiting = {}   # warp -> generation it waits to see completed
    while True:
        runnable = []
        for w, ops in enumerate(warps):
            if pc[w] >= len(ops):
                continue
            if w in waiting:
                _, kind, t = ops[pc[w]]
                if bars[(kind, t % STAGES)]["gen"] > waiting[w]:
                    runnable.append(w)
            else:
                runnable.append(w)
        if not runnable:
            assert all(pc[w] >= len(warps[w]) for w in range(len(warps))), \
                f"hang: {ntiles} tiles, warps stopped at {pc}"
            return
        w = rng.choice(runnable)
        op, kind, t = warps[w][pc[w]]
        if w in waiting:
            del waiting[w]
            pc[w] += 1
            continue
        b = bars.setdefault((kind, t % STAGES), {"tile": None, "arrived": set(), "gen": 0})
        if b["tile"] is None:
            b["tile"] = t
        assert b["tile"] == t, f"{kind}({t % STAGES}) mixes tiles {b['tile']} and {t} ({ntiles} tiles)"
        assert w not in b["arrived"], f"warp {w} arrives twice at {kind}({t % STAGES})"
        b["arrived"].add(w)
        if len(b["arrived"]) == LOADERS + 1:
            b.update(tile=None, arrived=set(), gen=b["gen"] + 1)
            pc[w] += 1
        elif op == "arrive":
            pc[w] += 1
        else:
            waiting[w] = b["gen"]


@pytest.mark.parametrize("ragged", [False, True])
def test_sigma_stage_handoff_completes_for_every_tile_count(ragged):
    rng = random.Random(7)
    for ntiles in range(1 if ragged else 0, 301):
        full = ntiles - 1 if ragged else ntiles
        for _ in range(4 if ntiles > 40 else 25):
            replay(ntiles, full, rng)


def test_old_order_would_hang():
    """Planted mistake: a loader that waits for a free stage before it
    announces the oldest landed tile, with the folder syncing the next tile
    first, never completes."""
    global loader_calls
    saved = loader_calls

    def waits_first(ntiles):
        ops = []
        for t in range(ntiles):
            if t >= STAGES:
                ops.append(("sync", "E", t - STAGES))
            if t >= STAGES - 1:
                ops.append(("arrive", "F", t - (STAGES - 1)))
        first = ntiles - (STAGES - 1) if ntiles > STAGES - 1 else 0
        for t in range(first, ntiles):
            ops.append(("arrive", "F", t))
        return ops

    loader_calls = waits_first
    try:
        with pytest.raises(AssertionError, match="hang"):
            replay(20, 20, random.Random(1))
    finally:
        loader_calls = saved
