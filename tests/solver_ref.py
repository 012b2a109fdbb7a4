"""Python restatement of the reference solver (solver.rs:21-108) used by the
tests to check the host pipeline's plans against the oracle's error table."""


def solve(tensors, budget):
    """tensors: list of lists of (bytes, err) sorted by bytes. Returns picks or None."""
    if sum(t[0][0] for t in tensors) > budget:
        return None

    def pick(lam):
        total, sel = 0, []
        for t in tensors:
            best, best_cost = 0, float("inf")
            for i, (b, e) in enumerate(t):
                cost = e + lam * float(b)
                if cost < best_cost:
                    best_cost, best = cost, i
            total += t[best][0]
            sel.append(best)
        return sel, total

    sel, total = pick(0.0)
    if total > budget:
        lo, hi = 0.0, 1.0
        while pick(hi)[1] > budget:
            hi *= 8.0
            if hi > 1e30:
                return None
        best = pick(hi)
        for _ in range(64):
            mid = 0.5 * (lo + hi)
            s, tot = pick(mid)
            if tot <= budget:
                hi, best = mid, (s, tot)
            else:
                lo = mid
        sel, total = best
    sel = list(sel)
    while True:
        slack = budget - total
        best_gain, move = 0.0, None
        for ti, t in enumerate(tensors):
            cb, ce = t[sel[ti]]
            for ci, (b, e) in enumerate(t):
                if b <= cb or e >= ce:
                    continue
                extra = b - cb
                if extra > slack:
                    continue
                gain = (ce - e) / float(extra)
                if gain > best_gain:
                    best_gain, move = gain, (ti, ci)
        if move is None:
            break
        ti, ci = move
        total += tensors[ti][ci][0] - tensors[ti][sel[ti]][0]
        sel[ti] = ci
    return sel
