// Multiple-choice knapsack (reference src/solver.rs:21-108).  Host-side: it
// is O(tensors x candidates x iterations) and runs in milliseconds.
#include "solver.hpp"

#include <limits>

namespace shh {

std::optional<std::vector<size_t>> solve(const std::vector<TensorChoices> &tensors, uint64_t budget) {
    uint64_t min_total = 0;
    for (auto &t : tensors) min_total += t.cands[0].bytes;
    if (min_total > budget) return std::nullopt;

    // lowest cost c.err + lambda*bytes per tensor; ties keep the first (solver.rs:27-44)
    auto pick = [&](double lambda, std::vector<size_t> &sel) -> uint64_t {
        uint64_t total = 0;
        sel.assign(tensors.size(), 0);
        for (size_t ti = 0; ti < tensors.size(); ti++) {
            const auto &t = tensors[ti];
            size_t best = 0;
            double best_cost = std::numeric_limits<double>::infinity();
            for (size_t i = 0; i < t.cands.size(); i++) {
                const double cost = t.cands[i].err + lambda * (double)t.cands[i].bytes;
                if (cost < best_cost) {
                    best_cost = cost;
                    best = i;
                }
            }
            total += t.cands[best].bytes;
            sel[ti] = best;
        }
        return total;
    };

    std::vector<size_t> best_sel;
    uint64_t best_total = pick(0.0, best_sel);
    if (best_total > budget) {
        // bisect lambda until the mix fits snugly (solver.rs:52-72)
        double lo = 0.0, hi = 1.0;
        std::vector<size_t> sel;
        while (pick(hi, sel) > budget) {
            hi *= 8.0;
            if (hi > 1e30) return std::nullopt;
        }
        best_total = pick(hi, best_sel);
        for (int it = 0; it < 64; it++) {
            const double mid = 0.5 * (lo + hi);
            const uint64_t total = pick(mid, sel);
            if (total <= budget) {
                hi = mid;
                best_sel = sel;
                best_total = total;
            } else {
                lo = mid;
            }
        }
    }
    // greedy top-up: best err reduction per byte that fits the slack (solver.rs:75-105)
    for (;;) {
        const uint64_t slack = budget - best_total;
        double best_gain = 0.0;
        bool have = false;
        size_t bt = 0, bc = 0;
        for (size_t ti = 0; ti < tensors.size(); ti++) {
            const auto &cur = tensors[ti].cands[best_sel[ti]];
            for (size_t ci = 0; ci < tensors[ti].cands.size(); ci++) {
                const auto &c = tensors[ti].cands[ci];
                if (c.bytes <= cur.bytes || c.err >= cur.err) continue;
                const uint64_t extra = c.bytes - cur.bytes;
                if (extra > slack) continue;
                const double gain = (cur.err - c.err) / (double)extra;
                if (gain > best_gain) {
                    best_gain = gain;
                    have = true;
                    bt = ti;
                    bc = ci;
                }
            }
        }
        if (!have) break;
        best_total += tensors[bt].cands[bc].bytes - tensors[bt].cands[best_sel[bt]].bytes;
        best_sel[bt] = bc;
    }
    return best_sel;
}

}  // namespace shh
