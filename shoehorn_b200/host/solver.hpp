// Exact-fit quant-mix solver (reference src/solver.rs:1-108): multiple-choice
// knapsack by Lagrangian bisection, then greedy upgrades into the slack.
#pragma once
#include <cstdint>
#include <optional>
#include <vector>

namespace shh {

struct Candidate {
    uint32_t ty = 0;
    uint64_t bytes = 0;
    double err = 0.0;  // imatrix-weighted squared error of the tensor in this type
};

struct TensorChoices {
    size_t tensor_idx = 0;
    std::vector<Candidate> cands;  // sorted by bytes ascending
};

// Chosen candidate index per entry, or nothing if even the smallest mix
// exceeds the budget.
std::optional<std::vector<size_t>> solve(const std::vector<TensorChoices> &tensors, uint64_t budget);

}  // namespace shh
