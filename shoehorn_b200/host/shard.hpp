// Row-range sharding of the plan / quantize flow over the ranks of one job,
// one process per GPU.  Rank r owns rows [n*r/W, n*(r+1)/W) of every tensor:
// it measures the error-table rows it owns, exchanges them with the other
// ranks (the only communication: an all-gather of per-row f64 errors, no
// collective on the data path), solves the same plan as every other rank,
// and encodes its own rows.  Rows depend only on themselves, their imatrix
// slice and read-only tables, so every byte and every error equals the
// single-process result; the per-tensor errors are still summed in row order
// (main.rs:553-555) after the exchange.
#pragma once
#include <cstdint>
#include <cstring>
#include <functional>
#include <vector>

#include "gguf.hpp"

namespace shh {

struct Shard {
    int rank = 0, world = 1;
    // Every rank's blob, in rank order (an all-gather of byte strings).
    std::function<std::vector<std::vector<uint8_t>>(const std::vector<uint8_t> &)> allgather;
    // Returns once every rank has called it.
    std::function<void()> barrier;
    bool active() const { return world > 1; }
};

// Rows [lo, hi) of an n_rows tensor owned by `rank` of `world`.
inline void shard_rows(uint64_t n_rows, int rank, int world, uint64_t &lo, uint64_t &hi) {
    lo = n_rows * (uint64_t)rank / (uint64_t)world;
    hi = n_rows * (uint64_t)(rank + 1) / (uint64_t)world;
}

// Sampled indices [i0, i1) (row i*step) that fall in rows [lo, hi).
inline void shard_samples(uint64_t lo, uint64_t hi, uint64_t step, uint64_t sampled, uint64_t &i0, uint64_t &i1) {
    auto ceil_div = [](uint64_t a, uint64_t b) { return (a + b - 1) / b; };
    i0 = ceil_div(lo, step);
    i1 = ceil_div(hi, step);
    if (i0 > sampled) i0 = sampled;
    if (i1 > sampled) i1 = sampled;
}

// One tensor's measured error rows: err[c][i] for candidate c and sampled
// row i (row i*step of an n_rows tensor).
struct MeasRows {
    uint64_t n_rows = 0, step = 1, sampled = 0;
    std::vector<std::vector<double>> err;
};

// The rows of `m` that `rank` owns, packed tensor by tensor, candidate by
// candidate, in row order.
inline std::vector<uint8_t> pack_rows(const std::vector<MeasRows> &m, int rank, int world) {
    std::vector<uint8_t> out;
    for (const auto &t : m) {
        uint64_t lo, hi, i0, i1;
        shard_rows(t.n_rows, rank, world, lo, hi);
        shard_samples(lo, hi, t.step, t.sampled, i0, i1);
        for (const auto &e : t.err) {
            const size_t at = out.size(), n = (size_t)(i1 - i0) * sizeof(double);
            out.resize(at + n);
            if (n) std::memcpy(out.data() + at, e.data() + i0, n);
        }
    }
    return out;
}

// Inverse of pack_rows for rank `rank`'s blob; throws on a size mismatch.
inline void unpack_rows(std::vector<MeasRows> &m, int rank, int world, const std::vector<uint8_t> &blob) {
    size_t at = 0;
    for (auto &t : m) {
        uint64_t lo, hi, i0, i1;
        shard_rows(t.n_rows, rank, world, lo, hi);
        shard_samples(lo, hi, t.step, t.sampled, i0, i1);
        for (auto &e : t.err) {
            const size_t n = (size_t)(i1 - i0) * sizeof(double);
            if (at + n > blob.size()) throw Error("error-table exchange: short blob from rank " + std::to_string(rank));
            if (n) std::memcpy(e.data() + i0, blob.data() + at, n);
            at += n;
        }
    }
    if (at != blob.size()) throw Error("error-table exchange: long blob from rank " + std::to_string(rank));
}

// All-gather of the measured rows: afterwards every rank holds every row.
inline void exchange_rows(std::vector<MeasRows> &m, const Shard &s) {
    if (!s.active()) return;
    if (!s.allgather) throw Error("sharded run without an all-gather");
    const auto all = s.allgather(pack_rows(m, s.rank, s.world));
    if ((int)all.size() != s.world) throw Error("error-table exchange: wrong number of ranks");
    for (int r = 0; r < s.world; r++)
        if (r != s.rank) unpack_rows(m, r, s.world, all[(size_t)r]);
}

// Per-candidate error of a tensor: the sampled rows summed in row order,
// scaled by n_rows / sampled (main.rs:546-560).
inline double tensor_error(const MeasRows &t, size_t c) {
    double err = 0.0;
    for (double e : t.err[c]) err += e;
    return err * ((double)t.n_rows / (double)t.sampled);
}

}  // namespace shh
