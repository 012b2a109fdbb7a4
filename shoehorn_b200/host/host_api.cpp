// C ABI of the host library (libshoehorn_host.so): the reference's host-side
// pieces that tests and other hosts call directly.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <thread>

#include "pipeline.hpp"

extern "C" {

// main.rs:209-232 parse_size; 0 on success.
int shh_parse_size(const char *s, uint64_t *out) {
    try {
        *out = shh::parse_size(s);
        return 0;
    } catch (...) {
        return -1;
    }
}

// solver.rs:21-108 over a flat candidate table: tensor t owns candidates
// [offsets[t], offsets[t+1]) sorted by bytes.  Returns 1 and fills sel (one
// index per tensor, relative to the tensor's first candidate) when the
// budget is feasible, 0 when even the smallest mix does not fit, -1 on a
// malformed table.
int shh_solve(const uint64_t *bytes, const double *errs, const int64_t *offsets, int64_t n_tensors, uint64_t budget,
              int64_t *sel) {
    if (n_tensors < 0 || !offsets) return -1;
    std::vector<shh::TensorChoices> ts((size_t)n_tensors);
    for (int64_t t = 0; t < n_tensors; t++) {
        if (offsets[t + 1] <= offsets[t]) return -1;
        ts[(size_t)t].tensor_idx = (size_t)t;
        for (int64_t c = offsets[t]; c < offsets[t + 1]; c++) ts[(size_t)t].cands.push_back({0, bytes[c], errs[c]});
    }
    auto r = shh::solve(ts, budget);
    if (!r) return 0;
    for (int64_t t = 0; t < n_tensors; t++) sel[t] = (int64_t)(*r)[(size_t)t];
    return 1;
}

// imatrix.rs:12-19 load: returns the number of entries (or -1), and the
// values of `name` when present (up to cap floats).
int64_t shh_imatrix_probe(const char *path, const char *name, float *vals, int64_t cap, int64_t *n_vals) {
    try {
        auto im = shh::load_imatrix(path);
        *n_vals = -1;
        auto it = im.find(name ? name : "");
        if (it != im.end()) {
            *n_vals = (int64_t)it->second.size();
            if (vals) std::memcpy(vals, it->second.data(), sizeof(float) * (size_t)std::min<int64_t>(cap, *n_vals));
        }
        return (int64_t)im.size();
    } catch (...) {
        return -1;
    }
}

// Re-serialise a GGUF file through this reader and writer (tests compare
// the result with an independent reader).  0 on success.
int shh_gguf_rewrite(const char *in_path, const char *out_path) {
    try {
        auto m = shh::Model::open(in_path);
        shh::write_streaming(out_path, m->kvs, m->tensors, m->alignment, [&](size_t i) {
            const auto &t = m->tensors[i];
            const uint8_t *p = m->tensor_data(t);
            return std::vector<uint8_t>(p, p + t.byte_size());
        });
        return 0;
    } catch (...) {
        return -1;
    }
}



// ---------------------------------------------------------------------------
// Sharded runs driven by a host program with its own process group (one
// process per GPU).  Communication goes through two callbacks:
//   allgather(user, mine, n_mine, all, cap, sizes): called twice per
//     exchange.  First with all == NULL: gather every rank's blob and return
//     the total size (or < 0 on failure).  Then with a buffer of that size:
//     copy the blobs into it in rank order, write each rank's size to
//     sizes[rank] and return the total.
//   barrier(user): returns 0 once every rank has called it.
// ---------------------------------------------------------------------------
typedef int64_t (*shh_allgather_fn)(void *user, const uint8_t *mine, int64_t n_mine, uint8_t *all, int64_t cap,
                                    int64_t *sizes);
typedef int (*shh_barrier_fn)(void *user);

// The process's peak resident set (VmHWM), 0 if unknown.
static uint64_t peak_rss_bytes() {
    FILE *f = fopen("/proc/self/status", "r");
    if (!f) return 0;
    char line[256];
    uint64_t kb = 0;
    while (fgets(line, sizeof line, f))
        if (strncmp(line, "VmHWM:", 6) == 0) {
            kb = strtoull(line + 6, nullptr, 10);
            break;
        }
    fclose(f);
    return kb * 1024;
}

static shh::Shard make_shard(int rank, int world, shh_allgather_fn ag, shh_barrier_fn bar, void *user) {
    shh::Shard s;
    s.rank = rank;
    s.world = world;
    if (ag)
        s.allgather = [ag, user, world](const std::vector<uint8_t> &mine) {
            const int64_t total = ag(user, mine.data(), (int64_t)mine.size(), nullptr, 0, nullptr);
            if (total < 0) throw shh::Error("all-gather failed");
            std::vector<uint8_t> all((size_t)total);
            std::vector<int64_t> sizes((size_t)world, 0);
            if (ag(user, mine.data(), (int64_t)mine.size(), all.data(), total, sizes.data()) != total)
                throw shh::Error("all-gather failed");
            std::vector<std::vector<uint8_t>> out((size_t)world);
            int64_t at = 0;
            for (int r = 0; r < world; r++) {
                if (sizes[(size_t)r] < 0 || at + sizes[(size_t)r] > total) throw shh::Error("all-gather sizes");
                out[(size_t)r].assign(all.begin() + at, all.begin() + at + sizes[(size_t)r]);
                at += sizes[(size_t)r];
            }
            return out;
        };
    if (bar)
        s.barrier = [bar, user]() {
            if (bar(user) != 0) throw shh::Error("barrier failed");
        };
    return s;
}

// The error-table exchange alone, on made-up errors (no GPU): tensors of
// n_rows[k] rows with n_cands[k] candidates, 128-row sampling unless
// sample_rows says otherwise.  This rank fills the sampled rows it owns with
// a fixed function of (tensor, candidate, row), exchanges them, and writes
// each (tensor, candidate) error -- rows summed in row order and scaled as
// the error table is -- to sums[k * max_cands + c].  0 on success.
int shh_shard_exchange_check(int64_t n_tensors, const uint64_t *n_rows, const int32_t *n_cands, uint64_t sample_rows,
                             int rank, int world, shh_allgather_fn ag, void *user, double *sums) {
    try {
        if (n_tensors < 0 || world < 1 || rank < 0 || rank >= world) return -1;
        int32_t max_c = 1;
        for (int64_t k = 0; k < n_tensors; k++) max_c = std::max(max_c, n_cands[k]);
        std::vector<shh::MeasRows> m((size_t)n_tensors);
        for (int64_t k = 0; k < n_tensors; k++) {
            auto &t = m[(size_t)k];
            t.n_rows = n_rows[k];
            t.step = std::max<uint64_t>(t.n_rows / std::min(sample_rows, std::max<uint64_t>(t.n_rows, 1)), 1);
            t.sampled = (t.n_rows + t.step - 1) / t.step;
            t.err.assign((size_t)n_cands[k], std::vector<double>((size_t)t.sampled, 0.0));
            uint64_t lo, hi, i0, i1;
            shh::shard_rows(t.n_rows, rank, world, lo, hi);
            shh::shard_samples(lo, hi, t.step, t.sampled, i0, i1);
            for (int32_t c = 0; c < n_cands[k]; c++)
                for (uint64_t i = i0; i < i1; i++) {
                    uint64_t x = ((uint64_t)k << 40) ^ ((uint64_t)c << 32) ^ (i * t.step);
                    x += 0x9E3779B97F4A7C15ull;
                    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
                    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
                    x ^= x >> 31;
                    // magnitudes over ~2^40 so that the summation order shows in the bits
                    t.err[(size_t)c][i] = std::ldexp((double)(x >> 11), (int)(x & 63) - 73);
                }
        }
        shh::exchange_rows(m, make_shard(rank, world, ag, nullptr, user));
        for (int64_t k = 0; k < n_tensors; k++)
            for (int32_t c = 0; c < n_cands[k]; c++)
                sums[(size_t)k * (size_t)max_c + (size_t)c] = shh::tensor_error(m[(size_t)k], (size_t)c);
        return 0;
    } catch (...) {
        return -1;
    }
}

// Plan (error table + solve) and encode of a synthetic model configuration
// ("qwen3-0.6b", "llama3-8b", "llama3-70b", "tiny") on this rank's rows, on
// CUDA device `device`.  The model is generated once; then one run per bit
// of `modes` (1: the reference's 128-row sampled error table, 2: every row,
// --exact-errors), each a barrier then measure, exchange, solve and encode.
// budget / reserve / uniform follow the CLI flags (uniform non-empty: a
// fixed mix, no solve, one run).  streaming != 0: no weight storage, every
// row is generated when the pipeline asks for it (host memory bounded by the
// staging buffers).  out_path empty: output in host memory; "-": copied to
// the host and discarded.  Writes a JSON array of timing records into json
// (with the process's peak resident set so far).  0 on success, -1 with the
// message in json on failure.
int shh_bench_model(const char *name, uint64_t seed, int modes, int streaming, const char *budget, const char *reserve,
                    uint64_t ctx, const char *uniform, int workers_per_gpu, int device, int rank, int world,
                    shh_allgather_fn ag, shh_barrier_fn bar, void *user, const char *out_path, char *json,
                    int64_t cap) {
    try {
        shh::FitArgs a;
        if (budget) a.budget = budget;
        if (reserve) a.reserve = reserve;
        if (uniform) a.uniform = uniform;
        a.ctx = ctx;
        a.workers_per_gpu = workers_per_gpu;
        const shh::Shard shard = make_shard(rank, world, ag, bar, user);
        const int threads = (int)std::max(1u, std::thread::hardware_concurrency() / (unsigned)std::max(world, 1));
        auto c0 = std::chrono::steady_clock::now();
        auto sm = streaming ? shh::synthetic_model_streaming(name, seed)
                            : shh::synthetic_model(name, seed, threads, rank, world);
        const double gen_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - c0).count();
        shh::GpuPool pool(1, a.timeout_ms, a.workers_per_gpu, device);
        uint64_t elems = 0, mine = 0;
        for (size_t i = 0; i < sm->view.tensors.size(); i++) {
            const auto &t = sm->view.tensors[i];
            uint64_t lo, hi;
            shh::shard_rows(t.n_rows(), rank, world, lo, hi);
            elems += t.n_elements();
            mine += (hi - lo) * t.ne0();
        }
        std::string out = "[";
        for (int mode = 1; mode <= 2; mode++) {
            if (!(modes & mode)) continue;
            a.exact_errors = mode == 2;
            if (shard.active()) shard.barrier();
            shh::Timing tm;
            const auto t0 = std::chrono::steady_clock::now();
            const shh::Plan plan = shh::build_plan(a, sm->view, sm->imatrix, pool, tm, shard);
            shh::write_quantized(out_path ? out_path : "", plan, sm->view, sm->imatrix, pool, tm, shard);
            const double wall = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            std::map<std::string, uint64_t> by_type;
            for (auto &e : plan.entries) by_type[shh::type_name(e.ty)] += sm->view.tensors[e.tensor_idx].n_elements();
            std::string mix;
            for (auto &kv : by_type) mix += (mix.empty() ? "" : ", ") + ("\"" + kv.first + "\": " + std::to_string(kv.second));
            char rec[4096];
            snprintf(rec, sizeof rec,
                     "{\"model\": \"%s\", \"rank\": %d, \"world\": %d, \"exact_errors\": %s, \"streaming\": %s, "
                     "\"elements\": %llu, \"rank_elements\": %llu, \"generate_s\": %.3f, \"measure_s\": %.4f, "
                     "\"gather_s\": %.4f, \"solve_s\": %.4f, \"setup_s\": %.4f, \"encode_s\": %.4f, "
                     "\"wall_s\": %.4f, \"plan_bytes\": %llu, \"budget_bytes\": %llu, \"peak_rss_bytes\": %llu, "
                     "\"mix_elements\": {%s}}",
                     name, rank, world, a.exact_errors ? "true" : "false", streaming ? "true" : "false",
                     (unsigned long long)elems, (unsigned long long)mine, gen_s, tm.measure_s, tm.gather_s, tm.solve_s,
                     tm.setup_s, tm.encode_s, wall, (unsigned long long)plan.total_bytes,
                     (unsigned long long)plan.budget.model_budget, (unsigned long long)peak_rss_bytes(), mix.c_str());
            out += (out.size() > 1 ? ", " : "") + std::string(rec);
            if (!a.uniform.empty()) break;
        }
        out += "]";
        if ((int64_t)out.size() >= cap) throw shh::Error("timing record too long");
        snprintf(json, (size_t)cap, "%s", out.c_str());
        return 0;
    } catch (const std::exception &e) {
        snprintf(json, (size_t)cap, "%s", e.what());
        return -1;
    }
}

// Rows r0 .. r0 + n - 1 of tensor `tensor` of a synthetic model, as the
// pipeline sees them: mode 0 from the whole model held in memory, 1 from
// rank `rank` of `world` row-sharded copies (the rows must be that rank's),
// 2 from the streaming source.  0 on success.
int shh_synthetic_rows(const char *name, uint64_t seed, int64_t tensor, uint64_t r0, uint64_t n, int mode, int rank,
                       int world, uint8_t *dst) {
    try {
        if (mode == 2) {
            auto sm = shh::synthetic_model_streaming(name, seed);
            sm->view.fill((size_t)tensor, r0, n, 1, dst);
            return 0;
        }
        auto sm = mode == 1 ? shh::synthetic_model(name, seed, 2, rank, world) : shh::synthetic_model(name, seed, 2);
        const auto &t = sm->view.tensors[(size_t)tensor];
        std::memcpy(dst, sm->view.row((size_t)tensor, r0), (size_t)(n * shh::row_bytes(t.ty, t.ne0())));
        return 0;
    } catch (...) {
        return -1;
    }
}

}  // extern "C"
