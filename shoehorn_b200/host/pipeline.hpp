// The plan / quantize flow of the reference (src/main.rs:272-751) over the
// CUDA library: budget model, candidate ladder, the fused error table on the
// GPUs, the knapsack solve, and the streaming GGUF v3 writer.  Tensors, and
// row ranges of large tensors, are spread over the GPUs of one box; there is
// no collective on this path, only a host-side gather of per-row errors
// (summed in row order) and of encoded byte ranges at precomputed offsets.
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "gguf.hpp"
#include "imatrix.hpp"
#include "shard.hpp"
#include "solver.hpp"

struct shc_ctx;

namespace shh {

struct FitArgs {  // main.rs:43-85, plus the GPU harness options
    std::string model, imatrix;
    uint64_t ctx = 8192;
    std::string budget, target, kv = "f16", reserve;
    bool calibrate = false;
    bool exact_errors = false;
    int gpus = 1;
    int workers_per_gpu = 4;  // concurrent jobs (own stream and context) per GPU (4 measured best of 2/3/4/6)
    std::string uniform;  // "TYPE[,tensor=TYPE...]": fixed mix instead of a solve
    int64_t timeout_ms = 3600 * 1000;
};

uint64_t parse_size(const std::string &s);  // main.rs:209-232
std::string fmt_size(uint64_t b);           // main.rs:252-260
double kv_bytes_per_element(const std::string &kv);

struct Hyper {  // main.rs:262-292
    std::string arch;
    uint64_t n_layer = 0, n_kv_head = 0, key_len = 0, val_len = 0, n_embd = 0, n_vocab = 0;
};
Hyper hyperparams(const std::vector<KV> &kvs);

struct Budget {  // main.rs:294-337
    uint64_t usable_vram = 0, kv_bytes = 0, compute_bytes = 0, reserve = 0, model_budget = 0;
    std::string source;
};
Budget compute_budget(const FitArgs &args, const Hyper &h);

struct Disposition {  // main.rs:339-380
    bool fixed = true;
    uint32_t ty = T_F32;
    std::vector<uint32_t> cands;  // sorted by row bytes (stable)
};
Disposition dispose(const TensorInfo &t);

struct PlanEntry {
    size_t tensor_idx = 0;
    uint32_t ty = 0;
    uint64_t bytes = 0;
    bool solved = false;
};

struct Timing {
    // setup_s: the encode's buffer set-up (pinned staging and device buffers
    // sized for the largest job on every worker, the in-memory output faulted
    // in), kept out of encode_s; gather_s: the error-table exchange of a
    // sharded run (waiting for the slowest rank included)
    double measure_s = 0, gather_s = 0, solve_s = 0, encode_s = 0, setup_s = 0;
};

struct Plan {
    std::vector<PlanEntry> entries;
    Budget budget;
    uint64_t total_bytes = 0;
    std::vector<TensorChoices> choices;
    std::vector<std::pair<size_t, uint32_t>> fixed;
    uint64_t fixed_bytes = 0;
};

// Tensor storage seen by the pipeline: infos plus either a host pointer to
// each tensor's raw bytes (an mmap'd GGUF, or synthetic data in host
// memory), or a streaming source that writes requested rows into a caller's
// buffer (synthetic models too large to hold: their rows are generated on
// demand into the workers' pinned staging buffers).
// A rank of a sharded run may hold only rows [row_lo[i], ...) of tensor i:
// data(i) then points at row row_lo[i] (row_lo empty: whole tensors).
struct ModelView {
    std::vector<KV> kvs;
    std::vector<TensorInfo> tensors;
    uint64_t alignment = 32;
    std::function<const uint8_t *(size_t)> data;
    // streaming source: rows r0, r0 + step, ... (n of them) of tensor i,
    // written back to back into dst
    std::function<void(size_t i, uint64_t r0, uint64_t n, uint64_t step, uint8_t *dst)> fill;
    uint64_t total_bytes = 0;
    std::vector<uint64_t> row_lo;
    bool streaming() const { return (bool)fill; }
    // host address of row r of tensor i (resident tensors only)
    const uint8_t *row(size_t i, uint64_t r) const {
        const auto &t = tensors[i];
        const uint64_t lo = row_lo.empty() ? 0 : row_lo[i];
        return data(i) + (r - lo) * row_bytes(t.ty, t.ne0());
    }
};
ModelView view_of(const Model &m);

// Worker threads, each with its own library context and stream, several per
// GPU so that one job's copies overlap another's kernels.
class GpuPool {
  public:
    // devices first_device .. first_device + n_gpus - 1
    GpuPool(int n_gpus, int64_t timeout_ms, int per_gpu = 4, int first_device = 0);
    ~GpuPool();
    int size() const { return (int)workers_.size(); }
    int gpus() const { return n_gpus_; }
    // Runs fn(worker, job) for jobs 0..n_jobs-1, pulled dynamically by the
    // workers in index order; rethrows the first failure.
    void run(size_t n_jobs, const std::function<void(int, size_t)> &fn);
    // Runs fn(worker) once on every worker, each on its own thread with its
    // device current; rethrows the first failure.
    void each(const std::function<void(int)> &fn);
    struct Worker;
    Worker &worker(int w) { return *workers_[(size_t)w]; }

  private:
    std::vector<std::unique_ptr<Worker>> workers_;
    int64_t timeout_ms_;
    int n_gpus_ = 1;
};

// main.rs:454-589 build_plan: measures every (tensor, candidate) error on
// the GPUs and solves for the budget (or applies the uniform mix).  With an
// active shard this rank measures the rows it owns and the table is
// completed by the exchange; every rank returns the same plan.
Plan build_plan(const FitArgs &args, const ModelView &m, const Imatrix &im, GpuPool &pool, Timing &tm,
                const Shard &shard = Shard());
void print_plan(const Plan &plan, const ModelView &m);
uint32_t file_type_code(const std::vector<PlanEntry> &entries);  // main.rs:628-659
// main.rs:691-751 write_quantized (without the calibration reuse path):
// writes out_path via a temporary file and a rename.  An empty out_path
// encodes into host memory; "-" copies every encoded range to the host and
// discards it (a sink for models whose output would not fit in memory).  With an active shard every rank encodes the
// rows it owns and writes them at their final offsets of the same file
// (rank 0 writes the header; the barrier orders creation and the rename).
void write_quantized(const std::string &out_path, const Plan &plan, const ModelView &m, const Imatrix &im,
                     GpuPool &pool, Timing &tm, const Shard &shard = Shard());

// Synthetic models of the benchmark configurations (weights generated from
// a seed straight into host memory).
struct HostBuffer {
    uint8_t *ptr = nullptr;
    size_t n = 0;
    bool pinned = false;
    explicit HostBuffer(size_t bytes);
    ~HostBuffer();
    HostBuffer(const HostBuffer &) = delete;
    HostBuffer &operator=(const HostBuffer &) = delete;
};
struct SyntheticModel {
    ModelView view;
    std::vector<std::unique_ptr<HostBuffer>> storage;
    Imatrix imatrix;
};
// With world > 1 only rows [n*rank/world, n*(rank+1)/world) of each 2-D
// tensor are generated (the rows that rank owns); values do not depend on
// the split.
std::unique_ptr<SyntheticModel> synthetic_model(const std::string &name, uint64_t seed, int threads, int rank = 0,
                                                int world = 1);
// The same models with no weight storage: view.fill generates any rows on
// demand (host memory stays bounded by the pipeline's staging buffers).
std::unique_ptr<SyntheticModel> synthetic_model_streaming(const std::string &name, uint64_t seed);

}  // namespace shh
