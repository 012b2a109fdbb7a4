// plan / quantize over the CUDA library (reference src/main.rs:209-751).
#include "pipeline.hpp"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <exception>
#include <map>
#include <mutex>
#include <thread>

#include "shoehorn_cuda.h"

namespace shh {

using Clock = std::chrono::steady_clock;
static double secs_since(Clock::time_point t0) {
    return std::chrono::duration<double>(Clock::now() - t0).count();
}

// ---------------------------------------------------------------------------
// sizes and the budget model (main.rs:209-337)
// ---------------------------------------------------------------------------
uint64_t parse_size(const std::string &s0) {
    std::string s = s0;
    while (!s.empty() && isspace((unsigned char)s.back())) s.pop_back();
    size_t b = 0;
    while (b < s.size() && isspace((unsigned char)s[b])) b++;
    s = s.substr(b);
    std::string lower = s;
    for (auto &c : lower) c = (char)tolower((unsigned char)c);
    auto ends = [&](const char *suf) {
        const size_t n = strlen(suf);
        return lower.size() >= n && lower.compare(lower.size() - n, n, suf) == 0;
    };
    std::string num;
    uint64_t mult = 1;
    if (ends("gib")) { num = lower.substr(0, lower.size() - 3); mult = 1ull << 30; }
    else if (ends("mib")) { num = lower.substr(0, lower.size() - 3); mult = 1ull << 20; }
    else if (ends("gb")) { num = lower.substr(0, lower.size() - 2); mult = 1000000000ull; }
    else if (ends("mb")) { num = lower.substr(0, lower.size() - 2); mult = 1000000ull; }
    else if (ends("g")) { num = lower.substr(0, lower.size() - 1); mult = 1ull << 30; }
    else if (ends("m")) { num = lower.substr(0, lower.size() - 1); mult = 1ull << 20; }
    else num = lower;
    while (!num.empty() && isspace((unsigned char)num.back())) num.pop_back();
    size_t nb = 0;
    while (nb < num.size() && isspace((unsigned char)num[nb])) nb++;
    num = num.substr(nb);
    char *end = nullptr;
    const double v = num.empty() ? NAN : strtod(num.c_str(), &end);
    if (num.empty() || end != num.c_str() + num.size() || std::isnan(v)) throw Error("bad size \"" + s0 + "\"");
    // a bare number up to 4096 means GiB (main.rs:228-230)
    if (mult == 1 && v != 0.0 && v <= 4096.0) mult = 1ull << 30;
    const double r = v * (double)mult;
    if (r <= 0) return 0;
    if (r >= 18446744073709551615.0) return UINT64_MAX;
    return (uint64_t)r;
}

std::string fmt_size(uint64_t b) {
    char buf[64];
    if (b >= (1ull << 30)) snprintf(buf, sizeof buf, "%.2f GiB", (double)b / (double)(1ull << 30));
    else if (b >= (1ull << 20)) snprintf(buf, sizeof buf, "%.1f MiB", (double)b / (double)(1ull << 20));
    else snprintf(buf, sizeof buf, "%llu B", (unsigned long long)b);
    return buf;
}

double kv_bytes_per_element(const std::string &kv) {
    if (kv == "f16") return 2.0;
    if (kv == "q8_0") return 34.0 / 32.0;
    if (kv == "q4_0") return 18.0 / 32.0;
    throw Error("unsupported --kv " + kv + " (use f16, q8_0, or q4_0)");
}

static const Value *find_kv(const std::vector<KV> &kvs, const std::string &key) {
    for (auto &p : kvs)
        if (p.first == key) return &p.second;
    return nullptr;
}

Hyper hyperparams(const std::vector<KV> &kvs) {
    Hyper h;
    const Value *a = find_kv(kvs, "general.architecture");
    if (!a || !a->as_str()) throw Error("missing general.architecture");
    h.arch = *a->as_str();
    auto get = [&](const std::string &key, uint64_t &out) {
        const Value *v = find_kv(kvs, h.arch + "." + key);
        return v && v->as_u64(out);
    };
    if (!get("block_count", h.n_layer)) throw Error("missing block_count");
    if (!get("embedding_length", h.n_embd)) h.n_embd = 0;
    uint64_t n_head = 1;
    if (!get("attention.head_count", n_head)) n_head = 1;
    n_head = std::max<uint64_t>(n_head, 1);
    if (!get("attention.head_count_kv", h.n_kv_head)) h.n_kv_head = n_head;
    if (!get("attention.key_length", h.key_len)) h.key_len = h.n_embd / n_head;
    if (!get("attention.value_length", h.val_len)) h.val_len = h.key_len;
    if (!get("vocab_size", h.n_vocab)) {
        const Value *t = find_kv(kvs, "tokenizer.ggml.tokens");
        h.n_vocab = (t && t->type == 9) ? t->arr.size() : 32000;
    }
    return h;
}

Budget compute_budget(const FitArgs &args, const Hyper &h) {
    Budget b;
    if (!args.budget.empty()) {
        b.usable_vram = parse_size(args.budget);
        b.source = "--budget " + args.budget;
    } else if (!args.target.empty()) {
        b.usable_vram = parse_size(args.target) * 74 / 100;
        b.source = "--target " + args.target + " (74% of RAM, macOS working-set approximation)";
    } else {
        // The reference probes Metal/NVML free memory (vram.rs); here the
        // first GPU's free memory stands in for it.
        size_t free_b = 0, total_b = 0;
        if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess)
            throw Error("no probeable GPU found; pass --budget");
        b.usable_vram = free_b;
        b.source = "CUDA free memory";
    }
    const double kv_elem = kv_bytes_per_element(args.kv);
    b.kv_bytes = (uint64_t)((double)h.n_layer * (double)args.ctx * (double)h.n_kv_head * (double)(h.key_len + h.val_len) *
                            kv_elem);
    const uint64_t ubatch = std::min<uint64_t>(512, args.ctx);
    b.compute_bytes = ubatch * h.n_vocab * 4 + ubatch * h.n_embd * 4 * 8;
    b.reserve = !args.reserve.empty() ? parse_size(args.reserve) : (args.calibrate ? (160ull << 20) : (512ull << 20));
    const uint64_t overhead = b.kv_bytes + b.compute_bytes + b.reserve;
    if (overhead >= b.usable_vram)
        throw Error("no room for weights: VRAM " + fmt_size(b.usable_vram) + " - KV " + fmt_size(b.kv_bytes) +
                    " - compute " + fmt_size(b.compute_bytes) + " - reserve " + fmt_size(b.reserve) +
                    " <= 0 (try smaller --ctx)");
    b.model_budget = b.usable_vram - overhead;
    return b;
}

static bool ends_with(const std::string &s, const char *suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

Disposition dispose(const TensorInfo &t) {
    Disposition d;
    const bool quantizable = t.dims.size() >= 2 && ends_with(t.name, ".weight") && t.ne0() % 32 == 0;
    if (!quantizable) {
        d.fixed = true;
        d.ty = (t.ty == T_F16 || t.ty == T_BF16 || t.ty == T_F32) ? T_F32 : t.ty;
        return d;
    }
    d.fixed = false;
    const bool sensitive = t.name == "token_embd.weight" || t.name == "output.weight";
    if (t.ne0() % 256 == 0) {
        d.cands = {T_IQ4_XS, T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0};
        if (!sensitive) d.cands.insert(d.cands.end(), {T_IQ2_XXS, T_IQ2_XS, T_IQ2_S, T_IQ3_XXS, T_IQ3_S});
    } else {
        d.cands = {T_IQ4_NL, T_Q4_0, T_Q4_1, T_Q5_0, T_Q5_1, T_Q8_0};
    }
    d.cands.push_back(T_F16);
    std::stable_sort(d.cands.begin(), d.cands.end(),
                     [&](uint32_t a, uint32_t b) { return row_bytes(a, t.ne0()) < row_bytes(b, t.ne0()); });
    return d;
}

ModelView view_of(const Model &m) {
    ModelView v;
    v.kvs = m.kvs;
    v.tensors = m.tensors;
    v.alignment = m.alignment;
    v.total_bytes = m.total_bytes();
    const Model *mp = &m;
    v.data = [mp](size_t i) { return mp->tensor_data(mp->tensors[i]); };
    return v;
}

// ---------------------------------------------------------------------------
// GPU workers
// ---------------------------------------------------------------------------
struct GpuPool::Worker {
    int dev = 0;
    shc_ctx *ctx = nullptr;
    cudaStream_t st = nullptr;
    std::vector<void *> dbuf = std::vector<void *>(8, nullptr);
    std::vector<size_t> dsz = std::vector<size_t>(8, 0);
    std::vector<void *> hbuf = std::vector<void *>(4, nullptr);
    std::vector<size_t> hsz = std::vector<size_t>(4, 0);
    void *d(int slot, size_t bytes) {
        if (dsz[(size_t)slot] < bytes) {
            if (dbuf[(size_t)slot]) cudaFree(dbuf[(size_t)slot]);
            dbuf[(size_t)slot] = nullptr;
            dsz[(size_t)slot] = 0;
            if (cudaMalloc(&dbuf[(size_t)slot], bytes) != cudaSuccess) throw Error("device allocation failed");
            dsz[(size_t)slot] = bytes;
        }
        return dbuf[(size_t)slot];
    }
    void *h(int slot, size_t bytes) {
        if (hsz[(size_t)slot] < bytes) {
            if (hbuf[(size_t)slot]) cudaFreeHost(hbuf[(size_t)slot]);
            hbuf[(size_t)slot] = nullptr;
            hsz[(size_t)slot] = 0;
            if (cudaMallocHost(&hbuf[(size_t)slot], bytes) != cudaSuccess) throw Error("pinned allocation failed");
            hsz[(size_t)slot] = bytes;
        }
        return hbuf[(size_t)slot];
    }
};

static void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e));
}
static void shc_check(int rc, const char *what) {
    if (rc != SHC_OK) throw Error(std::string(what) + ": " + shc_status_string(rc));
}

GpuPool::GpuPool(int n_gpus, int64_t timeout_ms, int per_gpu, int first_device) : timeout_ms_(timeout_ms) {
    int avail = 0;
    if (cudaGetDeviceCount(&avail) != cudaSuccess || avail < 1) throw Error("no CUDA device");
    if (first_device < 0 || first_device >= avail) throw Error("no CUDA device " + std::to_string(first_device));
    avail -= first_device;
    if (n_gpus < 1 || n_gpus > avail) n_gpus = n_gpus < 1 ? 1 : avail;
    n_gpus_ = n_gpus;
    if (per_gpu < 1) per_gpu = 1;
    // workers interleave the devices so the first jobs (the largest) spread
    for (int w = 0; w < n_gpus * per_gpu; w++) {
        auto wk = std::make_unique<Worker>();
        wk->dev = first_device + w % n_gpus;
        cuda_check(cudaSetDevice(wk->dev), "cudaSetDevice");
        shc_check(shc_init(wk->dev, &wk->ctx), "shc_init");
        cuda_check(cudaStreamCreateWithFlags(&wk->st, cudaStreamNonBlocking), "cudaStreamCreate");
        workers_.push_back(std::move(wk));
    }
    cudaSetDevice(first_device);
}

GpuPool::~GpuPool() {
    for (auto &w : workers_) {
        cudaSetDevice(w->dev);
        cudaStreamSynchronize(w->st);
        for (auto p : w->dbuf)
            if (p) cudaFree(p);
        for (auto p : w->hbuf)
            if (p) cudaFreeHost(p);
        cudaStreamDestroy(w->st);
        shc_free(w->ctx);
    }
}

void GpuPool::run(size_t n_jobs, const std::function<void(int, size_t)> &fn) {
    std::atomic<size_t> next{0};
    std::exception_ptr err;
    std::mutex mu;
    std::vector<std::thread> th;
    for (int w = 0; w < size(); w++) {
        th.emplace_back([&, w]() {
            cudaSetDevice(workers_[(size_t)w]->dev);
            for (;;) {
                const size_t j = next.fetch_add(1);
                if (j >= n_jobs) break;
                {
                    std::lock_guard<std::mutex> lk(mu);
                    if (err) break;
                }
                try {
                    fn(w, j);
                } catch (...) {
                    std::lock_guard<std::mutex> lk(mu);
                    if (!err) err = std::current_exception();
                    break;
                }
            }
        });
    }
    for (auto &t : th) t.join();
    if (err) std::rethrow_exception(err);
}

void GpuPool::each(const std::function<void(int)> &fn) {
    std::exception_ptr err;
    std::mutex mu;
    std::vector<std::thread> th;
    for (int w = 0; w < size(); w++) {
        th.emplace_back([&, w]() {
            cudaSetDevice(workers_[(size_t)w]->dev);
            try {
                fn(w);
            } catch (...) {
                std::lock_guard<std::mutex> lk(mu);
                if (!err) err = std::current_exception();
            }
        });
    }
    for (auto &t : th) t.join();
    if (err) std::rethrow_exception(err);
}

// Bring rows of one tensor to the device as an f32/f16/bf16 view: a strided
// host->device gather, then a device decode for block-quantized storage
// (the reference decodes with quant.rs:581 decode_row before measuring).
struct DevRows {
    const void *ptr;
    uint32_t src_type;
};
// Rows r0, r0 + step, ... (n of them) of tensor ti: copied from the view's
// resident bytes, or generated by its streaming source into the worker's
// pinned staging buffer first.  The caller synchronises the worker's stream
// before its next job, so the staging buffer is free again by then.
static DevRows rows_to_device(GpuPool::Worker &wk, const ModelView &m, size_t ti, uint64_t r0, uint64_t n,
                              uint64_t step) {
    const TensorInfo &t = m.tensors[ti];
    const uint64_t ne0 = t.ne0(), srb = row_bytes(t.ty, ne0);
    void *raw = wk.d(0, (size_t)(n * srb + 16));
    if (m.streaming()) {
        uint8_t *stage = static_cast<uint8_t *>(wk.h(2, (size_t)(n * srb)));
        m.fill(ti, r0, n, step, stage);
        cuda_check(cudaMemcpyAsync(raw, stage, (size_t)(n * srb), cudaMemcpyHostToDevice, wk.st), "row upload");
    } else {
        cuda_check(cudaMemcpy2DAsync(raw, srb, m.row(ti, r0), srb * step, srb, n, cudaMemcpyHostToDevice, wk.st),
                   "row upload");
    }
    if (t.ty == T_F32 || t.ty == T_F16 || t.ty == T_BF16) return {raw, t.ty};
    void *f = wk.d(1, (size_t)(n * ne0 * 4 + 16));
    shc_check(shc_decode_rows(wk.ctx, t.ty, static_cast<const uint8_t *>(raw), (int64_t)n, (int64_t)ne0,
                              static_cast<float *>(f), wk.st),
              "decode source rows");
    return {f, SHC_SRC_F32};
}

// ---------------------------------------------------------------------------
// build_plan (main.rs:454-589)
// ---------------------------------------------------------------------------
static uint64_t rows_per_mat_of(const TensorInfo &t) { return t.dims.size() >= 3 ? t.dims[1] : t.n_rows(); }

// Parse "TYPE[,name=TYPE...]" for the uniform harness mode.
static void parse_uniform(const std::string &spec, uint32_t &def, std::map<std::string, uint32_t> &over) {
    size_t p = 0;
    bool first = true;
    while (p <= spec.size()) {
        const size_t c = spec.find(',', p);
        const std::string item = spec.substr(p, c == std::string::npos ? std::string::npos : c - p);
        const size_t eq = item.find('=');
        uint32_t ty;
        if (eq == std::string::npos) {
            if (!type_from_name(item, ty)) throw Error("unknown type in --uniform: " + item);
            if (!first) throw Error("--uniform: the default type must come first");
            def = ty;
        } else {
            if (!type_from_name(item.substr(eq + 1), ty)) throw Error("unknown type in --uniform: " + item);
            over[item.substr(0, eq)] = ty;
        }
        first = false;
        if (c == std::string::npos) break;
        p = c + 1;
    }
}

static std::pair<std::vector<PlanEntry>, uint64_t> assemble_entries(const ModelView &m,
                                                                    const std::vector<std::pair<size_t, uint32_t>> &fixed,
                                                                    const std::vector<TensorChoices> &choices,
                                                                    const std::vector<size_t> &sel) {
    std::vector<PlanEntry> entries;
    for (auto &f : fixed) {
        const auto &t = m.tensors[f.first];
        entries.push_back({f.first, f.second, row_bytes(f.second, t.ne0()) * t.n_rows(), false});
    }
    uint64_t solved = 0;
    for (size_t i = 0; i < choices.size(); i++) {
        const auto &c = choices[i].cands[sel[i]];
        solved += c.bytes;
        entries.push_back({choices[i].tensor_idx, c.ty, c.bytes, true});
    }
    std::stable_sort(entries.begin(), entries.end(),
                     [](const PlanEntry &a, const PlanEntry &b) { return a.tensor_idx < b.tensor_idx; });
    return {entries, solved};
}

Plan build_plan(const FitArgs &args, const ModelView &m, const Imatrix &im, GpuPool &pool, Timing &tm,
                const Shard &shard) {
    Plan plan;
    const Hyper h = hyperparams(m.kvs);
    const bool uniform = !args.uniform.empty();
    if (!uniform) plan.budget = compute_budget(args, h);
    if (args.imatrix.empty() && im.empty())
        fprintf(stderr, "warning: no imatrix given; quantizing with activation-agnostic weights\n");
    fprintf(stderr, "model: %s | %zu tensors | arch %s | ctx %llu\n", fmt_size(m.total_bytes).c_str(),
            m.tensors.size(), h.arch.c_str(), (unsigned long long)args.ctx);
    size_t already = 0;
    for (auto &t : m.tensors)
        if (!(t.ty == T_F16 || t.ty == T_BF16 || t.ty == T_F32)) already++;
    if (already * 2 > m.tensors.size())
        fprintf(stderr, "warning: source is already quantized; re-quantizing compounds the loss - start from the "
                        "BF16/F16 GGUF if one exists\n");
    {
        uint64_t train_ctx;
        const Value *v = find_kv(m.kvs, h.arch + ".context_length");
        if (v && v->as_u64(train_ctx) && args.ctx > train_ctx)
            fprintf(stderr, "warning: --ctx %llu exceeds the model's training context %llu; budgeting for it anyway\n",
                    (unsigned long long)args.ctx, (unsigned long long)train_ctx);
    }
    if (!uniform)
        fprintf(stderr, "budget: %s usable (%s) - %s KV - %s compute est - %s reserve = %s for weights\n",
                fmt_size(plan.budget.usable_vram).c_str(), plan.budget.source.c_str(),
                fmt_size(plan.budget.kv_bytes).c_str(), fmt_size(plan.budget.compute_bytes).c_str(),
                fmt_size(plan.budget.reserve).c_str(), fmt_size(plan.budget.model_budget).c_str());

    std::vector<std::pair<size_t, std::vector<uint32_t>>> to_solve;
    size_t n_with_im = 0;
    for (size_t i = 0; i < m.tensors.size(); i++) {
        const auto &t = m.tensors[i];
        const Disposition d = dispose(t);
        if (d.fixed) {
            plan.fixed_bytes += row_bytes(d.ty, t.ne0()) * t.n_rows();
            plan.fixed.emplace_back(i, d.ty);
        } else {
            if (lookup(im, t.name)) n_with_im++;
            to_solve.emplace_back(i, d.cands);
        }
    }
    fprintf(stderr, "tensors: %zu to solve (%zu with imatrix data), %zu fixed (%s)\n", to_solve.size(), n_with_im,
            plan.fixed.size(), fmt_size(plan.fixed_bytes).c_str());

    if (uniform) {
        uint32_t def = T_Q4_K;
        std::map<std::string, uint32_t> over;
        parse_uniform(args.uniform, def, over);
        std::vector<size_t> sel;
        for (auto &ts : to_solve) {
            const auto &t = m.tensors[ts.first];
            auto it = over.find(t.name);
            const uint32_t ty = it != over.end() ? it->second : def;
            TensorChoices tc;
            tc.tensor_idx = ts.first;
            tc.cands.push_back({ty, row_bytes(ty, t.ne0()) * t.n_rows(), 0.0});
            plan.choices.push_back(tc);
            sel.push_back(0);
        }
        auto [entries, solved] = assemble_entries(m, plan.fixed, plan.choices, sel);
        plan.entries = entries;
        plan.total_bytes = plan.fixed_bytes + solved;
        plan.budget.model_budget = plan.total_bytes;
        plan.budget.usable_vram = plan.total_bytes;
        plan.budget.source = "--uniform " + args.uniform;
        return plan;
    }
    if (plan.fixed_bytes >= plan.budget.model_budget) throw Error("fixed tensors alone exceed the weight budget");

    // ---- measure weighted error for every (tensor, candidate) on the GPUs ----
    const auto t0 = Clock::now();
    const uint64_t sample_rows = args.exact_errors ? UINT64_MAX : 128;
    std::vector<MeasRows> meas(to_solve.size());  // err[cand][sampled row]
    struct Job {
        size_t k;        // index into to_solve
        uint64_t i0, i1; // sampled-row range
        double cost;
    };
    std::vector<Job> jobs;
    double total_cost = 0;
    for (size_t k = 0; k < to_solve.size(); k++) {
        const auto &t = m.tensors[to_solve[k].first];
        const uint64_t n_rows = t.n_rows();
        const uint64_t step = std::max<uint64_t>(n_rows / std::min(sample_rows, std::max<uint64_t>(n_rows, 1)), 1);
        const uint64_t sampled = (n_rows + step - 1) / step;
        meas[k].n_rows = n_rows;
        meas[k].step = step;
        meas[k].sampled = sampled;
        meas[k].err.assign(to_solve[k].second.size(), std::vector<double>((size_t)sampled, 0.0));
        total_cost += (double)sampled * (double)t.ne0() * (double)to_solve[k].second.size() / (double)shard.world;
    }
    const double max_job_cost = std::max(total_cost / (8.0 * pool.size()), 1.0);
    for (size_t k = 0; k < to_solve.size(); k++) {
        const auto &t = m.tensors[to_solve[k].first];
        const uint64_t step = meas[k].step, sampled = meas[k].sampled, rpm = rows_per_mat_of(t);
        const double per_row = (double)t.ne0() * (double)to_solve[k].second.size();
        // rows per job: bounded by cost and by ~256 MiB of f32 rows; never across a matrix
        uint64_t cap = std::max<uint64_t>(1, (uint64_t)(max_job_cost / per_row));
        cap = std::min<uint64_t>(cap, std::max<uint64_t>(1, (256ull << 20) / (t.ne0() * 4)));
        // this rank's sampled rows (all of them without a shard)
        uint64_t lo, hi, i_lo, i_hi;
        shard_rows(t.n_rows(), shard.rank, shard.world, lo, hi);
        shard_samples(lo, hi, step, sampled, i_lo, i_hi);
        uint64_t i = i_lo;
        while (i < i_hi) {
            uint64_t end = std::min(i_hi, i + cap);
            const uint64_t mat = (i * step) / rpm;
            while (end > i + 1 && ((end - 1) * step) / rpm != mat) end--;
            jobs.push_back({k, i, end, per_row * (double)(end - i)});
            i = end;
        }
    }
    std::stable_sort(jobs.begin(), jobs.end(), [](const Job &a, const Job &b) { return a.cost > b.cost; });
    pool.run(jobs.size(), [&](int w, size_t j) {
        auto &wk = pool.worker(w);
        const Job &jb = jobs[j];
        const size_t ti = to_solve[jb.k].first;
        const auto &t = m.tensors[ti];
        const auto &types = to_solve[jb.k].second;
        const uint64_t ne0 = t.ne0(), step = meas[jb.k].step, ni = jb.i1 - jb.i0;
        const DevRows src = rows_to_device(wk, m, ti, jb.i0 * step, ni, step);
        const std::vector<float> *tim = lookup(im, t.name);
        const float *ims = row_slice(tim, ne0, rows_per_mat_of(t), jb.i0 * step);
        float *dim = nullptr;
        if (ims) {
            dim = static_cast<float *>(wk.d(2, ne0 * 4));
            cuda_check(cudaMemcpyAsync(dim, ims, ne0 * 4, cudaMemcpyHostToDevice, wk.st), "imatrix upload");
        }
        double *derr = static_cast<double *>(wk.d(3, types.size() * ni * 8));
        shc_check(shc_row_errors(wk.ctx, types.data(), (int)types.size(), src.src_type, src.ptr, (int64_t)ni,
                                 (int64_t)ne0, dim, ims ? (int64_t)ne0 : 0, 0, 0, 1, derr, wk.st),
                  "row errors");
        double *herr = static_cast<double *>(wk.h(0, types.size() * ni * 8));
        cuda_check(cudaMemcpyAsync(herr, derr, types.size() * ni * 8, cudaMemcpyDeviceToHost, wk.st), "error download");
        shc_check(shc_sync(wk.ctx, wk.st, args.timeout_ms), "row errors");
        for (size_t c = 0; c < types.size(); c++)
            std::memcpy(meas[jb.k].err[c].data() + jb.i0, herr + c * ni, ni * 8);
    });
    tm.measure_s = secs_since(t0);
    const auto tg = Clock::now();
    exchange_rows(meas, shard);  // the other ranks' rows (a no-op without a shard)
    tm.gather_s = secs_since(tg);
    for (size_t k = 0; k < to_solve.size(); k++) {
        const auto &t = m.tensors[to_solve[k].first];
        TensorChoices tc;
        tc.tensor_idx = to_solve[k].first;
        for (size_t c = 0; c < to_solve[k].second.size(); c++) {
            const uint32_t ty = to_solve[k].second[c];
            // rows in row order, as the reference's closure folds them
            tc.cands.push_back({ty, row_bytes(ty, t.ne0()) * t.n_rows(), tensor_error(meas[k], c)});
        }
        plan.choices.push_back(std::move(tc));
    }

    const auto t1 = Clock::now();
    const uint64_t weight_budget = plan.budget.model_budget - plan.fixed_bytes;
    auto sel = solve(plan.choices, weight_budget);
    tm.solve_s = secs_since(t1);
    if (!sel) {
        uint64_t mn = 0;
        for (auto &tc : plan.choices) mn += tc.cands[0].bytes;
        throw Error("even the smallest mix (" + fmt_size(mn) + " + " + fmt_size(plan.fixed_bytes) +
                    " fixed) exceeds the weight budget " + fmt_size(plan.budget.model_budget) +
                    "; lower --ctx / --reserve or use a smaller model");
    }
    auto [entries, solved] = assemble_entries(m, plan.fixed, plan.choices, *sel);
    plan.entries = entries;
    plan.total_bytes = plan.fixed_bytes + solved;
    return plan;
}

void print_plan(const Plan &plan, const ModelView &m) {
    printf("\n%-42s %16s %7s %12s %6s\n", "tensor", "shape", "type", "size", "bpw");
    std::map<std::string, std::pair<size_t, uint64_t>> by_type;
    uint64_t total_elems = 0;
    for (auto &t : m.tensors) total_elems += t.n_elements();
    for (auto &e : plan.entries) {
        const auto &t = m.tensors[e.tensor_idx];
        std::string shape;
        for (size_t i = 0; i < t.dims.size(); i++) shape += (i ? "x" : "") + std::to_string(t.dims[i]);
        const double bpw = (double)e.bytes * 8.0 / (double)t.n_elements();
        auto &bt = by_type[type_name(e.ty)];
        bt.first++;
        bt.second += e.bytes;
        printf("%-42s %16s %7s %12s %6.2f\n", t.name.c_str(), shape.c_str(), type_name(e.ty).c_str(),
               fmt_size(e.bytes).c_str(), bpw);
    }
    printf("\nby type:\n");
    for (auto &kv : by_type) printf("  %6s: %3zu tensors, %s\n", kv.first.c_str(), kv.second.first, fmt_size(kv.second.second).c_str());
    const Budget &b = plan.budget;
    printf("\nweights: %s of %s budget (%.3f%% used, %s slack) | overall %.3f bpw\n", fmt_size(plan.total_bytes).c_str(),
           fmt_size(b.model_budget).c_str(), 100.0 * (double)plan.total_bytes / (double)std::max<uint64_t>(b.model_budget, 1),
           fmt_size(b.model_budget - std::min(b.model_budget, plan.total_bytes)).c_str(),
           (double)plan.total_bytes * 8.0 / (double)std::max<uint64_t>(total_elems, 1));
    printf("projected VRAM at ctx: %s weights + %s KV + %s compute + %s reserve = %s of %s available\n",
           fmt_size(plan.total_bytes).c_str(), fmt_size(b.kv_bytes).c_str(), fmt_size(b.compute_bytes).c_str(),
           fmt_size(b.reserve).c_str(), fmt_size(plan.total_bytes + b.kv_bytes + b.compute_bytes + b.reserve).c_str(),
           fmt_size(b.usable_vram).c_str());
}

uint32_t file_type_code(const std::vector<PlanEntry> &entries) {
    uint64_t best_bytes = 0;
    uint32_t best = 1;
    for (auto &e : entries) {
        if (!e.solved) continue;
        uint32_t code;
        switch (e.ty) {
        case T_F16: code = 1; break;
        case T_Q4_0: code = 2; break;
        case T_Q4_1: code = 3; break;
        case T_Q5_0: code = 8; break;
        case T_Q5_1: code = 9; break;
        case T_Q8_0: code = 7; break;
        case T_Q2_K: code = 10; break;
        case T_Q3_K: code = 11; break;
        case T_Q4_K: code = 15; break;
        case T_Q5_K: code = 17; break;
        case T_Q6_K: code = 18; break;
        case T_IQ2_XXS: code = 19; break;
        case T_IQ2_XS: code = 20; break;
        case T_IQ3_XXS: code = 23; break;
        case T_IQ4_NL: code = 25; break;
        case T_IQ3_S: code = 26; break;
        case T_IQ2_S: code = 28; break;
        case T_IQ4_XS: code = 30; break;
        default: code = 1;
        }
        if (e.bytes > best_bytes) {
            best_bytes = e.bytes;
            best = code;
        }
    }
    return best;
}

// ---------------------------------------------------------------------------
// write_quantized (main.rs:691-751): output laid out up front, tensors encoded
// by the GPUs in row ranges straight into a memory map of the temporary file
// ---------------------------------------------------------------------------
void write_quantized(const std::string &out_path, const Plan &plan, const ModelView &m, const Imatrix &im,
                     GpuPool &pool, Timing &tm, const Shard &shard) {
    const auto s0 = Clock::now();
    std::vector<TensorInfo> infos;
    for (auto &e : plan.entries) {
        const auto &t = m.tensors[e.tensor_idx];
        TensorInfo ti;
        ti.name = t.name;
        ti.dims = t.dims;
        ti.ty = e.ty;
        infos.push_back(ti);
    }
    std::vector<KV> kvs;
    for (auto &kv : m.kvs)
        if (kv.first != "general.file_type" && kv.first != "general.quantization_version" && kv.first.rfind("split.", 0) != 0)
            kvs.push_back(kv);
    kvs.emplace_back("general.file_type", Value::U32(file_type_code(plan.entries)));
    kvs.emplace_back("general.quantization_version", Value::U32(2));
    const Layout L = layout_for(kvs, infos, m.alignment);
    const bool lead = shard.rank == 0;
    // rows [lo, hi) of every entry are this rank's (all rows without a shard)
    std::vector<uint64_t> lo(plan.entries.size()), hi(plan.entries.size()), drb(plan.entries.size());
    for (size_t ei = 0; ei < plan.entries.size(); ei++) {
        const auto &t = m.tensors[plan.entries[ei].tensor_idx];
        shard_rows(t.n_rows(), shard.rank, shard.world, lo[ei], hi[ei]);
        drb[ei] = row_bytes(plan.entries[ei].ty, t.ne0());
    }
    // An empty out_path encodes into host memory (benchmarks without a disk
    // write): this rank's header and rows, back to back.  Otherwise *.tmp
    // next to the output, renamed when complete; every rank writes its rows
    // with positional writes from the workers' pinned buffers at their final
    // offsets, so no page of the output is faulted in through a mapping.
    const bool discard = out_path == "-";
    const bool to_file = !out_path.empty() && !discard;
    const std::string tmp = out_path + ".tmp";
    uint8_t *map = nullptr;
    uint64_t map_len = 0;
    std::vector<uint64_t> local_base(plan.entries.size(), 0);
    int fd = -1;
    if (to_file) {
        if (lead) {
            fd = ::open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0644);
            if (fd < 0) throw Error("creating " + tmp);
            if (ftruncate(fd, (off_t)L.total) != 0) {
                ::close(fd);
                throw Error("sizing " + tmp);
            }
        }
        if (shard.active()) {
            shard.barrier();  // the file exists at its full size before the other ranks open it
            if (!lead) {
                fd = ::open(tmp.c_str(), O_RDWR);
                if (fd < 0) throw Error("opening " + tmp);
            }
        }
    } else if (!discard) {
        map_len = lead ? L.data_start : 0;
        for (size_t ei = 0; ei < plan.entries.size(); ei++) {
            local_base[ei] = map_len;
            map_len += (hi[ei] - lo[ei]) * drb[ei];
        }
        if (map_len) {
            map = static_cast<uint8_t *>(mmap(nullptr, map_len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0));
            if (map == MAP_FAILED) throw Error("mapping the output");
            madvise(map, map_len, MADV_HUGEPAGE);
            // faulted in up front by several threads (an in-memory consumer hands
            // over a buffer it owns; the kernel's page zeroing is the cost)
            const unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
            std::vector<std::thread> th;
            const uint64_t per = (map_len + nt - 1) / nt;
            for (unsigned i = 0; i < nt; i++)
                th.emplace_back([map, per, i, total = map_len]() {
                    const uint64_t a = per * i, b = std::min<uint64_t>(total, a + per);
                    for (uint64_t o = a; o < b; o += 4096) map[o] = 0;
                });
            for (auto &t : th) t.join();
        }
    }
    auto pwrite_all = [&](uint64_t off, const void *p, size_t n) {
        const uint8_t *b = static_cast<const uint8_t *>(p);
        while (n) {
            const ssize_t w = pwrite(fd, b, n, (off_t)off);
            if (w <= 0) throw Error("writing " + tmp);
            b += w;
            off += (uint64_t)w;
            n -= (size_t)w;
        }
    };
    // rows starting at row r0 of entry ei
    auto put_rows = [&](size_t ei, uint64_t r0, const void *p, size_t n) {
        if (discard) return;
        if (to_file) pwrite_all(L.data_start + L.offsets[ei] + r0 * drb[ei], p, n);
        else std::memcpy(map + local_base[ei] + (r0 - lo[ei]) * drb[ei], p, n);
    };
    struct Job {
        size_t e;
        uint64_t r0, r1;
        double cost;
    };
    std::vector<Job> jobs;
    uint64_t total_elems = 0;
    for (size_t ei = 0; ei < plan.entries.size(); ei++)
        total_elems += (hi[ei] - lo[ei]) * m.tensors[plan.entries[ei].tensor_idx].ne0();
    const uint64_t cap_elems = std::max<uint64_t>(1ull << 20, std::min<uint64_t>(64ull << 20, total_elems / (8 * pool.size())));
    for (size_t ei = 0; ei < plan.entries.size(); ei++) {
        const auto &e = plan.entries[ei];
        const auto &t = m.tensors[e.tensor_idx];
        const uint64_t ne0 = t.ne0(), rpm = rows_per_mat_of(t);
        if (e.ty == t.ty) continue;  // copied untouched, below
        const uint64_t rows_cap = std::max<uint64_t>(1, cap_elems / std::max<uint64_t>(ne0, 1));
        for (uint64_t r = lo[ei]; r < hi[ei];) {
            uint64_t end = std::min(hi[ei], r + rows_cap);
            const uint64_t mat = r / rpm;
            end = std::min(end, (mat + 1) * rpm);
            jobs.push_back({ei, r, end, (double)(end - r) * (double)ne0});
            r = end;
        }
    }
    std::stable_sort(jobs.begin(), jobs.end(), [](const Job &a, const Job &b) { return a.cost > b.cost; });
    // Every worker's buffers sized once for the largest job: growing them
    // inside the encode would cudaMalloc/cudaFree (device-wide
    // synchronisations) and pin host pages mid-stream.
    size_t need_raw = 16, need_f = 0, need_im = 16, need_out = 16;
    for (const Job &jb : jobs) {
        const auto &e = plan.entries[jb.e];
        const auto &t = m.tensors[e.tensor_idx];
        const uint64_t ne0 = t.ne0(), n = jb.r1 - jb.r0;
        need_raw = std::max<size_t>(need_raw, (size_t)(n * row_bytes(t.ty, ne0) + 16));
        if (!(t.ty == T_F32 || t.ty == T_F16 || t.ty == T_BF16))
            need_f = std::max<size_t>(need_f, (size_t)(n * ne0 * 4 + 16));
        need_im = std::max<size_t>(need_im, (size_t)(ne0 * 4));
        need_out = std::max<size_t>(need_out, (size_t)(n * row_bytes(e.ty, ne0) + 16));
    }
    if (!jobs.empty())
        pool.each([&](int w) {
            auto &wk = pool.worker(w);
            wk.d(0, need_raw);
            if (need_f) wk.d(1, need_f);
            wk.d(2, need_im);
            wk.d(4, need_out);
            wk.h(1, need_out);
            if (m.streaming()) wk.h(2, need_raw);
        });
    tm.setup_s = secs_since(s0);
    const auto t0 = Clock::now();
    if (lead) {
        const auto hdr = header_bytes(kvs, infos, m.alignment, L);
        if (to_file) pwrite_all(0, hdr.data(), hdr.size());
        else if (map) std::memcpy(map, hdr.data(), hdr.size());
    }
    for (size_t ei = 0; ei < plan.entries.size(); ei++) {  // tensors copied untouched (main.rs:735-737)
        const auto &e = plan.entries[ei];
        if (e.ty != m.tensors[e.tensor_idx].ty || hi[ei] <= lo[ei]) continue;
        const size_t nb = (size_t)((hi[ei] - lo[ei]) * drb[ei]);
        if (m.streaming()) {
            std::vector<uint8_t> tmpb(nb);
            m.fill(e.tensor_idx, lo[ei], hi[ei] - lo[ei], 1, tmpb.data());
            put_rows(ei, lo[ei], tmpb.data(), nb);
        } else {
            put_rows(ei, lo[ei], m.row(e.tensor_idx, lo[ei]), nb);
        }
    }
    pool.run(jobs.size(), [&](int w, size_t j) {
        auto &wk = pool.worker(w);
        const Job &jb = jobs[j];
        const auto &e = plan.entries[jb.e];
        const auto &t = m.tensors[e.tensor_idx];
        const uint64_t ne0 = t.ne0(), n = jb.r1 - jb.r0, rb = drb[jb.e];
        const DevRows src = rows_to_device(wk, m, e.tensor_idx, jb.r0, n, 1);
        const std::vector<float> *tim = lookup(im, t.name);
        const float *ims = row_slice(tim, ne0, rows_per_mat_of(t), jb.r0);
        float *dim = nullptr;
        if (ims) {
            dim = static_cast<float *>(wk.d(2, ne0 * 4));
            cuda_check(cudaMemcpyAsync(dim, ims, ne0 * 4, cudaMemcpyHostToDevice, wk.st), "imatrix upload");
        }
        uint8_t *dout = static_cast<uint8_t *>(wk.d(4, n * rb + 16));
        shc_check(shc_encode_rows(wk.ctx, e.ty, src.src_type, src.ptr, (int64_t)n, (int64_t)ne0, dim,
                                  ims ? (int64_t)ne0 : 0, 0, 0, dout, wk.st),
                  "encode rows");
        uint8_t *hout = static_cast<uint8_t *>(wk.h(1, n * rb));
        cuda_check(cudaMemcpyAsync(hout, dout, n * rb, cudaMemcpyDeviceToHost, wk.st), "encoded download");
        shc_check(shc_sync(wk.ctx, wk.st, 3600 * 1000), "encode rows");
        put_rows(jb.e, jb.r0, hout, n * rb);
    });
    if (map) munmap(map, map_len);
    if (fd >= 0 && ::close(fd) != 0) throw Error("closing " + tmp);
    if (to_file && shard.active()) shard.barrier();  // every rank's rows are in the file
    if (to_file && lead && rename(tmp.c_str(), out_path.c_str()) != 0)
        throw Error("renaming " + tmp + " -> " + out_path);
    tm.encode_s = secs_since(t0);
    fprintf(stderr, "wrote %s (%s)\n", to_file ? out_path.c_str() : discard ? "(discarded)" : "(memory)",
            fmt_size(to_file || discard ? L.total : map_len).c_str());
}

}  // namespace shh
