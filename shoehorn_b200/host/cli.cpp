// shoehorn-gpu: the reference's `plan` and `quantize` subcommands
// (src/main.rs:36-107, 923-943) over the B200 library, plus harness commands
// for synthetic models:
//   shoehorn-gpu plan     -m MODEL [-i IMATRIX] [--ctx N] [--budget S | --target S] [--kv T]
//                         [--reserve S] [--exact-errors] [--gpus N] [--uniform SPEC]
//   shoehorn-gpu quantize (same) -o OUT
//   shoehorn-gpu synth NAME OUT.gguf [--imatrix OUT.imatrix] [--seed N]
//   shoehorn-gpu bench-model NAME [plan flags] [-o OUT]   (synthetic model in memory; JSON timing line)
#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "pipeline.hpp"

using namespace shh;

static void usage() {
    fprintf(stderr,
            "usage: shoehorn-gpu plan|quantize -m MODEL [-i IMATRIX] [-o OUT] [--ctx N] [--budget S|--target S]\n"
            "                    [--kv f16|q8_0|q4_0] [--reserve S] [--exact-errors] [--gpus N] [--uniform SPEC]\n"
            "       shoehorn-gpu synth NAME OUT.gguf [--imatrix OUT.imatrix] [--seed N]\n"
            "       shoehorn-gpu bench-model NAME [plan flags] [-o OUT]\n");
}

static void write_legacy_imatrix(const std::string &path, const Imatrix &im) {
    FILE *f = fopen(path.c_str(), "wb");
    if (!f) throw Error("creating " + path);
    auto i32 = [&](int32_t v) { fwrite(&v, 4, 1, f); };
    i32((int32_t)im.size());
    for (auto &kv : im) {
        i32((int32_t)kv.first.size());
        fwrite(kv.first.data(), 1, kv.first.size(), f);
        i32(1);  // ncall
        i32((int32_t)kv.second.size());
        fwrite(kv.second.data(), 4, kv.second.size(), f);
    }
    fclose(f);
}

int main(int argc, char **argv) {
    if (argc < 2) {
        usage();
        return 2;
    }
    const std::string cmd = argv[1];
    FitArgs a;
    std::string out, synth_name, synth_out, synth_im;
    uint64_t seed = 20261201;
    int pos = 0;
    for (int i = 2; i < argc; i++) {
        const std::string s = argv[i];
        auto val = [&]() -> std::string {
            if (i + 1 >= argc) throw Error("missing value for " + s);
            return argv[++i];
        };
        try {
            if (s == "-m" || s == "--model") a.model = val();
            else if (s == "-i" || s == "--imatrix") (cmd == "synth" ? synth_im : a.imatrix) = val();
            else if (s == "-o" || s == "--output") out = val();
            else if (s == "--ctx") a.ctx = std::stoull(val());
            else if (s == "--budget") a.budget = val();
            else if (s == "--target") a.target = val();
            else if (s == "--kv") a.kv = val();
            else if (s == "--reserve") a.reserve = val();
            else if (s == "--calibrate") a.calibrate = true;
            else if (s == "--exact-errors") a.exact_errors = true;
            else if (s == "--gpus") a.gpus = std::stoi(val());
            else if (s == "--streams") a.workers_per_gpu = std::stoi(val());
            else if (s == "--uniform") a.uniform = val();
            else if (s == "--seed") seed = std::stoull(val());
            else if (!s.empty() && s[0] != '-') {
                if (pos == 0) synth_name = s;
                else if (pos == 1) synth_out = s;
                pos++;
            } else {
                fprintf(stderr, "unknown argument %s\n", s.c_str());
                usage();
                return 2;
            }
        } catch (const std::exception &e) {
            fprintf(stderr, "error: %s\n", e.what());
            return 2;
        }
    }
    if (!a.budget.empty() && !a.target.empty()) {
        fprintf(stderr, "error: --budget conflicts with --target\n");
        return 2;
    }
    if (a.calibrate) {
        fprintf(stderr, "error: --calibrate needs llama.cpp, which this build does not drive\n");
        return 2;
    }
    const int threads = (int)std::max(1u, std::thread::hardware_concurrency());
    try {
        if (cmd == "synth") {
            if (synth_name.empty() || synth_out.empty()) throw Error("synth NAME OUT.gguf");
            auto sm = synthetic_model(synth_name, seed, threads);
            write_streaming(synth_out, sm->view.kvs, sm->view.tensors, sm->view.alignment,
                            [&](size_t i) {
                                const auto &t = sm->view.tensors[i];
                                const uint8_t *p = sm->view.data(i);
                                return std::vector<uint8_t>(p, p + t.byte_size());
                            });
            if (!synth_im.empty()) write_legacy_imatrix(synth_im, sm->imatrix);
            fprintf(stderr, "wrote %s (%s)\n", synth_out.c_str(), fmt_size(sm->view.total_bytes).c_str());
            return 0;
        }
        if (cmd == "plan" || cmd == "quantize") {
            if (a.model.empty()) throw Error("--model is required");
            if (cmd == "quantize" && out.empty()) throw Error("--output is required");
            auto model = Model::open(a.model);
            const ModelView mv = view_of(*model);
            Imatrix im;
            if (!a.imatrix.empty()) im = load_imatrix(a.imatrix);
            GpuPool pool(a.gpus, a.timeout_ms, a.workers_per_gpu);
            Timing tm;
            const Plan plan = build_plan(a, mv, im, pool, tm);
            print_plan(plan, mv);
            if (cmd == "quantize") write_quantized(out, plan, mv, im, pool, tm);
            fprintf(stderr, "timing: measure %.3f s, solve %.3f s, encode %.3f s on %d GPU(s)\n", tm.measure_s,
                    tm.solve_s, tm.encode_s, pool.gpus());
            return 0;
        }
        if (cmd == "bench-model") {
            if (synth_name.empty()) throw Error("bench-model NAME");
            const auto g0 = std::chrono::steady_clock::now();
            auto sm = synthetic_model(synth_name, seed, threads);
            const double gen_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - g0).count();
            GpuPool pool(a.gpus, a.timeout_ms, a.workers_per_gpu);
            Timing tm;
            const auto t0 = std::chrono::steady_clock::now();
            const Plan plan = build_plan(a, sm->view, sm->imatrix, pool, tm);
            write_quantized(out, plan, sm->view, sm->imatrix, pool, tm);
            const double wall = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            uint64_t elems = 0;
            for (auto &t : sm->view.tensors) elems += t.n_elements();
            printf("{\"model\": \"%s\", \"gpus\": %d, \"exact_errors\": %s, \"uniform\": \"%s\", \"elements\": %llu, "
                   "\"generate_s\": %.3f, \"measure_s\": %.3f, \"solve_s\": %.4f, \"setup_s\": %.3f, "
                   "\"encode_s\": %.3f, \"wall_s\": %.3f, \"plan_bytes\": %llu, \"budget_bytes\": %llu}\n",
                   synth_name.c_str(), pool.gpus(), a.exact_errors ? "true" : "false", a.uniform.c_str(),
                   (unsigned long long)elems, gen_s, tm.measure_s, tm.solve_s, tm.setup_s, tm.encode_s, wall,
                   (unsigned long long)plan.total_bytes, (unsigned long long)plan.budget.model_budget);
            return 0;
        }
    } catch (const std::exception &e) {
        fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    usage();
    return 2;
}
