// C ABI of the host library (libshoehorn_host.so): the reference's host-side
// pieces that tests and other hosts call directly.
#include <cstring>

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

}  // extern "C"
