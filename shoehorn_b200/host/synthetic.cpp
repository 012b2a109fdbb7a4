// Synthetic models of the benchmark configurations: BF16 weights drawn from
// a counter-based generator (seeded per tensor, so any tensor can be
// regenerated alone), F32 norms of 1.0, and a per-column log-normal imatrix.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "pipeline.hpp"

namespace shh {

HostBuffer::HostBuffer(size_t bytes) : n(bytes) {
    if (cudaMallocHost((void **)&ptr, bytes ? bytes : 1) == cudaSuccess) {
        pinned = true;
    } else {
        cudaGetLastError();
        ptr = static_cast<uint8_t *>(malloc(bytes ? bytes : 1));
        if (!ptr) throw Error("host allocation failed");
    }
}
HostBuffer::~HostBuffer() {
    if (pinned) cudaFreeHost(ptr);
    else free(ptr);
}

namespace {
inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
// Standard normal quantiles z_k = Phi^-1(p_k) at p_k = (k + 1/2) / kIcdfBins
// for k = -1 .. kIcdfBins (the two outer points extrapolate the first and
// last bins), found by bisection on Phi(z) = erfc(-z / sqrt 2) / 2.  A
// uniform u in [0, 1) maps to z by linear interpolation between the two
// quantiles around it: a table sampler of N(0, 1) to within ~1e-4 in z,
// several times faster than Box-Muller, so synthetic models of 70 B
// weights can be generated as they stream.
constexpr int kIcdfBins = 4096;
struct IcdfTable {
    float z[kIcdfBins + 2];
    IcdfTable() {
        for (int k = -1; k <= kIcdfBins; k++) {
            const double p = ((double)k + 0.5) / kIcdfBins;
            double lo = -10.0, hi = 10.0;
            for (int it = 0; it < 100; it++) {
                const double mid = 0.5 * (lo + hi);
                if (0.5 * std::erfc(-mid / std::sqrt(2.0)) < p) lo = mid;
                else hi = mid;
            }
            z[k + 1] = (float)(0.5 * (lo + hi));
        }
    }
};
const IcdfTable &icdf() {
    static const IcdfTable t;
    return t;
}
inline float normal_of(const IcdfTable &t, uint32_t u24) {  // u24: 24 uniform bits
    const float f = (float)u24 * ((float)kIcdfBins / 16777216.0f) + 0.5f;  // in [0.5, kIcdfBins + 0.5)
    const int k = (int)f;                                                   // f >= 0: truncation is floor
    const float a = t.z[k], b = t.z[k + 1];
    return a + (f - (float)k) * (b - a);
}
// Two standard normals for counter p of stream `key`.
inline void normal2(uint64_t key, uint64_t p, float &z0, float &z1) {
    const IcdfTable &t = icdf();
    const uint64_t r = splitmix64(key ^ (p * 0xD1B54A32D192ED03ull));
    z0 = normal_of(t, (uint32_t)(r >> 40));
    z1 = normal_of(t, (uint32_t)(r & 0xFFFFFFu));
}
inline uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return (uint16_t)((u + 0x7FFF + ((u >> 16) & 1)) >> 16);
}

struct Spec {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t ty;
};

// The weights of a spec tensor: N(0, stdv) BF16 from stream seed + index.
struct ModelSpec {
    std::vector<KV> kvs;
    std::vector<Spec> specs;
    float stdv = 0.02f;
    bool boost = false;  // 1% of imatrix columns x100
};

// Elements [e0, e0 + n) of a tensor whose element pair p is normal2(key, p):
// any range of rows can be generated alone and equals the same rows of the
// whole tensor (e0 even).
void fill_normal_bf16(uint8_t *dst, uint64_t e0, uint64_t n, uint64_t key, float stdv, int threads) {
    uint16_t *o = reinterpret_cast<uint16_t *>(dst);
    const uint64_t p0 = e0 / 2, pairs = (n + 1) / 2;
    auto part = [=](int t, int nt) {
        const uint64_t a = pairs * (uint64_t)t / (uint64_t)nt, b = pairs * (uint64_t)(t + 1) / (uint64_t)nt;
        for (uint64_t p = a; p < b; p++) {
            float z0, z1;
            normal2(key, p0 + p, z0, z1);
            o[2 * p] = to_bf16(z0 * stdv);
            if (2 * p + 1 < n) o[2 * p + 1] = to_bf16(z1 * stdv);
        }
    };
    if (threads <= 1) {
        part(0, 1);
        return;
    }
    std::vector<std::thread> th;
    for (int t = 0; t < threads; t++) th.emplace_back(part, t, threads);
    for (auto &x : th) x.join();
}
}  // namespace

// The reference's end-to-end fixture (e2e_tests.rs:10-67): five tensors,
// BF16 rows from a 64-bit LCG seeded tensor index + 1, F32 from seed 99.
static std::unique_ptr<SyntheticModel> e2e_model() {
    auto sm = std::make_unique<SyntheticModel>();
    auto &v = sm->view;
    v.kvs.emplace_back("general.architecture", Value::Str("llama"));
    v.kvs.emplace_back("llama.block_count", Value::U32(2));
    v.kvs.emplace_back("llama.embedding_length", Value::U32(256));
    v.kvs.emplace_back("llama.attention.head_count", Value::U32(4));
    v.kvs.emplace_back("llama.attention.head_count_kv", Value::U32(2));
    v.kvs.emplace_back("llama.vocab_size", Value::U32(256));
    const std::vector<Spec> specs = {{"token_embd.weight", {256, 128}, T_BF16},
                                     {"blk.0.attn_q.weight", {256, 256}, T_BF16},
                                     {"blk.0.ffn_down.weight", {256, 64}, T_BF16},
                                     {"blk.1.attn_q.weight", {256, 256}, T_BF16},
                                     {"output_norm.weight", {256}, T_F32}};
    for (size_t i = 0; i < specs.size(); i++) {
        TensorInfo t;
        t.name = specs[i].name;
        t.dims = specs[i].dims;
        t.ty = specs[i].ty;
        auto buf = std::make_unique<HostBuffer>((size_t)t.byte_size());
        uint64_t st = t.ty == T_BF16 ? (uint64_t)i + 1 : 99;
        auto next = [&]() {
            st = st * 6364136223846793005ull + 1442695040888963407ull;
            return (float)(st >> 33) / (float)(1ull << 31) - 0.5f;
        };
        for (uint64_t e = 0; e < t.n_elements(); e++) {
            if (t.ty == T_BF16) {
                const uint16_t b = to_bf16(next());
                std::memcpy(buf->ptr + 2 * e, &b, 2);
            } else {
                const float f = next();
                std::memcpy(buf->ptr + 4 * e, &f, 4);
            }
        }
        v.tensors.push_back(t);
        v.total_bytes += t.byte_size();
        sm->storage.push_back(std::move(buf));
    }
    SyntheticModel *raw = sm.get();
    v.data = [raw](size_t i) { return (const uint8_t *)raw->storage[i]->ptr; };
    return sm;
}

static ModelSpec model_spec(const std::string &name) {
    ModelSpec ms;
    auto &specs = ms.specs;
    std::string arch;
    uint64_t n_layer, n_embd, n_head, n_kv, head_dim, n_ff, n_vocab, ctx_len;
    bool tied, qk_norm;
    if (name == "qwen3-0.6b") {
        arch = "qwen3"; n_layer = 28; n_embd = 1024; n_head = 16; n_kv = 8; head_dim = 128; n_ff = 3072;
        n_vocab = 151936; ctx_len = 40960; tied = true; qk_norm = true;
    } else if (name == "llama3-8b") {
        arch = "llama"; n_layer = 32; n_embd = 4096; n_head = 32; n_kv = 8; head_dim = 128; n_ff = 14336;
        n_vocab = 128256; ctx_len = 8192; tied = false; qk_norm = false;
    } else if (name == "llama3-70b") {
        arch = "llama"; n_layer = 80; n_embd = 8192; n_head = 64; n_kv = 8; head_dim = 128; n_ff = 28672;
        n_vocab = 128256; ctx_len = 8192; tied = false; qk_norm = false; ms.stdv = 0.015f; ms.boost = true;
    } else if (name == "tiny") {  // e2e_tests.rs:28-67 shapes
        arch = "llama"; n_layer = 2; n_embd = 256; n_head = 4; n_kv = 2; head_dim = 64; n_ff = 64;
        n_vocab = 256; ctx_len = 2048; tied = false; qk_norm = false;
    } else {
        throw Error("unknown synthetic model " + name + " (qwen3-0.6b, llama3-8b, llama3-70b, tiny, e2e)");
    }
    const uint64_t q_out = n_head * head_dim, kv_out = n_kv * head_dim;
    specs.push_back({"token_embd.weight", {n_embd, n_vocab}, T_BF16});
    for (uint64_t l = 0; l < n_layer; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        specs.push_back({p + "attn_norm.weight", {n_embd}, T_F32});
        specs.push_back({p + "attn_q.weight", {n_embd, q_out}, T_BF16});
        specs.push_back({p + "attn_k.weight", {n_embd, kv_out}, T_BF16});
        specs.push_back({p + "attn_v.weight", {n_embd, kv_out}, T_BF16});
        specs.push_back({p + "attn_output.weight", {q_out, n_embd}, T_BF16});
        if (qk_norm) {
            specs.push_back({p + "attn_q_norm.weight", {head_dim}, T_F32});
            specs.push_back({p + "attn_k_norm.weight", {head_dim}, T_F32});
        }
        specs.push_back({p + "ffn_norm.weight", {n_embd}, T_F32});
        specs.push_back({p + "ffn_gate.weight", {n_embd, n_ff}, T_BF16});
        specs.push_back({p + "ffn_up.weight", {n_embd, n_ff}, T_BF16});
        specs.push_back({p + "ffn_down.weight", {n_ff, n_embd}, T_BF16});
    }
    specs.push_back({"output_norm.weight", {n_embd}, T_F32});
    if (!tied) specs.push_back({"output.weight", {n_embd, n_vocab}, T_BF16});

    auto &kv = ms.kvs;
    kv.emplace_back("general.architecture", Value::Str(arch));
    kv.emplace_back("general.name", Value::Str("synthetic " + name));
    kv.emplace_back(arch + ".block_count", Value::U32((uint32_t)n_layer));
    kv.emplace_back(arch + ".context_length", Value::U32((uint32_t)ctx_len));
    kv.emplace_back(arch + ".embedding_length", Value::U32((uint32_t)n_embd));
    kv.emplace_back(arch + ".feed_forward_length", Value::U32((uint32_t)n_ff));
    kv.emplace_back(arch + ".attention.head_count", Value::U32((uint32_t)n_head));
    kv.emplace_back(arch + ".attention.head_count_kv", Value::U32((uint32_t)n_kv));
    kv.emplace_back(arch + ".attention.key_length", Value::U32((uint32_t)head_dim));
    kv.emplace_back(arch + ".attention.value_length", Value::U32((uint32_t)head_dim));
    kv.emplace_back(arch + ".vocab_size", Value::U32((uint32_t)n_vocab));
    kv.emplace_back("general.file_type", Value::U32(32));  // MOSTLY_BF16
    return ms;
}

// Per-column importance exp(N(0,1)) of a 2-D tensor (1% of columns x100
// with boost); token_embd gets none (real imatrices never cover it).
static void add_imatrix(SyntheticModel &sm, const TensorInfo &t, size_t i, uint64_t seed, bool boost) {
    if (t.ty == T_F32 || t.name == "token_embd.weight" || t.dims.size() != 2) return;
    std::vector<float> im((size_t)t.ne0());
    const uint64_t key = splitmix64(seed ^ 0x1A7B1C00ull ^ i);
    for (uint64_t c = 0; c < t.ne0(); c += 2) {
        float z0, z1;
        normal2(key, c / 2, z0, z1);
        im[(size_t)c] = std::exp(z0);
        if (c + 1 < t.ne0()) im[(size_t)c + 1] = std::exp(z1);
    }
    if (boost)
        for (uint64_t c = 0; c < t.ne0(); c++)
            if (splitmix64(key + 7919 * c) % 100 == 0) im[(size_t)c] *= 100.0f;
    sm.imatrix[t.name.substr(0, t.name.size() - 7)] = std::move(im);  // imatrix entries drop ".weight"
}

std::unique_ptr<SyntheticModel> synthetic_model(const std::string &name, uint64_t seed, int threads, int rank,
                                                int world) {
    if (name == "e2e") {
        if (world > 1) throw Error("the e2e fixture is not generated in shards");
        return e2e_model();
    }
    const ModelSpec ms = model_spec(name);
    auto sm = std::make_unique<SyntheticModel>();
    auto &v = sm->view;
    v.kvs = ms.kvs;
    v.alignment = 32;
    for (size_t i = 0; i < ms.specs.size(); i++) {
        TensorInfo t;
        t.name = ms.specs[i].name;
        t.dims = ms.specs[i].dims;
        t.ty = ms.specs[i].ty;
        uint64_t lo, hi;  // the rows this rank holds
        shard_rows(t.n_rows(), rank, world, lo, hi);
        v.row_lo.push_back(lo);
        const uint64_t rb = row_bytes(t.ty, t.ne0());
        auto buf = std::make_unique<HostBuffer>((size_t)((hi - lo) * rb));
        if (t.ty == T_F32) {
            float *f = reinterpret_cast<float *>(buf->ptr);
            for (uint64_t e = 0; e < (hi - lo) * t.ne0(); e++) f[e] = 1.0f;
        } else {
            fill_normal_bf16(buf->ptr, lo * t.ne0(), (hi - lo) * t.ne0(), seed + i, ms.stdv, threads);
        }
        add_imatrix(*sm, t, i, seed, ms.boost);
        v.tensors.push_back(t);
        v.total_bytes += t.byte_size();
        sm->storage.push_back(std::move(buf));
    }
    SyntheticModel *raw = sm.get();
    v.data = [raw](size_t i) { return (const uint8_t *)raw->storage[i]->ptr; };
    return sm;
}

std::unique_ptr<SyntheticModel> synthetic_model_streaming(const std::string &name, uint64_t seed) {
    if (name == "e2e") throw Error("the e2e fixture is not streamed");
    const ModelSpec ms = model_spec(name);
    auto sm = std::make_unique<SyntheticModel>();
    auto &v = sm->view;
    v.kvs = ms.kvs;
    v.alignment = 32;
    for (size_t i = 0; i < ms.specs.size(); i++) {
        TensorInfo t;
        t.name = ms.specs[i].name;
        t.dims = ms.specs[i].dims;
        t.ty = ms.specs[i].ty;
        add_imatrix(*sm, t, i, seed, ms.boost);
        v.tensors.push_back(t);
        v.total_bytes += t.byte_size();
    }
    const float stdv = ms.stdv;
    SyntheticModel *raw = sm.get();
    v.fill = [raw, seed, stdv](size_t i, uint64_t r0, uint64_t n, uint64_t step, uint8_t *dst) {
        const TensorInfo &t = raw->view.tensors[i];
        const uint64_t ne0 = t.ne0(), rb = row_bytes(t.ty, ne0);
        if (t.ty == T_F32) {
            for (uint64_t k = 0; k < n; k++) {
                float *f = reinterpret_cast<float *>(dst + k * rb);
                for (uint64_t e = 0; e < ne0; e++) f[e] = 1.0f;
            }
            return;
        }
        // large requests are split over a few threads (the pipeline's
        // workers already run one request each)
        const int nt = n * ne0 >= (4u << 20) ? 4 : 1;
        std::vector<std::thread> th;
        for (int tt = 0; tt < nt; tt++)
            th.emplace_back([=]() {
                for (uint64_t k = n * (uint64_t)tt / (uint64_t)nt; k < n * (uint64_t)(tt + 1) / (uint64_t)nt; k++)
                    fill_normal_bf16(dst + k * rb, (r0 + k * step) * ne0, ne0, seed + i, stdv, 1);
            });
        for (auto &x : th) x.join();
    };
    return sm;
}

}  // namespace shh
