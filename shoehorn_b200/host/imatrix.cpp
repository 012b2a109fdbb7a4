// Imatrix loading (reference src/imatrix.rs:12-141).
#include "imatrix.hpp"

#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>

#include "gguf.hpp"

namespace shh {

Imatrix load_imatrix(const std::string &path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error("reading imatrix " + path);
    std::vector<uint8_t> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (buf.size() >= 4 && std::memcmp(buf.data(), "GGUF", 4) == 0) return load_imatrix_gguf(buf.data(), buf.size());
    return load_imatrix_legacy(buf.data(), buf.size());
}

static bool strip_suffix(const std::string &s, const char *suf, std::string &out) {
    const size_t n = std::strlen(suf);
    if (s.size() < n || s.compare(s.size() - n, n, suf) != 0) return false;
    out = s.substr(0, s.size() - n);
    return true;
}

Imatrix load_imatrix_gguf(const uint8_t *buf, size_t len) {
    const GgufFile f = read_gguf(buf, len);
    std::map<std::string, std::vector<float>> sums, counts;
    for (auto &t : f.tensors) {
        const uint64_t start = f.data_start + t.offset, n = t.byte_size();
        if (start + n > len) throw Error("imatrix tensor " + t.name + " extends past the end of the file");
        std::vector<float> vals((size_t)(n / 4));
        std::memcpy(vals.data(), buf + start, vals.size() * 4);
        std::string name;
        if (strip_suffix(t.name, ".in_sum2", name)) sums[name] = std::move(vals);
        else if (strip_suffix(t.name, ".counts", name)) counts[name] = std::move(vals);
    }
    if (sums.empty()) throw Error("GGUF imatrix contains no *.in_sum2 tensors");
    Imatrix out;
    for (auto &kv : sums) {
        std::vector<float> s = kv.second;
        auto c = counts.find(kv.first);
        if (c != counts.end() && !c->second.empty()) {
            const size_t clen = c->second.size();
            const size_t ratio = s.size() / std::max<size_t>(clen, 1);
            for (size_t i = 0; i < s.size(); i++) {
                const float cnt = c->second[std::min(i / std::max<size_t>(ratio, 1), clen - 1)];
                if (cnt > 0.0f) s[i] /= cnt;
            }
        }
        sanitize(s);
        out[kv.first] = std::move(s);
    }
    return out;
}

Imatrix load_imatrix_legacy(const uint8_t *buf, size_t len) {
    size_t pos = 0;
    auto rd_i32 = [&]() -> int32_t {
        if (pos + 4 > len) throw Error("legacy imatrix truncated at " + std::to_string(pos));
        int32_t v;
        std::memcpy(&v, buf + pos, 4);
        pos += 4;
        return v;
    };
    const int32_t n_entries = rd_i32();
    if (n_entries < 0 || n_entries >= 1000000)
        throw Error("implausible legacy imatrix entry count " + std::to_string(n_entries) + "; not an imatrix file?");
    Imatrix out;
    for (int32_t e = 0; e < n_entries; e++) {
        const int32_t name_len = rd_i32();
        if (name_len < 0 || pos + (size_t)name_len > len) throw Error("legacy imatrix truncated in name");
        std::string name(reinterpret_cast<const char *>(buf + pos), (size_t)name_len);
        pos += (size_t)name_len;
        const int32_t ncall = rd_i32();
        const int32_t nval = rd_i32();
        if (nval < 0 || pos + (size_t)nval * 4 > len) throw Error("legacy imatrix truncated in values for " + name);
        std::vector<float> vals((size_t)nval);
        std::memcpy(vals.data(), buf + pos, (size_t)nval * 4);
        pos += (size_t)nval * 4;
        if (ncall > 0)
            for (auto &v : vals) v /= (float)ncall;
        sanitize(vals);
        out[name] = std::move(vals);
    }
    return out;
}

void sanitize(std::vector<float> &vals) {
    float maxv = 0.0f;
    for (float v : vals)
        if (std::isfinite(v) && v > maxv) maxv = v;
    const float floor_v = maxv > 0.0f ? maxv * 1e-9f : 1.0f;
    for (auto &v : vals)
        if (!std::isfinite(v) || v <= 0.0f) v = floor_v;
}

const float *row_slice(const std::vector<float> *im, uint64_t ne0, uint64_t rows_per_mat, uint64_t row) {
    if (!im) return nullptr;
    if (im->size() == ne0) return im->data();
    if (rows_per_mat > 0 && ne0 > 0 && im->size() % ne0 == 0) {
        const uint64_t mat = row / rows_per_mat, n_mats = im->size() / ne0;
        const uint64_t m = std::min(mat, n_mats - 1);
        return im->data() + m * ne0;
    }
    return nullptr;
}

const std::vector<float> *lookup(const Imatrix &im, const std::string &name) {
    auto it = im.find(name);
    if (it != im.end()) return &it->second;
    std::string t = name;
    const std::string suf = ".weight";
    while (t.size() >= suf.size() && t.compare(t.size() - suf.size(), suf.size(), suf) == 0) t.resize(t.size() - suf.size());
    it = im.find(t);
    return it != im.end() ? &it->second : nullptr;
}

}  // namespace shh
