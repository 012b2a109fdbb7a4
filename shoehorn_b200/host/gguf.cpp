// GGUF v2/v3 reader and streaming v3 writer (reference src/gguf.rs:13-549).
#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>

namespace shh {

std::pair<uint64_t, uint64_t> block_layout(uint32_t t) {
    switch (t) {
    case T_F32: return {1, 4};
    case T_F16: case T_BF16: return {1, 2};
    case T_Q4_0: return {32, 18};
    case T_Q4_1: return {32, 20};
    case T_Q5_0: return {32, 22};
    case T_Q5_1: return {32, 24};
    case T_Q8_0: return {32, 34};
    case T_Q2_K: return {256, 84};
    case T_Q3_K: return {256, 110};
    case T_Q4_K: return {256, 144};
    case T_Q5_K: return {256, 176};
    case T_Q6_K: return {256, 210};
    case T_IQ2_XXS: return {256, 66};
    case T_IQ2_XS: return {256, 74};
    case T_IQ2_S: return {256, 82};
    case T_IQ3_XXS: return {256, 98};
    case T_IQ3_S: return {256, 110};
    case T_IQ4_NL: return {32, 18};
    case T_IQ4_XS: return {256, 136};
    default: return {1, 0};
    }
}

uint64_t row_bytes(uint32_t ty, uint64_t n) {
    auto [bs, tb] = block_layout(ty);
    if (n % bs != 0) throw Error("row size " + std::to_string(n) + " not divisible by block " + std::to_string(bs));
    return n / bs * tb;
}

static const struct { uint32_t ty; const char *name; } kNames[] = {
    {T_F32, "F32"}, {T_F16, "F16"}, {T_BF16, "BF16"}, {T_Q4_0, "Q4_0"}, {T_Q4_1, "Q4_1"}, {T_Q5_0, "Q5_0"},
    {T_Q5_1, "Q5_1"}, {T_Q8_0, "Q8_0"}, {T_Q2_K, "Q2_K"}, {T_Q3_K, "Q3_K"}, {T_Q4_K, "Q4_K"}, {T_Q5_K, "Q5_K"}, {T_Q6_K, "Q6_K"},
    {T_IQ2_XXS, "IQ2_XXS"}, {T_IQ2_XS, "IQ2_XS"}, {T_IQ2_S, "IQ2_S"}, {T_IQ3_XXS, "IQ3_XXS"}, {T_IQ3_S, "IQ3_S"},
    {T_IQ4_NL, "IQ4_NL"}, {T_IQ4_XS, "IQ4_XS"}};

std::string type_name(uint32_t ty) {
    for (auto &n : kNames)
        if (n.ty == ty) return n.name;
    return "type" + std::to_string(ty);
}

bool type_from_name(const std::string &name, uint32_t &ty) {
    for (auto &n : kNames)
        if (name == n.name) {
            ty = n.ty;
            return true;
        }
    return false;
}

bool Value::as_u64(uint64_t &out) const {
    switch (type) {
    case 0: case 2: case 4: case 10: out = raw; return true;
    case 1: if ((int8_t)raw >= 0) { out = (uint64_t)(int8_t)raw; return true; } return false;
    case 3: if ((int16_t)raw >= 0) { out = (uint64_t)(int16_t)raw; return true; } return false;
    case 5: if ((int32_t)raw >= 0) { out = (uint64_t)(int32_t)raw; return true; } return false;
    case 11: if ((int64_t)raw >= 0) { out = raw; return true; } return false;
    default: return false;
    }
}

uint64_t TensorInfo::n_elements() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
}
uint64_t TensorInfo::n_rows() const {
    uint64_t n = 1;
    for (size_t i = 1; i < dims.size(); i++) n *= dims[i];
    return n;
}

namespace {
int scalar_width(uint32_t ty) {
    switch (ty) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return -1;
    }
}

struct Reader {
    const uint8_t *buf;
    size_t len, pos = 0;
    const uint8_t *take(size_t n) {
        if (pos + n > len) throw Error("unexpected EOF at " + std::to_string(pos) + " (+" + std::to_string(n) + ")");
        const uint8_t *p = buf + pos;
        pos += n;
        return p;
    }
    uint64_t uint(int w) {
        const uint8_t *p = take((size_t)w);
        uint64_t v = 0;
        for (int i = 0; i < w; i++) v |= (uint64_t)p[i] << (8 * i);
        return v;
    }
    std::string str() {
        uint64_t n = uint(8);
        if (n > len) throw Error("string length out of range");
        const uint8_t *p = take((size_t)n);
        return std::string(reinterpret_cast<const char *>(p), (size_t)n);
    }
    Value value(uint32_t ty, int depth = 0) {
        if (depth > 8) throw Error("GGUF arrays nested too deeply");
        Value v;
        v.type = ty;
        if (ty == 8) {
            v.s = str();
        } else if (ty == 9) {
            v.elem_type = (uint32_t)uint(4);
            uint64_t count = uint(8);
            if (count > len) throw Error("array length out of range");
            v.arr.reserve((size_t)std::min<uint64_t>(count, 1u << 24));
            for (uint64_t i = 0; i < count; i++) v.arr.push_back(value(v.elem_type, depth + 1));
        } else {
            const int w = scalar_width(ty);
            if (w < 0) throw Error("unknown GGUF value type " + std::to_string(ty));
            v.raw = uint(w);
        }
        return v;
    }
};

struct Writer {
    std::vector<uint8_t> &out;
    void uint(uint64_t v, int w) {
        for (int i = 0; i < w; i++) out.push_back((uint8_t)(v >> (8 * i)));
    }
    void str(const std::string &s) {
        uint(s.size(), 8);
        out.insert(out.end(), s.begin(), s.end());
    }
    void value(const Value &v) {
        if (v.type == 8) {
            str(v.s);
        } else if (v.type == 9) {
            uint(v.elem_type, 4);
            uint(v.arr.size(), 8);
            for (auto &e : v.arr) value(e);
        } else {
            uint(v.raw, scalar_width(v.type));
        }
    }
};
}  // namespace

GgufFile read_gguf(const uint8_t *buf, size_t len) {
    Reader r{buf, len};
    const uint32_t magic = (uint32_t)r.uint(4);
    if (magic != 0x46554747u) {
        char m[32];
        snprintf(m, sizeof m, "%#x", magic);
        throw Error(std::string("not a GGUF file (magic ") + m + ")");
    }
    const uint32_t version = (uint32_t)r.uint(4);
    if (version < 2 || version > 3) throw Error("unsupported GGUF version " + std::to_string(version));
    const uint64_t n_tensors = r.uint(8), n_kv = r.uint(8);
    if (n_tensors > len || n_kv > len) throw Error("implausible GGUF header counts");
    GgufFile f;
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key = r.str();
        const uint32_t ty = (uint32_t)r.uint(4);
        try {
            f.kvs.emplace_back(key, r.value(ty));
        } catch (const Error &e) {
            throw Error("reading value for key " + key + ": " + e.what());
        }
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
        TensorInfo t;
        t.name = r.str();
        const uint32_t nd = (uint32_t)r.uint(4);
        if (nd > 8) throw Error("tensor " + t.name + " has " + std::to_string(nd) + " dims");
        for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.uint(8));
        t.ty = (uint32_t)r.uint(4);
        t.offset = r.uint(8);
        f.tensors.push_back(std::move(t));
    }
    f.alignment = 32;
    for (auto &kv : f.kvs)
        if (kv.first == "general.alignment") {
            uint64_t a;
            if (kv.second.as_u64(a)) f.alignment = a;
            break;
        }
    if (f.alignment == 0) throw Error("general.alignment is zero");
    f.data_start = (r.pos + f.alignment - 1) / f.alignment * f.alignment;
    return f;
}

std::vector<std::string> split_siblings(const std::string &path) {
    const size_t slash = path.find_last_of('/');
    const std::string dir = slash == std::string::npos ? "" : path.substr(0, slash + 1);
    const std::string name = slash == std::string::npos ? path : path.substr(slash + 1);
    auto single = std::vector<std::string>{path};
    if (name.size() < 5 || name.compare(name.size() - 5, 5, ".gguf") != 0) return single;
    const std::string base = name.substr(0, name.size() - 5);
    const size_t of = base.rfind("-of-");
    if (of == std::string::npos) return single;
    const std::string head = base.substr(0, of), count_s = base.substr(of + 4);
    const size_t dash = head.rfind('-');
    if (dash == std::string::npos) return single;
    const std::string stem = head.substr(0, dash), no_s = head.substr(dash + 1);
    auto digits = [](const std::string &x) {
        if (x.size() != 5) return false;
        for (char c : x)
            if (c < '0' || c > '9') return false;
        return true;
    };
    if (!digits(no_s) || !digits(count_s)) return single;
    const int no = std::stoi(no_s), count = std::stoi(count_s);
    if (count <= 1) return single;
    if (no != 1) {
        char b[96];
        snprintf(b, sizeof b, "open the first shard of a split model (...-00001-of-%05d.gguf)", count);
        throw Error(b);
    }
    std::vector<std::string> out;
    for (int i = 1; i <= count; i++) {
        char b[32];
        snprintf(b, sizeof b, "-%05d-of-%05d.gguf", i, count);
        std::string p = dir + stem + b;
        struct stat st;
        if (stat(p.c_str(), &st) != 0) throw Error("missing shard " + p);
        out.push_back(p);
    }
    return out;
}

std::unique_ptr<Model> Model::open(const std::string &path) {
    auto m = std::unique_ptr<Model>(new Model());
    const auto paths = split_siblings(path);
    for (size_t si = 0; si < paths.size(); si++) {
        const int fd = ::open(paths[si].c_str(), O_RDONLY);
        if (fd < 0) throw Error("opening " + paths[si]);
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            throw Error("stat " + paths[si]);
        }
        Map mp;
        mp.len = (size_t)st.st_size;
        mp.ptr = mp.len ? mmap(nullptr, mp.len, PROT_READ, MAP_SHARED, fd, 0) : nullptr;
        ::close(fd);
        if (mp.len && mp.ptr == MAP_FAILED) throw Error("mmap " + paths[si]);
        m->maps_.push_back(mp);
        GgufFile g;
        try {
            g = read_gguf(static_cast<const uint8_t *>(mp.ptr), mp.len);
        } catch (const Error &e) {
            throw Error("parsing " + paths[si] + ": " + e.what());
        }
        if (si == 0) {
            m->kvs = g.kvs;
            m->alignment = g.alignment;
        }
        for (auto &t : g.tensors) {
            t.offset += g.data_start;
            t.shard = si;
            if (t.offset + t.byte_size() > mp.len) throw Error("tensor " + t.name + " extends past the end of its file");
            m->tensors.push_back(t);
        }
    }
    if (paths.size() > 1)
        fprintf(stderr, "opened split model: %zu shards, %zu tensors\n", paths.size(), m->tensors.size());
    return m;
}

Model::~Model() {
    for (auto &mp : maps_)
        if (mp.ptr && mp.len) munmap(mp.ptr, mp.len);
}

const Value *Model::kv(const std::string &key) const {
    for (auto &p : kvs)
        if (p.first == key) return &p.second;
    return nullptr;
}

const uint8_t *Model::tensor_data(const TensorInfo &t) const {
    return static_cast<const uint8_t *>(maps_[t.shard].ptr) + t.offset;
}

uint64_t Model::total_bytes() const {
    uint64_t n = 0;
    for (auto &mp : maps_) n += mp.len;
    return n;
}

Layout layout_for(const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos, uint64_t alignment) {
    Layout L;
    std::vector<uint8_t> tmp;
    Writer w{tmp};
    uint64_t hdr = 4 + 4 + 8 + 8;
    for (auto &kv : kvs) {
        tmp.clear();
        w.str(kv.first);
        w.uint(kv.second.type, 4);
        w.value(kv.second);
        hdr += tmp.size();
    }
    for (auto &t : infos) hdr += 8 + t.name.size() + 4 + 8 * t.dims.size() + 4 + 8;
    L.header_len = hdr;
    L.data_start = (hdr + alignment - 1) / alignment * alignment;
    uint64_t off = 0;
    for (auto &t : infos) {
        off = (off + alignment - 1) / alignment * alignment;
        L.offsets.push_back(off);
        off += t.byte_size();
    }
    L.total = L.data_start + off;
    return L;
}

std::vector<uint8_t> header_bytes(const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos, uint64_t alignment,
                                  const Layout &L) {
    (void)alignment;
    std::vector<uint8_t> out;
    Writer w{out};
    w.uint(0x46554747u, 4);
    w.uint(3, 4);
    w.uint(infos.size(), 8);
    w.uint(kvs.size(), 8);
    for (auto &kv : kvs) {
        w.str(kv.first);
        w.uint(kv.second.type, 4);
        w.value(kv.second);
    }
    for (size_t i = 0; i < infos.size(); i++) {
        w.str(infos[i].name);
        w.uint(infos[i].dims.size(), 4);
        for (auto d : infos[i].dims) w.uint(d, 8);
        w.uint(infos[i].ty, 4);
        w.uint(L.offsets[i], 8);
    }
    out.resize(L.data_start, 0);
    return out;
}

uint64_t write_streaming(const std::string &path, const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos,
                         uint64_t alignment, const std::function<std::vector<uint8_t>(size_t)> &produce) {
    const Layout L = layout_for(kvs, infos, alignment);
    FILE *f = fopen(path.c_str(), "wb");
    if (!f) throw Error("creating " + path);
    std::vector<char> iobuf(1 << 20);
    setvbuf(f, iobuf.data(), _IOFBF, iobuf.size());
    auto put = [&](const void *p, size_t n) {
        if (n && fwrite(p, 1, n, f) != n) {
            fclose(f);
            throw Error("writing " + path);
        }
    };
    const auto hdr = header_bytes(kvs, infos, alignment, L);
    put(hdr.data(), hdr.size());
    uint64_t pos = 0;
    std::vector<uint8_t> zeros;
    for (size_t i = 0; i < infos.size(); i++) {
        if (L.offsets[i] > pos) {
            zeros.assign((size_t)(L.offsets[i] - pos), 0);
            put(zeros.data(), zeros.size());
            pos = L.offsets[i];
        }
        const auto data = produce(i);
        if (data.size() != infos[i].byte_size()) {
            fclose(f);
            throw Error("tensor " + infos[i].name + " data size mismatch: " + std::to_string(data.size()) + " vs " +
                        std::to_string(infos[i].byte_size()));
        }
        put(data.data(), data.size());
        pos += data.size();
    }
    if (fclose(f) != 0) throw Error("closing " + path);
    return L.data_start + pos;
}

}  // namespace shh
