// GGUF v2/v3 reader and streaming v3 writer (reference src/gguf.rs).
#pragma once
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <variant>
#include <vector>

namespace shh {

// ggml type ids (gguf.rs:13-83).
enum : uint32_t {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13,
    T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18, T_IQ4_NL = 20, T_IQ3_S = 21, T_IQ2_S = 22,
    T_IQ4_XS = 23, T_BF16 = 30
};

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// (elements per block, bytes per block); {1, 0} for unknown types (gguf.rs:86-107)
std::pair<uint64_t, uint64_t> block_layout(uint32_t ty);
// gguf.rs:109-113: throws on a ragged row like the reference's assert
uint64_t row_bytes(uint32_t ty, uint64_t n_per_row);
std::string type_name(uint32_t ty);
bool type_from_name(const std::string &name, uint32_t &ty);

// GGUF metadata value (gguf.rs:141-197)
struct Value {
    uint32_t type = 0;  // 0 U8, 1 I8, 2 U16, 3 I16, 4 U32, 5 I32, 6 F32, 7 Bool, 8 Str, 9 Arr, 10 U64, 11 I64, 12 F64
    uint64_t raw = 0;   // little-endian payload of scalar values, zero-extended
    std::string s;
    uint32_t elem_type = 0;  // for arrays
    std::vector<Value> arr;

    static Value U32(uint32_t v) { Value x; x.type = 4; x.raw = v; return x; }
    static Value Str(const std::string &v) { Value x; x.type = 8; x.s = v; return x; }
    bool operator==(const Value &o) const {
        return type == o.type && raw == o.raw && s == o.s && elem_type == o.elem_type && arr == o.arr;
    }
    bool as_u64(uint64_t &out) const;  // gguf.rs:159-171
    const std::string *as_str() const { return type == 8 ? &s : nullptr; }
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;  // dims[0] is the row length
    uint32_t ty = 0;
    uint64_t offset = 0;  // relative to the data section (absolute within its shard after Model::open)
    size_t shard = 0;
    uint64_t n_elements() const;
    uint64_t ne0() const { return dims.empty() ? 0 : dims[0]; }
    uint64_t n_rows() const;
    uint64_t byte_size() const { return row_bytes(ty, ne0()) * n_rows(); }
};

using KV = std::pair<std::string, Value>;

struct GgufFile {
    std::vector<KV> kvs;
    std::vector<TensorInfo> tensors;
    uint64_t data_start = 0;
    uint64_t alignment = 32;
};

// gguf.rs:379-421
GgufFile read_gguf(const uint8_t *buf, size_t len);

// A model on disk: one file or a llama.cpp split (-00001-of-0000N.gguf),
// memory-mapped (gguf.rs:244-325).
class Model {
  public:
    static std::unique_ptr<Model> open(const std::string &path);
    ~Model();
    const Value *kv(const std::string &key) const;
    const uint8_t *tensor_data(const TensorInfo &t) const;
    uint64_t total_bytes() const;
    std::vector<KV> kvs;
    std::vector<TensorInfo> tensors;
    uint64_t alignment = 32;

  private:
    struct Map {
        void *ptr = nullptr;
        size_t len = 0;
    };
    std::vector<Map> maps_;
};

std::vector<std::string> split_siblings(const std::string &path);

// Size of the header (magic .. tensor infos) the writer emits, and the
// aligned data offsets of each tensor (gguf.rs:476-483, 497-515).
struct Layout {
    uint64_t header_len = 0;
    uint64_t data_start = 0;
    std::vector<uint64_t> offsets;
    uint64_t total = 0;  // data_start + end of the last tensor
};
Layout layout_for(const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos, uint64_t alignment);

// Serialise the header into `out` (exactly layout.data_start bytes including
// the alignment padding).
std::vector<uint8_t> header_bytes(const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos, uint64_t alignment,
                                  const Layout &layout);

// gguf.rs:457-538 write_streaming: header, then produce(i) per tensor in
// order (size checked against the info), zero padding between tensors.
uint64_t write_streaming(const std::string &path, const std::vector<KV> &kvs, const std::vector<TensorInfo> &infos,
                         uint64_t alignment, const std::function<std::vector<uint8_t>(size_t)> &produce);

}  // namespace shh
