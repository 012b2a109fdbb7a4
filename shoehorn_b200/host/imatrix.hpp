// Imatrix loading (reference src/imatrix.rs): legacy binary and GGUF formats.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace shh {

using Imatrix = std::map<std::string, std::vector<float>>;

Imatrix load_imatrix(const std::string &path);                    // imatrix.rs:12-19
Imatrix load_imatrix_gguf(const uint8_t *buf, size_t len);         // imatrix.rs:23-59
Imatrix load_imatrix_legacy(const uint8_t *buf, size_t len);       // imatrix.rs:63-104
void sanitize(std::vector<float> &vals);                           // imatrix.rs:107-120
// imatrix.rs:124-141: nullptr means "no imatrix" for this row
const float *row_slice(const std::vector<float> *im, uint64_t ne0, uint64_t rows_per_mat, uint64_t row);
// main.rs:538-544 lookup: exact name, then the name with ".weight" trimmed
const std::vector<float> *lookup(const Imatrix &im, const std::string &tensor_name);

}  // namespace shh
