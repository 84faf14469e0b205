// GGUF v3 reader for the CUDA host runtime: mmap + header/metadata/tensor-info
// parse with the same validity rules as the reference's loader
// (src/parsing/gguf.cpp:145-242, src/base/config.cpp:171-255): magic "GGUF",
// version 3, non-zero tensor and metadata counts, lower_snake_case dotted keys,
// `general.alignment` (default 32), tensor types F32/F16/BF16 only, 1..4
// non-zero dims, data inside the file. Tensor data stays in the mapping.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <variant>
#include <vector>

namespace minfer {

enum class DataType : int { F32 = 0, F16 = 1, BF16 = 2, INVALID = -1 };

size_t dtype_size(DataType t);
const char* dtype_name(DataType t);

struct MetaValue {
    // scalars are widened; arrays of numbers / strings are kept as vectors
    enum Kind { UINT, INT, FLOAT, BOOL, STRING, ARRAY_NUM, ARRAY_STR } kind = UINT;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    bool b = false;
    std::string s;
    std::vector<double> nums;
    std::vector<std::string> strs;
};

struct TensorView {
    std::string name;
    DataType dtype = DataType::INVALID;
    std::vector<uint64_t> ne;        // GGUF order: innermost first
    std::vector<uint64_t> shape;     // logical: outermost first
    const uint8_t* data = nullptr;   // inside the mapping
    size_t bytes = 0;
    size_t numel = 0;
};

class GGUFFile {
public:
    GGUFFile() = default;
    ~GGUFFile();
    GGUFFile(const GGUFFile&) = delete;
    GGUFFile& operator=(const GGUFFile&) = delete;

    // Returns 0 on success, -1 with `error()` set otherwise.
    int open(const std::string& path);
    const std::string& error() const { return err_; }

    bool has(const std::string& key) const { return meta_.count(key) != 0; }
    const MetaValue* get(const std::string& key) const;
    uint64_t get_uint(const std::string& key) const;  // throws std::runtime_error if missing
    double get_float(const std::string& key) const;
    const std::string& get_string(const std::string& key) const;

    bool has_tensor(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorView& tensor(const std::string& name) const;  // throws if missing
    const std::map<std::string, TensorView>& tensors() const { return tensors_; }
    size_t file_size() const { return size_; }

private:
    int fail(const std::string& m);
    std::string err_;
    void* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, MetaValue> meta_;
    std::map<std::string, TensorView> tensors_;
};

}  // namespace minfer
