#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace minfer {

size_t dtype_size(DataType t) {
    switch (t) {
        case DataType::F32: return 4;
        case DataType::F16: return 2;
        case DataType::BF16: return 2;
        default: return 0;
    }
}

const char* dtype_name(DataType t) {
    switch (t) {
        case DataType::F32: return "F32";
        case DataType::F16: return "F16";
        case DataType::BF16: return "BF16";
        default: return "INVALID";
    }
}

namespace {

// GGUF value type codes (include/minfer/parsing/gguf.hpp ValueType)
enum : uint32_t { T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    size_t file_size;

    void need(size_t n) {
        if ((size_t)(end - p) < n) throw std::runtime_error("read past the end of the file");
    }
    template <typename T>
    T rd() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = rd<uint64_t>();
        if (n > file_size) throw std::runtime_error("string length larger than the file");
        need(n);
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

bool valid_key(const std::string& k) {
    // lower_snake_case segments separated by single dots, ASCII, < 65536 bytes
    if (k.empty() || k.size() > 65535) return false;
    bool seg_start = true;
    for (char c : k) {
        if (c == '.') {
            if (seg_start) return false;
            seg_start = true;
            continue;
        }
        const bool ok = (c >= 'a' && c <= 'z') || (c >= '0' && c <= '9') || c == '_';
        if (!ok) return false;
        seg_start = false;
    }
    return !seg_start;
}

double num_of(Cursor& c, uint32_t t, MetaValue& mv, bool scalar) {
    switch (t) {
        case T_U8: { auto v = c.rd<uint8_t>(); if (scalar) { mv.kind = MetaValue::UINT; mv.u = v; } return v; }
        case T_I8: { auto v = c.rd<int8_t>(); if (scalar) { mv.kind = MetaValue::INT; mv.i = v; } return v; }
        case T_U16: { auto v = c.rd<uint16_t>(); if (scalar) { mv.kind = MetaValue::UINT; mv.u = v; } return v; }
        case T_I16: { auto v = c.rd<int16_t>(); if (scalar) { mv.kind = MetaValue::INT; mv.i = v; } return v; }
        case T_U32: { auto v = c.rd<uint32_t>(); if (scalar) { mv.kind = MetaValue::UINT; mv.u = v; } return v; }
        case T_I32: { auto v = c.rd<int32_t>(); if (scalar) { mv.kind = MetaValue::INT; mv.i = v; } return v; }
        case T_F32: { auto v = c.rd<float>(); if (scalar) { mv.kind = MetaValue::FLOAT; mv.f = v; } return v; }
        case T_U64: { auto v = c.rd<uint64_t>(); if (scalar) { mv.kind = MetaValue::UINT; mv.u = v; } return (double)v; }
        case T_I64: { auto v = c.rd<int64_t>(); if (scalar) { mv.kind = MetaValue::INT; mv.i = v; } return (double)v; }
        case T_F64: { auto v = c.rd<double>(); if (scalar) { mv.kind = MetaValue::FLOAT; mv.f = v; } return v; }
        case T_BOOL: { auto v = c.rd<uint8_t>(); if (scalar) { mv.kind = MetaValue::BOOL; mv.b = v != 0; } return v; }
        default: throw std::runtime_error("invalid metadata value type");
    }
}

void read_value(Cursor& c, uint32_t t, MetaValue& mv, int depth) {
    if (t == T_STR) {
        mv.kind = MetaValue::STRING;
        mv.s = c.str();
        return;
    }
    if (t == T_ARR) {
        if (depth > 4) throw std::runtime_error("nested arrays too deep");
        const uint32_t et = c.rd<uint32_t>();
        const uint64_t n = c.rd<uint64_t>();
        if (n > c.file_size) throw std::runtime_error("array length larger than the file");
        if (et == T_STR) {
            mv.kind = MetaValue::ARRAY_STR;
            mv.strs.reserve(n);
            for (uint64_t k = 0; k < n; ++k) mv.strs.push_back(c.str());
        } else if (et == T_ARR) {
            MetaValue sub;  // nested arrays are parsed and dropped
            for (uint64_t k = 0; k < n; ++k) read_value(c, et, sub, depth + 1);
            mv.kind = MetaValue::ARRAY_NUM;
        } else {
            mv.kind = MetaValue::ARRAY_NUM;
            mv.nums.reserve(n);
            MetaValue dummy;
            for (uint64_t k = 0; k < n; ++k) mv.nums.push_back(num_of(c, et, dummy, false));
        }
        return;
    }
    num_of(c, t, mv, true);
}

}  // namespace

GGUFFile::~GGUFFile() {
    if (map_) munmap(map_, size_);
}

int GGUFFile::fail(const std::string& m) {
    err_ = m;
    return -1;
}

int GGUFFile::open(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail("cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        return fail("cannot stat " + path);
    }
    size_ = (size_t)st.st_size;
    if (size_ < 24) {
        ::close(fd);
        return fail("file too small to be GGUF");
    }
    map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) {
        map_ = nullptr;
        return fail("mmap failed for " + path);
    }
    const uint8_t* base = static_cast<const uint8_t*>(map_);
    Cursor c{base, base + size_, size_};
    try {
        const uint32_t magic = c.rd<uint32_t>();
        const uint32_t version = c.rd<uint32_t>();
        const uint64_t n_tensors = c.rd<uint64_t>();
        const uint64_t n_kv = c.rd<uint64_t>();
        if (magic != 0x46554747u) return fail("bad magic (not a GGUF file)");
        if (version != 3) return fail("only GGUF version 3 is supported (file has " + std::to_string(version) + ")");
        if (n_tensors == 0 || n_kv == 0) return fail("tensor count or metadata count is zero");
        if (n_tensors > size_ || n_kv > size_) return fail("counts larger than the file");
        for (uint64_t k = 0; k < n_kv; ++k) {
            std::string key = c.str();
            if (!valid_key(key)) return fail("invalid metadata key: " + key);
            const uint32_t t = c.rd<uint32_t>();
            MetaValue mv;
            read_value(c, t, mv, 0);
            meta_[key] = std::move(mv);
        }
        struct Info {
            std::string name;
            std::vector<uint64_t> ne;
            uint32_t type;
            uint64_t off;
        };
        std::vector<Info> infos;
        infos.reserve(n_tensors);
        for (uint64_t k = 0; k < n_tensors; ++k) {
            Info in;
            in.name = c.str();
            const uint32_t nd = c.rd<uint32_t>();
            if (nd == 0 || nd > 4) return fail("tensor " + in.name + " has 0 or more than 4 dimensions");
            for (uint32_t d = 0; d < nd; ++d) in.ne.push_back(c.rd<uint64_t>());
            in.type = c.rd<uint32_t>();
            in.off = c.rd<uint64_t>();
            infos.push_back(std::move(in));
        }
        uint64_t align = 32;
        auto it = meta_.find("general.alignment");
        if (it != meta_.end() && it->second.kind == MetaValue::UINT && it->second.u > 0) align = it->second.u;
        const uint64_t pos = (uint64_t)(c.p - base);
        const uint64_t data0 = pos + (align - pos % align) % align;
        if (data0 > size_) return fail("tensor data starts past the end of the file");
        const uint64_t data_size = size_ - data0;
        for (auto& in : infos) {
            TensorView tv;
            tv.name = in.name;
            switch (in.type) {
                case 0: tv.dtype = DataType::F32; break;
                case 1: tv.dtype = DataType::F16; break;
                case 30: tv.dtype = DataType::BF16; break;
                default: return fail("tensor " + in.name + " has unsupported type " + std::to_string(in.type));
            }
            size_t numel = 1;
            for (uint64_t d : in.ne) {
                if (d == 0) return fail("tensor " + in.name + " has a zero dimension");
                if (numel > SIZE_MAX / d) return fail("tensor " + in.name + " size overflow");
                numel *= d;
            }
            const size_t bytes = numel * dtype_size(tv.dtype);
            if (in.off > data_size || bytes > data_size - in.off)
                return fail("tensor " + in.name + " extends past the end of the file");
            tv.ne = in.ne;
            tv.shape.assign(in.ne.rbegin(), in.ne.rend());
            tv.data = base + data0 + in.off;
            tv.bytes = bytes;
            tv.numel = numel;
            tensors_[tv.name] = std::move(tv);
        }
    } catch (const std::exception& e) {
        return fail(std::string("parse error: ") + e.what());
    }
    return 0;
}

const MetaValue* GGUFFile::get(const std::string& key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? nullptr : &it->second;
}

uint64_t GGUFFile::get_uint(const std::string& key) const {
    const MetaValue* v = get(key);
    if (!v) throw std::runtime_error("missing metadata key " + key);
    if (v->kind == MetaValue::UINT) return v->u;
    if (v->kind == MetaValue::INT && v->i >= 0) return (uint64_t)v->i;
    throw std::runtime_error("metadata key " + key + " is not a non-negative integer");
}

double GGUFFile::get_float(const std::string& key) const {
    const MetaValue* v = get(key);
    if (!v) throw std::runtime_error("missing metadata key " + key);
    if (v->kind == MetaValue::FLOAT) return v->f;
    if (v->kind == MetaValue::UINT) return (double)v->u;
    if (v->kind == MetaValue::INT) return (double)v->i;
    throw std::runtime_error("metadata key " + key + " is not a number");
}

const std::string& GGUFFile::get_string(const std::string& key) const {
    const MetaValue* v = get(key);
    if (!v || v->kind != MetaValue::STRING) throw std::runtime_error("missing string metadata key " + key);
    return v->s;
}

const TensorView& GGUFFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("missing tensor " + name);
    return it->second;
}

}  // namespace minfer
