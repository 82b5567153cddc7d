// Minimal GGUF v2/v3 reader for the packed upload path: parses the header,
// metadata and tensor descriptors (reference src/gguf/gguf_parser.cpp:46-174,
// same tensor-data alignment rule) and memory-maps the file so each tensor's
// packed bytes can be copied to HBM unchanged, without an FP32 expansion on the
// host (the reference dequantises every tensor at load,
// src/models/transformer.cpp:162-204).
#include "gguf_reader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <stdexcept>

namespace ib {

namespace {

// Reads from [p, end).  Every length comes from the file, so each check compares it
// with the bytes left instead of forming p + n, which a huge n would wrap.
struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    uint64_t left() const { return (uint64_t)(end - p); }
    template <typename T>
    T get() {
        if (left() < sizeof(T)) throw std::runtime_error("GGUF: truncated file");
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        uint64_t n = get<uint64_t>();
        if (n > left()) throw std::runtime_error("GGUF: truncated string");
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
    void skip(uint64_t n, uint64_t elem_size) {
        if (elem_size == 0 || n > left() / elem_size)
            throw std::runtime_error("GGUF: truncated value");
        p += n * elem_size;
    }
};

// Float metadata as an integer, where it has one.
int64_t float_to_int(double f) {
    return std::isfinite(f) && std::fabs(f) < 9.0e18 ? (int64_t)f : 0;
}

size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

}  // namespace

GGUFFile::~GGUFFile() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

void GGUFFile::open(const std::string& path) {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("Cannot open GGUF file: " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        throw std::runtime_error("Cannot stat GGUF file: " + path);
    }
    size_ = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw std::runtime_error("Cannot map GGUF file: " + path);
    base_ = static_cast<const uint8_t*>(m);

    Cursor c{base_, base_ + size_};
    if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("Invalid GGUF magic");
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) throw std::runtime_error("Unsupported GGUF version");
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key = c.str();
        uint32_t t = c.get<uint32_t>();
        Meta mv;
        mv.type = t;
        if (t == 8) {
            mv.s = c.str();
        } else if (t == 9) {
            uint32_t at = c.get<uint32_t>();
            uint64_t n = c.get<uint64_t>();
            if (at == 8) {
                for (uint64_t j = 0; j < n; ++j) c.str();
            } else {
                size_t sz = scalar_size(at);
                if (!sz) throw std::runtime_error("GGUF: bad array type");
                c.skip(n, sz);
            }
            mv.array_len = n;
        } else {
            size_t sz = scalar_size(t);
            if (!sz) throw std::runtime_error("GGUF: unknown metadata type");
            switch (t) {
                case 0: mv.i = c.get<uint8_t>(); break;
                case 1: mv.i = c.get<int8_t>(); break;
                case 2: mv.i = c.get<uint16_t>(); break;
                case 3: mv.i = c.get<int16_t>(); break;
                case 4: mv.i = c.get<uint32_t>(); break;
                case 5: mv.i = c.get<int32_t>(); break;
                case 6: mv.f = c.get<float>(); mv.i = float_to_int(mv.f); break;
                case 7: mv.i = c.get<uint8_t>(); break;
                case 10: mv.i = (int64_t)c.get<uint64_t>(); break;
                case 11: mv.i = c.get<int64_t>(); break;
                case 12: {
                    const double d = c.get<double>();
                    mv.f = (float)d;
                    mv.i = float_to_int(d);
                    break;
                }
            }
            if (t != 6 && t != 12) mv.f = (float)mv.i;
        }
        meta_[key] = mv;
    }
    for (uint64_t i = 0; i < n_tensors; ++i) {
        TensorInfo ti;
        ti.name = c.str();
        uint32_t nd = c.get<uint32_t>();
        for (uint32_t d = 0; d < nd; ++d) ti.dims.push_back((int64_t)c.get<uint64_t>());
        ti.type = (int)c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        tensors_.push_back(ti);
    }
    uint64_t align = 32;
    auto it = meta_.find("general.alignment");
    if (it != meta_.end() && it->second.i > 0) align = (uint64_t)it->second.i;
    if (align > (1u << 30)) throw std::runtime_error("GGUF: alignment out of range");
    data_offset_ = ((size_t)(c.p - base_) + align - 1) / align * align;
}

const GGUFFile::TensorInfo* GGUFFile::find(const std::string& name) const {
    for (const auto& t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

const uint8_t* GGUFFile::data(const TensorInfo& t, size_t bytes) const {
    const uint64_t room = data_offset_ <= size_ ? size_ - data_offset_ : 0;
    if (t.offset > room || bytes > room - t.offset)
        throw std::runtime_error("GGUF: tensor data out of range: " + t.name);
    return base_ + data_offset_ + t.offset;
}

int64_t GGUFFile::get_int(const std::string& key, int64_t def) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? def : it->second.i;
}

float GGUFFile::get_float(const std::string& key, float def) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? def : it->second.f;
}

}  // namespace ib
