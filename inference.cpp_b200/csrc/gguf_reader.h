// Memory-mapped GGUF reader (packed upload path).
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace ib {

class GGUFFile {
public:
    struct TensorInfo {
        std::string name;
        std::vector<int64_t> dims;  // ne0 first
        int type = 0;
        uint64_t offset = 0;
    };
    struct Meta {
        uint32_t type = 0;
        int64_t i = 0;
        float f = 0.f;
        std::string s;
        uint64_t array_len = 0;
    };

    GGUFFile() = default;
    ~GGUFFile();
    GGUFFile(const GGUFFile&) = delete;
    GGUFFile& operator=(const GGUFFile&) = delete;

    void open(const std::string& path);
    const TensorInfo* find(const std::string& name) const;
    const uint8_t* data(const TensorInfo& t, size_t bytes) const;
    int64_t get_int(const std::string& key, int64_t def) const;
    float get_float(const std::string& key, float def) const;
    bool has(const std::string& key) const { return meta_.count(key) != 0; }
    const std::vector<TensorInfo>& tensors() const { return tensors_; }

private:
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
    size_t data_offset_ = 0;
    std::map<std::string, Meta> meta_;
    std::vector<TensorInfo> tensors_;
};

}  // namespace ib
