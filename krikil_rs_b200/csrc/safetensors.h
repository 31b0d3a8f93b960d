// Minimal safetensors reader: 8-byte little-endian header length, a JSON
// header mapping tensor names to {dtype, shape, data_offsets}, then the raw
// little-endian tensor bytes (the format safetensors 0.5 reads for
// src/model.rs:237-254).
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace krk {

struct TensorInfo {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte offsets into the data section
};

// The file is mapped read-only (no copy of the tensor bytes on the host); the
// mapping lives as long as the object.
class SafeTensorsFile {
public:
    SafeTensorsFile() = default;
    SafeTensorsFile(const SafeTensorsFile&) = delete;
    SafeTensorsFile& operator=(const SafeTensorsFile&) = delete;
    ~SafeTensorsFile() { unmap(); }
    // Returns false and sets err on failure (missing file, short read,
    // malformed header, offsets outside the data section).
    bool open(const std::string& path, std::string& err);
    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorInfo* info(const std::string& name) const {
        auto it = tensors_.find(name);
        return it == tensors_.end() ? nullptr : &it->second;
    }
    const uint8_t* data(const TensorInfo& t) const { return base_ + data_off_ + t.begin; }

private:
    void unmap();
    const uint8_t* base_ = nullptr;
    size_t size_ = 0;
    size_t data_off_ = 0;
    std::map<std::string, TensorInfo> tensors_;
};

}  // namespace krk
