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

class SafeTensorsFile {
public:
    // Returns false and sets err on failure (missing file, short read,
    // malformed header, offsets outside the data section).
    bool open(const std::string& path, std::string& err);
    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorInfo* info(const std::string& name) const {
        auto it = tensors_.find(name);
        return it == tensors_.end() ? nullptr : &it->second;
    }
    const uint8_t* data(const TensorInfo& t) const { return bytes_.data() + data_off_ + t.begin; }

private:
    std::vector<uint8_t> bytes_;
    size_t data_off_ = 0;
    std::map<std::string, TensorInfo> tensors_;
};

}  // namespace krk
