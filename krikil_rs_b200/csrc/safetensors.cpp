#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <stdio.h>
#include <string.h>

namespace krk {
namespace {

// A small recursive-descent JSON reader for the safetensors header.
struct Json {
    const char* p;
    const char* e;
    std::string err;

    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(char c) {
        ws();
        if (p < e && *p == c) { ++p; return true; }
        return false;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool str(std::string& out) {
        ws();
        if (p >= e || *p != '"') return fail("expected string");
        ++p;
        out.clear();
        while (p < e && *p != '"') {
            if (*p == '\\') {
                ++p;
                if (p >= e) return fail("bad escape");
                char c = *p++;
                switch (c) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (e - p < 4) return fail("bad \\u escape");
                        unsigned v = 0;
                        for (int i = 0; i < 4; ++i) {
                            char h = *p++;
                            v <<= 4;
                            if (h >= '0' && h <= '9') v |= h - '0';
                            else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
                            else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
                            else return fail("bad \\u escape");
                        }
                        if (v < 0x80) out += (char)v;
                        else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 0x3F)); }
                        else {
                            out += (char)(0xE0 | (v >> 12));
                            out += (char)(0x80 | ((v >> 6) & 0x3F));
                            out += (char)(0x80 | (v & 0x3F));
                        }
                        break;
                    }
                    default: out += c;
                }
            } else {
                out += *p++;
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool integer(int64_t& v) {
        ws();
        bool neg = false;
        if (p < e && *p == '-') { neg = true; ++p; }
        if (p >= e || *p < '0' || *p > '9') return fail("expected integer");
        uint64_t x = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            uint64_t nx = x * 10 + (uint64_t)(*p - '0');
            if (nx / 10 != x) return fail("integer overflow");
            x = nx;
            ++p;
        }
        if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return fail("expected integer");
        v = neg ? -(int64_t)x : (int64_t)x;
        return true;
    }
    // Skips any JSON value (used for __metadata__ and unknown keys).
    bool skip() {
        ws();
        if (p >= e) return fail("unexpected end");
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{') {
            ++p;
            if (lit('}')) return true;
            do {
                std::string k;
                if (!str(k) || !lit(':') || !skip()) return false;
            } while (lit(','));
            return lit('}') || fail("expected }");
        }
        if (*p == '[') {
            ++p;
            if (lit(']')) return true;
            do {
                if (!skip()) return false;
            } while (lit(','));
            return lit(']') || fail("expected ]");
        }
        const char* s = p;
        while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') ++p;
        return p > s || fail("bad value");
    }
    bool int_array(std::vector<int64_t>& out) {
        out.clear();
        if (!lit('[')) return fail("expected [");
        if (lit(']')) return true;
        do {
            int64_t v;
            if (!integer(v)) return false;
            out.push_back(v);
        } while (lit(','));
        return lit(']') || fail("expected ]");
    }
    bool tensor(TensorInfo& t) {
        if (!lit('{')) return fail("expected {");
        bool have_off = false, have_dtype = false;
        if (!lit('}')) {
            do {
                std::string k;
                if (!str(k) || !lit(':')) return false;
                if (k == "dtype") {
                    if (!str(t.dtype)) return false;
                    have_dtype = true;
                } else if (k == "shape") {
                    if (!int_array(t.shape)) return false;
                } else if (k == "data_offsets") {
                    std::vector<int64_t> o;
                    if (!int_array(o)) return false;
                    if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) return fail("bad data_offsets");
                    t.begin = (uint64_t)o[0];
                    t.end = (uint64_t)o[1];
                    have_off = true;
                } else if (!skip()) {
                    return false;
                }
            } while (lit(','));
            if (!lit('}')) return fail("expected }");
        }
        return (have_off && have_dtype) || fail("tensor entry lacks dtype or data_offsets");
    }
};

}  // namespace

void SafeTensorsFile::unmap() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    base_ = nullptr;
    size_ = 0;
}

bool SafeTensorsFile::open(const std::string& path, std::string& err) {
    unmap();
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        err = "Failed to open model file: " + path;
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
        ::close(fd);
        err = "Failed to read model file: " + path;
        return false;
    }
    const size_t sz = (size_t)st.st_size;
    if (sz < 8) {
        ::close(fd);
        err = "Failed to parse safetensors from " + path + ": file too short";
        return false;
    }
    void* p = mmap(nullptr, sz, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) {
        err = "Failed to read model file: " + path;
        return false;
    }
    madvise(p, sz, MADV_SEQUENTIAL);
    base_ = static_cast<const uint8_t*>(p);
    size_ = sz;
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base_[i];
    if (hlen > (uint64_t)sz - 8) {
        err = "Failed to parse safetensors from " + path + ": header length exceeds file";
        return false;
    }
    data_off_ = 8 + (size_t)hlen;
    const uint64_t data_len = (uint64_t)sz - data_off_;
    Json js{reinterpret_cast<const char*>(base_) + 8, reinterpret_cast<const char*>(base_) + 8 + hlen, ""};
    tensors_.clear();
    bool ok = js.lit('{');
    if (ok && !js.lit('}')) {
        do {
            std::string name;
            if (!js.str(name) || !js.lit(':')) { ok = false; break; }
            if (name == "__metadata__") {
                if (!js.skip()) { ok = false; break; }
                continue;
            }
            TensorInfo t;
            if (!js.tensor(t)) { ok = false; break; }
            if (t.end > data_len) {
                js.err = "tensor '" + name + "' data_offsets exceed the file";
                ok = false;
                break;
            }
            tensors_[name] = t;
        } while (js.lit(','));
        if (ok && !js.lit('}')) ok = js.fail("expected }");
    } else if (!ok) {
        js.fail("expected {");
    }
    if (!ok) {
        err = "Failed to parse safetensors from " + path + ": " + (js.err.empty() ? "malformed header" : js.err);
        return false;
    }
    return true;
}

}  // namespace krk
