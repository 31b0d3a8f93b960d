// json.cpp -- recursive-descent JSON reader (see json.h).
#include "json.h"

#include <cstdint>
#include <cstdlib>
#include <cstring>

namespace krk {
namespace json {

const Value* Value::get(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

namespace {

constexpr int MAX_DEPTH = 512;

void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
        s.push_back((char)cp);
    } else if (cp < 0x800) {
        s.push_back((char)(0xC0 | (cp >> 6)));
        s.push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        s.push_back((char)(0xE0 | (cp >> 12)));
        s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        s.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
        s.push_back((char)(0xF0 | (cp >> 18)));
        s.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
        s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
        s.push_back((char)(0x80 | (cp & 0x3F)));
    }
}

struct Reader {
    const char* p;
    const char* end;
    const char* begin;
    std::string err;

    bool fail(const char* what) {
        if (err.empty()) err = std::string(what) + " at byte " + std::to_string(p - begin);
        return false;
    }
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if ((size_t)(end - p) < n || memcmp(p, w, n) != 0) return fail("invalid literal");
        p += n;
        return true;
    }
    bool hex4(uint32_t& v) {
        if (end - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad hex digit in \\u escape");
        }
        return true;
    }
    bool string(std::string& s) {
        if (p >= end || *p != '"') return fail("expected string");
        ++p;
        s.clear();
        while (true) {
            if (p >= end) return fail("unterminated string");
            const unsigned char c = (unsigned char)*p;
            if (c == '"') {
                ++p;
                return true;
            }
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') {
                s.push_back((char)c);
                ++p;
                continue;
            }
            ++p;
            if (p >= end) return fail("unterminated escape");
            const char e = *p++;
            switch (e) {
                case '"': s.push_back('"'); break;
                case '\\': s.push_back('\\'); break;
                case '/': s.push_back('/'); break;
                case 'b': s.push_back('\b'); break;
                case 'f': s.push_back('\f'); break;
                case 'n': s.push_back('\n'); break;
                case 'r': s.push_back('\r'); break;
                case 't': s.push_back('\t'); break;
                case 'u': {
                    uint32_t cp = 0;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
                        uint32_t lo = 0;
                        if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
                        p += 2;
                        if (!hex4(lo)) return false;
                        if (lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return fail("lone surrogate");
                    }
                    put_utf8(s, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
    }
    bool number(double& v) {
        const char* s = p;
        if (p < end && *p == '-') ++p;
        if (p >= end || !(*p >= '0' && *p <= '9')) return fail("bad number");
        while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' ||
                           *p == '-'))
            ++p;
        const std::string tok(s, p);
        char* e = nullptr;
        v = strtod(tok.c_str(), &e);
        if (e != tok.c_str() + tok.size()) return fail("bad number");
        return true;
    }
    bool value(Value& v, int depth) {
        if (depth > MAX_DEPTH) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        switch (*p) {
            case 'n': v.kind = Value::Null; return lit("null");
            case 't': v.kind = Value::Bool; v.b = true; return lit("true");
            case 'f': v.kind = Value::Bool; v.b = false; return lit("false");
            case '"': v.kind = Value::String; return string(v.str);
            case '[': {
                v.kind = Value::Array;
                ++p;
                ws();
                if (p < end && *p == ']') {
                    ++p;
                    return true;
                }
                while (true) {
                    v.arr.emplace_back();
                    if (!value(v.arr.back(), depth + 1)) return false;
                    ws();
                    if (p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (p < end && *p == ']') {
                        ++p;
                        return true;
                    }
                    return fail("expected , or ]");
                }
            }
            case '{': {
                v.kind = Value::Object;
                ++p;
                ws();
                if (p < end && *p == '}') {
                    ++p;
                    return true;
                }
                while (true) {
                    ws();
                    std::string key;
                    if (!string(key)) return false;
                    ws();
                    if (p >= end || *p != ':') return fail("expected :");
                    ++p;
                    v.obj.emplace_back(std::move(key), Value());
                    if (!value(v.obj.back().second, depth + 1)) return false;
                    ws();
                    if (p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (p < end && *p == '}') {
                        ++p;
                        return true;
                    }
                    return fail("expected , or }");
                }
            }
            default:
                v.kind = Value::Number;
                return number(v.num);
        }
    }
};

}  // namespace

bool parse(const char* text, size_t n, Value& out, std::string& err) {
    Reader r{text, text + n, text, {}};
    out = Value();
    if (!r.value(out, 0)) {
        err = r.err;
        return false;
    }
    r.ws();
    if (r.p != r.end) {
        r.fail("trailing characters");
        err = r.err;
        return false;
    }
    return true;
}

}  // namespace json
}  // namespace krk
