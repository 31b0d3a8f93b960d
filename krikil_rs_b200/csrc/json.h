// json.h -- a small JSON reader for the text front end's files
// (tokenizer.json): RFC 8259 values into a tree, objects keeping their key
// order.  Host code only.
#pragma once

#include <cstddef>
#include <string>
#include <utility>
#include <vector>

namespace krk {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object };
    Kind kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;

    // member `key` of an object, or nullptr (also for non-objects)
    const Value* get(const std::string& key) const;
    bool is_null() const { return kind == Null; }
};

// Parses a whole document; on failure returns false and sets err (with the
// byte offset of the problem).
bool parse(const char* text, size_t n, Value& out, std::string& err);

}  // namespace json
}  // namespace krk
