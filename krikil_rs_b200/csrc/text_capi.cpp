// text_capi.cpp -- the C ABI of include/krikil_text.h over tokenizer.h and
// chat_template.h.
#include <sys/stat.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/krikil_text.h"
#include "chat_template.h"
#include "tokenizer.h"

namespace krk {
int report_error(int status, const std::string& msg);  // capi.cu: sets krk_last_error()
}

struct krk_tokenizer {
    std::unique_ptr<krk::Tokenizer> t;
};

namespace {

int ok_or_small(size_t need, size_t cap, bool have_buf) {
    if (have_buf && cap < need) return krk::report_error(KRK_INVALID, "output buffer too small");
    return KRK_OK;
}

// Copies s into out (with a NUL if it fits) under the buffer rule of the header.
int put_string(const std::string& s, char* out, size_t cap, size_t* len_out) {
    if (!len_out) return krk::report_error(KRK_INVALID, "null length pointer");
    *len_out = s.size();
    if (!out) return KRK_OK;
    if (const int rc = ok_or_small(s.size(), cap, true)) return rc;
    memcpy(out, s.data(), s.size());
    if (cap > s.size()) out[s.size()] = '\0';
    return KRK_OK;
}

bool exists(const std::string& p) {
    struct stat st;
    return stat(p.c_str(), &st) == 0;
}

// Path::parent of a path string: false where Rust's parent() is None
// ("" and "/"); "" for a bare file name.
bool parent_of(std::string p, std::string& parent) {
    while (p.size() > 1 && p.back() == '/') p.pop_back();
    if (p.empty() || p == "/") return false;
    const size_t s = p.rfind('/');
    if (s == std::string::npos) {
        parent.clear();
    } else if (s == 0) {
        parent = "/";
    } else {
        parent = p.substr(0, s);
        while (parent.size() > 1 && parent.back() == '/') parent.pop_back();
    }
    return true;
}

std::string join(const std::string& dir, const char* name) {
    if (dir.empty()) return name;
    if (dir.back() == '/') return dir + name;
    return dir + "/" + name;
}

}  // namespace

extern "C" {

int krk_tokenizer_load(const char* path, krk_tokenizer** out) {
    if (!path || !out) return krk::report_error(KRK_INVALID, "null argument");
    *out = nullptr;
    std::string err;
    std::unique_ptr<krk::Tokenizer> t = krk::Tokenizer::from_file(path, err);
    if (!t) return krk::report_error(KRK_IO, std::string("Failed to load tokenizer from ") + path + ": " + err);
    *out = new krk_tokenizer{std::move(t)};
    return KRK_OK;
}

int krk_tokenizer_free(krk_tokenizer* tok) {
    delete tok;
    return KRK_OK;
}

int krk_tokenizer_encode(const krk_tokenizer* tok, const char* text, size_t len, uint32_t* ids, size_t cap,
                         size_t* n_out) {
    if (!tok || (!text && len) || !n_out) return krk::report_error(KRK_INVALID, "null argument");
    std::vector<uint32_t> v;
    std::string err;
    if (!tok->t->encode(text ? text : "", len, v, err))
        return krk::report_error(KRK_INVALID, "Failed to encode text: " + err);
    *n_out = v.size();
    if (!ids) return KRK_OK;
    if (const int rc = ok_or_small(v.size(), cap, true)) return rc;
    if (!v.empty()) memcpy(ids, v.data(), v.size() * sizeof(uint32_t));
    return KRK_OK;
}

int krk_tokenizer_decode(const krk_tokenizer* tok, const uint32_t* ids, size_t n, int skip_special, char* out,
                         size_t cap, size_t* len_out) {
    if (!tok || (!ids && n)) return krk::report_error(KRK_INVALID, "null argument");
    return put_string(tok->t->decode(ids, n, skip_special != 0), out, cap, len_out);
}

int krk_tokenizer_token_to_id(const krk_tokenizer* tok, const char* token, int64_t* id) {
    if (!tok || !token || !id) return krk::report_error(KRK_INVALID, "null argument");
    *id = tok->t->token_to_id(token);
    return KRK_OK;
}

int krk_tokenizer_eos_token_id(const krk_tokenizer* tok, uint32_t* id) {
    if (!tok || !id) return krk::report_error(KRK_INVALID, "null argument");
    const int64_t e = tok->t->token_to_id("<|eos|>");
    *id = e < 0 ? 0u : (uint32_t)e;  // src/tokenizer.rs:5, :19-21
    return KRK_OK;
}

int krk_tokenizer_vocab_size(const krk_tokenizer* tok, size_t* n) {
    if (!tok || !n) return krk::report_error(KRK_INVALID, "null argument");
    *n = tok->t->vocab_size();
    return KRK_OK;
}

int krk_tokenizer_resolve_path(const char* model_path, const char* explicit_path, char* out, size_t cap,
                               size_t* len_out) {
    if (!model_path) return krk::report_error(KRK_INVALID, "null model path");
    if (explicit_path) {
        if (exists(explicit_path)) return put_string(explicit_path, out, cap, len_out);
        return krk::report_error(KRK_IO, std::string("Explicit tokenizer path not found: ") + explicit_path);
    }
    std::string dir;
    if (!parent_of(model_path, dir)) dir = ".";
    const std::string sibling = join(dir, "tokenizer.json");
    if (exists(sibling)) return put_string(sibling, out, cap, len_out);
    if (exists("tokenizer.json")) return put_string("tokenizer.json", out, cap, len_out);
    return krk::report_error(KRK_IO, "Could not find tokenizer.json. Looked at " + sibling +
                                         " and tokenizer.json. Use --tokenizer to specify its path.");
}

int krk_chat_template_render(const char* source, const char* const* roles, const char* const* contents, size_t n,
                             int add_generation_prompt, char* out, size_t cap, size_t* len_out) {
    if (n && (!roles || !contents)) return krk::report_error(KRK_INVALID, "null messages");
    std::vector<krk::ChatMessage> msgs(n);
    for (size_t i = 0; i < n; ++i) {
        if (!roles[i] || !contents[i]) return krk::report_error(KRK_INVALID, "null message field");
        msgs[i].role = roles[i];
        msgs[i].content = contents[i];
    }
    std::string text, err;
    if (!krk::render_chat_template(source ? source : krk::DEFAULT_CHAT_TEMPLATE, msgs, add_generation_prompt != 0,
                                   text, err))
        return krk::report_error(KRK_INVALID, err);
    return put_string(text, out, cap, len_out);
}

const char* krk_default_chat_template(void) { return krk::DEFAULT_CHAT_TEMPLATE; }

}  // extern "C"
