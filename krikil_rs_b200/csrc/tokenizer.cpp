// tokenizer.cpp -- byte-level BPE (see tokenizer.h).
//
// Encoding follows what the `tokenizers` crate does for the Pebble tokenizer
// (src/tokenizer.rs:25-32 calls Tokenizer::encode(text, false)):
//  1. split the text on added tokens (leftmost, then longest match);
//  2. split every other stretch with the GPT-2 pattern
//       's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
//     (first alternative that matches wins, as in a backtracking engine);
//  3. map each byte of a piece to its byte-level character and apply the BPE
//     merges lowest rank first, the leftmost pair among equal ranks, one merge
//     at a time (a stale queue entry is skipped when the pair at its position
//     no longer yields the entry's merged token).
// Decoding maps tokens back to bytes (a token with a character outside the
// byte-level alphabet keeps its own UTF-8) and converts them lossily.
#include "tokenizer.h"

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <fstream>
#include <queue>
#include <sstream>

#include "json.h"

namespace krk {
namespace {

#include "unicode_classes.inc"

enum CharClass : uint8_t { C_OTHER, C_LETTER, C_NUMBER, C_SPACE };

template <size_t N>
bool in_ranges(const uint32_t (&r)[N][2], uint32_t cp) {
    size_t lo = 0, hi = N;
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (r[mid][1] < cp) lo = mid + 1;
        else hi = mid;
    }
    return lo < N && r[lo][0] <= cp;
}

CharClass classify(uint32_t cp) {
    if (in_ranges(UNI_SPACE, cp)) return C_SPACE;
    if (in_ranges(UNI_LETTER, cp)) return C_LETTER;
    if (in_ranges(UNI_NUMBER, cp)) return C_NUMBER;
    return C_OTHER;
}

struct AsciiClasses {
    CharClass c[128];
    AsciiClasses() {
        for (uint32_t i = 0; i < 128; ++i) c[i] = classify(i);
    }
};

inline CharClass char_class(uint32_t cp) {
    static const AsciiClasses ascii;
    return cp < 128 ? ascii.c[cp] : classify(cp);
}

// Strict UTF-8 decoding into code points and their byte offsets (offs has
// one more entry: the end).
bool decode_utf8(const char* s, size_t n, std::vector<uint32_t>& cps, std::vector<size_t>& offs) {
    const unsigned char* u = reinterpret_cast<const unsigned char*>(s);
    cps.clear();
    offs.clear();
    size_t i = 0;
    while (i < n) {
        const unsigned char c = u[i];
        uint32_t cp;
        size_t len;
        if (c < 0x80) {
            cp = c;
            len = 1;
        } else if (c >= 0xC2 && c <= 0xDF) {
            cp = c & 0x1F;
            len = 2;
        } else if (c >= 0xE0 && c <= 0xEF) {
            cp = c & 0x0F;
            len = 3;
        } else if (c >= 0xF0 && c <= 0xF4) {
            cp = c & 0x07;
            len = 4;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (size_t k = 1; k < len; ++k) {
            if ((u[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (u[i + k] & 0x3F);
        }
        if ((len == 3 && (cp < 0x800 || (cp >= 0xD800 && cp < 0xE000))) || (len == 4 && (cp < 0x10000 || cp > 0x10FFFF)))
            return false;
        cps.push_back(cp);
        offs.push_back(i);
        i += len;
    }
    offs.push_back(n);
    return true;
}

bool read_file(const std::string& path, std::string& out, std::string& err) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        const int e = errno;
        err = std::string(strerror(e)) + " (os error " + std::to_string(e) + ")";
        return false;
    }
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

bool is_false_or_absent(const json::Value* v) { return !v || v->is_null() || (v->kind == json::Value::Bool && !v->b); }

}  // namespace

uint32_t byte_level_char(uint8_t b) {
    // printable bytes keep their code point, the other 68 are numbered from 256 on
    auto printable = [](int x) { return (x >= 0x21 && x <= 0x7E) || (x >= 0xA1 && x <= 0xAC) || (x >= 0xAE && x <= 0xFF); };
    if (printable(b)) return b;
    uint32_t n = 0;
    for (int x = 0; x < b; ++x)
        if (!printable(x)) ++n;
    return 256 + n;
}

void append_utf8(std::string& s, uint32_t cp) {
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

std::string utf8_lossy(const std::string& bytes) {
    static const char REPL[] = "\xEF\xBF\xBD";
    const unsigned char* u = reinterpret_cast<const unsigned char*>(bytes.data());
    const size_t n = bytes.size();
    std::string out;
    out.reserve(n);
    size_t i = 0;
    while (i < n) {
        const unsigned char c = u[i];
        if (c < 0x80) {
            out.push_back((char)c);
            ++i;
            continue;
        }
        // the allowed range of the second byte depends on the lead byte
        // (Unicode 3.9, table 3-7); later bytes are 80..BF
        size_t len = 0;
        unsigned char lo2 = 0x80, hi2 = 0xBF;
        if (c >= 0xC2 && c <= 0xDF) len = 2;
        else if (c == 0xE0) { len = 3; lo2 = 0xA0; }
        else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) len = 3;
        else if (c == 0xED) { len = 3; hi2 = 0x9F; }
        else if (c == 0xF0) { len = 4; lo2 = 0x90; }
        else if (c >= 0xF1 && c <= 0xF3) len = 4;
        else if (c == 0xF4) { len = 4; hi2 = 0x8F; }
        if (len == 0) {  // not a lead byte
            out += REPL;
            ++i;
            continue;
        }
        size_t k = 1;
        while (k < len && i + k < n) {
            const unsigned char t = u[i + k];
            const bool ok = k == 1 ? (t >= lo2 && t <= hi2) : (t >= 0x80 && t <= 0xBF);
            if (!ok) break;
            ++k;
        }
        if (k == len) out.append(bytes, i, len);
        else out += REPL;  // the maximal valid prefix becomes one replacement
        i += k;
    }
    return out;
}

std::unique_ptr<Tokenizer> Tokenizer::from_file(const std::string& path, std::string& err) {
    std::string text;
    if (!read_file(path, text, err)) return nullptr;
    return from_json(text, err);
}

std::unique_ptr<Tokenizer> Tokenizer::from_json(const std::string& text, std::string& err) {
    json::Value root;
    if (!json::parse(text.data(), text.size(), root, err)) {
        err = "invalid JSON: " + err;
        return nullptr;
    }
    auto bad = [&](const std::string& m) {
        err = m;
        return std::unique_ptr<Tokenizer>();
    };
    if (root.kind != json::Value::Object) return bad("tokenizer file is not a JSON object");
    std::unique_ptr<Tokenizer> t(new Tokenizer());

    const json::Value* norm = root.get("normalizer");
    if (norm && !norm->is_null()) return bad("unsupported normalizer");
    const json::Value* pre = root.get("pre_tokenizer");
    bool use_regex = true;
    if (!pre || pre->kind != json::Value::Object || !pre->get("type") || pre->get("type")->str != "ByteLevel")
        return bad("unsupported pre_tokenizer (a ByteLevel one is required)");
    if (const json::Value* v = pre->get("add_prefix_space")) t->add_prefix_space_ = v->kind == json::Value::Bool && v->b;
    if (const json::Value* v = pre->get("use_regex")) use_regex = !(v->kind == json::Value::Bool && !v->b);
    if (!use_regex) return bad("unsupported pre_tokenizer option use_regex = false");
    const json::Value* dec = root.get("decoder");
    if (!dec || dec->kind != json::Value::Object || !dec->get("type") || dec->get("type")->str != "ByteLevel")
        return bad("unsupported decoder (a ByteLevel one is required)");

    const json::Value* model = root.get("model");
    if (!model || model->kind != json::Value::Object) return bad("missing model");
    if (const json::Value* ty = model->get("type"))
        if (ty->str != "BPE") return bad("unsupported model type " + ty->str);
    if (!is_false_or_absent(model->get("dropout"))) return bad("unsupported BPE dropout");
    if (!is_false_or_absent(model->get("byte_fallback"))) return bad("unsupported BPE byte_fallback");
    if (!is_false_or_absent(model->get("ignore_merges"))) return bad("unsupported BPE ignore_merges");
    if (const json::Value* v = model->get("unk_token"))
        if (!v->is_null()) return bad("unsupported BPE unk_token");
    for (const char* k : {"continuing_subword_prefix", "end_of_word_suffix"})
        if (const json::Value* v = model->get(k))
            if (!v->is_null() && !(v->kind == json::Value::String && v->str.empty()))
                return bad(std::string("unsupported BPE ") + k);

    const json::Value* vocab = model->get("vocab");
    if (!vocab || vocab->kind != json::Value::Object) return bad("missing model vocab");
    uint32_t max_id = 0;
    for (const auto& kv : vocab->obj) {
        if (kv.second.kind != json::Value::Number || kv.second.num < 0 || kv.second.num > 0x7FFFFFFF)
            return bad("bad vocab id for " + kv.first);
        const uint32_t id = (uint32_t)kv.second.num;
        t->vocab_[kv.first] = id;
        max_id = std::max(max_id, id);
    }

    const json::Value* added = root.get("added_tokens");
    if (added && added->kind == json::Value::Array) {
        for (const auto& a : added->arr) {
            const json::Value* id = a.get("id");
            const json::Value* content = a.get("content");
            if (!id || id->kind != json::Value::Number || !content || content->kind != json::Value::String)
                return bad("bad added token");
            if (!is_false_or_absent(a.get("single_word"))) return bad("unsupported added-token option single_word");
            Added ad;
            ad.content = content->str;
            ad.id = (uint32_t)id->num;
            ad.special = !is_false_or_absent(a.get("special"));
            ad.lstrip = !is_false_or_absent(a.get("lstrip"));
            ad.rstrip = !is_false_or_absent(a.get("rstrip"));
            if (ad.content.empty()) return bad("empty added token");
            t->added_.push_back(ad);
            max_id = std::max(max_id, ad.id);
        }
    }

    t->id_to_token_.assign((size_t)max_id + 1, std::string());
    t->id_known_.assign((size_t)max_id + 1, 0);
    t->id_special_.assign((size_t)max_id + 1, 0);
    std::unordered_map<std::string, int> distinct;
    for (const auto& kv : t->vocab_) {
        t->id_to_token_[kv.second] = kv.first;
        t->id_known_[kv.second] = 1;
        distinct[kv.first] = 1;
    }
    for (const auto& ad : t->added_) {
        t->id_to_token_[ad.id] = ad.content;
        t->id_known_[ad.id] = 1;
        t->id_special_[ad.id] = ad.special ? 1 : 0;
        distinct[ad.content] = 1;
    }
    t->vocab_size_ = distinct.size();

    for (int b = 0; b < 256; ++b) {
        std::string ch;
        append_utf8(ch, byte_level_char((uint8_t)b));
        const auto it = t->vocab_.find(ch);
        t->byte_id_[b] = it == t->vocab_.end() ? -1 : (int64_t)it->second;
    }

    const json::Value* merges = model->get("merges");
    if (!merges || merges->kind != json::Value::Array) return bad("missing BPE merges");
    uint32_t rank = 0;
    for (const auto& m : merges->arr) {
        std::string a, b;
        if (m.kind == json::Value::String) {
            const size_t sp = m.str.find(' ');
            if (sp == std::string::npos || m.str.find(' ', sp + 1) != std::string::npos)
                return bad("bad merge \"" + m.str + "\"");
            a = m.str.substr(0, sp);
            b = m.str.substr(sp + 1);
        } else if (m.kind == json::Value::Array && m.arr.size() == 2 && m.arr[0].kind == json::Value::String &&
                   m.arr[1].kind == json::Value::String) {
            a = m.arr[0].str;
            b = m.arr[1].str;
        } else {
            return bad("bad merge entry");
        }
        const auto ia = t->vocab_.find(a), ib = t->vocab_.find(b), iab = t->vocab_.find(a + b);
        if (ia == t->vocab_.end() || ib == t->vocab_.end()) return bad("merge token missing from vocab: " + a + " " + b);
        if (iab == t->vocab_.end()) return bad("merged token missing from vocab: " + a + b);
        const uint64_t key = (uint64_t)ia->second << 32 | ib->second;
        t->merges_.emplace(key, Merge{rank, iab->second});  // the first (lowest) rank of a pair stays
        ++rank;
    }
    return t;
}

int64_t Tokenizer::token_to_id(const std::string& token) const {
    for (const auto& ad : added_)
        if (ad.content == token) return ad.id;
    const auto it = vocab_.find(token);
    return it == vocab_.end() ? -1 : (int64_t)it->second;
}

void Tokenizer::bpe_piece(const std::string& bytes, std::vector<uint32_t>& ids) const {
    struct Sym {
        uint32_t id;
        int prev, next;
        bool alive;
    };
    std::vector<Sym> sy;
    sy.reserve(bytes.size());
    for (unsigned char c : bytes) {
        const int64_t id = byte_id_[c];
        if (id < 0) continue;  // a byte outside the vocabulary is dropped (no unknown token)
        const int i = (int)sy.size();
        sy.push_back(Sym{(uint32_t)id, i - 1, -1, true});
        if (i > 0) sy[i - 1].next = i;
    }
    if (sy.empty()) return;
    struct Cand {
        uint32_t rank;
        int pos;
        uint32_t id;
        bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
    };
    std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> q;
    auto pair_of = [&](int l) -> const Merge* {
        const int r = sy[l].next;
        if (r < 0) return nullptr;
        const auto it = merges_.find((uint64_t)sy[l].id << 32 | sy[r].id);
        return it == merges_.end() ? nullptr : &it->second;
    };
    for (int i = 0; i + 1 < (int)sy.size(); ++i)
        if (const Merge* m = pair_of(i)) q.push(Cand{m->rank, i, m->id});
    while (!q.empty()) {
        const Cand c = q.top();
        q.pop();
        Sym& l = sy[c.pos];
        if (!l.alive || l.next < 0) continue;
        const Merge* m = pair_of(c.pos);
        if (!m || m->id != c.id) continue;  // stale: the pair here changed
        Sym& r = sy[l.next];
        l.id = c.id;
        l.next = r.next;
        r.alive = false;
        if (l.next >= 0) sy[l.next].prev = c.pos;
        if (l.prev >= 0)
            if (const Merge* mp = pair_of(l.prev)) q.push(Cand{mp->rank, l.prev, mp->id});
        if (const Merge* mn = pair_of(c.pos)) q.push(Cand{mn->rank, c.pos, mn->id});
    }
    for (int i = 0; i >= 0; i = sy[i].next) ids.push_back(sy[i].id);
}

void Tokenizer::encode_segment(const std::vector<uint32_t>& cps, size_t lo, size_t hi,
                               std::vector<uint32_t>& ids) const {
    std::vector<uint32_t> seg;
    if (add_prefix_space_ && (lo == hi || cps[lo] != ' ')) seg.push_back(' ');
    seg.insert(seg.end(), cps.begin() + (long)lo, cps.begin() + (long)hi);
    const size_t n = seg.size();
    std::vector<CharClass> cl(n);
    for (size_t i = 0; i < n; ++i) cl[i] = char_class(seg[i]);
    auto run = [&](size_t from, CharClass k) {
        size_t j = from;
        while (j < n && cl[j] == k) ++j;
        return j;
    };
    std::string piece;
    size_t i = 0;
    while (i < n) {
        size_t end = i + 1;
        const uint32_t c0 = seg[i];
        const uint32_t c1 = i + 1 < n ? seg[i + 1] : 0, c2 = i + 2 < n ? seg[i + 2] : 0;
        if (c0 == '\'' && (c1 == 's' || c1 == 't' || c1 == 'm' || c1 == 'd')) {
            end = i + 2;
        } else if (c0 == '\'' && ((c1 == 'r' && c2 == 'e') || (c1 == 'v' && c2 == 'e') || (c1 == 'l' && c2 == 'l'))) {
            end = i + 3;
        } else if (c0 == ' ' && i + 1 < n && cl[i + 1] != C_SPACE) {
            end = run(i + 1, cl[i + 1]);  // " ?\p{L}+", " ?\p{N}+", " ?[^\s\p{L}\p{N}]+"
        } else if (cl[i] != C_SPACE) {
            end = run(i, cl[i]);
        } else {
            const size_t j = run(i, C_SPACE);  // "\s+(?!\S)", else "\s+"
            end = (j == n || j - i == 1) ? j : j - 1;
        }
        piece.clear();
        for (size_t k = i; k < end; ++k) append_utf8(piece, seg[k]);
        bpe_piece(piece, ids);
        i = end;
    }
}

bool Tokenizer::encode(const char* text, size_t len, std::vector<uint32_t>& ids, std::string& err) const {
    ids.clear();
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    if (!decode_utf8(text, len, cps, offs)) {
        err = "input is not valid UTF-8";
        return false;
    }
    // added tokens as code-point sequences
    std::vector<std::vector<uint32_t>> acp(added_.size());
    for (size_t a = 0; a < added_.size(); ++a) {
        std::vector<size_t> o;
        decode_utf8(added_[a].content.data(), added_[a].content.size(), acp[a], o);
    }
    const size_t n = cps.size();
    size_t seg_lo = 0, i = 0;
    while (i < n) {
        int best = -1;
        size_t best_len = 0;
        for (size_t a = 0; a < acp.size(); ++a) {
            const auto& s = acp[a];
            if (s.empty() || s.size() <= best_len || i + s.size() > n) continue;
            if (std::equal(s.begin(), s.end(), cps.begin() + (long)i)) {
                best = (int)a;
                best_len = s.size();
            }
        }
        if (best < 0) {
            ++i;
            continue;
        }
        size_t mlo = i, mhi = i + best_len;
        if (added_[best].lstrip)
            while (mlo > seg_lo && char_class(cps[mlo - 1]) == C_SPACE) --mlo;
        if (added_[best].rstrip)
            while (mhi < n && char_class(cps[mhi]) == C_SPACE) ++mhi;
        if (mlo > seg_lo) encode_segment(cps, seg_lo, mlo, ids);
        ids.push_back(added_[best].id);
        seg_lo = i = mhi;
    }
    if (seg_lo < n) encode_segment(cps, seg_lo, n, ids);
    return true;
}

std::string Tokenizer::decode(const uint32_t* ids, size_t n, bool skip_special) const {
    static const struct Inverse {
        int16_t byte_of[324];  // byte-level characters are below 324
        Inverse() {
            for (int16_t& x : byte_of) x = -1;
            for (int b = 0; b < 256; ++b) byte_of[byte_level_char((uint8_t)b)] = (int16_t)b;
        }
    } inv;
    std::string bytes;
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    for (size_t k = 0; k < n; ++k) {
        const uint32_t id = ids[k];
        if (id >= id_to_token_.size() || !id_known_[id]) continue;
        if (skip_special && id_special_[id]) continue;
        const std::string& tok = id_to_token_[id];
        bool mapped = decode_utf8(tok.data(), tok.size(), cps, offs);
        std::string tb;
        for (size_t c = 0; mapped && c < cps.size(); ++c) {
            if (cps[c] >= 324 || inv.byte_of[cps[c]] < 0) mapped = false;
            else tb.push_back((char)inv.byte_of[cps[c]]);
        }
        bytes += mapped ? tb : tok;
    }
    return utf8_lossy(bytes);
}

}  // namespace krk
