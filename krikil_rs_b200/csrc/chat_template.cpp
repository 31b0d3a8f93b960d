// chat_template.cpp -- a Jinja-subset renderer for chat templates (see
// chat_template.h): a lexer that cuts the source into text and tags, a
// recursive-descent parser into a small tree, and a tree walker.
#include "chat_template.h"

#include <cctype>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <utility>

namespace krk {

const char* const DEFAULT_CHAT_TEMPLATE =
    "{% for message in messages %}{% if message['role'] == 'user' %}user: {% elif message['role'] == 'assistant' "
    "%}assistant: {% else %}{{ message['role'] }}: {% endif %}{% if message['content'] is string %}{{ "
    "message['content'] }}{% else %}{% for part in message['content'] %}{{ part['text'] }}{% endfor %}{% endif "
    "%} {% endfor %}{% if add_generation_prompt %}assistant: {% endif %}";

namespace {

struct SyntaxError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct RenderError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// ------------------------------------------------------------------ values
struct Val;
using List = std::vector<Val>;
using Map = std::vector<std::pair<std::string, Val>>;

struct Val {
    enum Kind { Undef, None, Bool, Int, Float, Str, Seq, Obj } k = Undef;
    bool b = false;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    std::shared_ptr<List> list;
    std::shared_ptr<Map> map;

    static Val none() { Val v; v.k = None; return v; }
    static Val boolean(bool x) { Val v; v.k = Bool; v.b = x; return v; }
    static Val integer(int64_t x) { Val v; v.k = Int; v.i = x; return v; }
    static Val real(double x) { Val v; v.k = Float; v.f = x; return v; }
    static Val str(std::string x) { Val v; v.k = Str; v.s = std::move(x); return v; }
    static Val seq(List x) { Val v; v.k = Seq; v.list = std::make_shared<List>(std::move(x)); return v; }
    static Val obj(Map x) { Val v; v.k = Obj; v.map = std::make_shared<Map>(std::move(x)); return v; }

    bool number() const { return k == Int || k == Float; }
    double as_double() const { return k == Int ? (double)i : f; }
    bool truthy() const {
        switch (k) {
            case Bool: return b;
            case Int: return i != 0;
            case Float: return f != 0.0;
            case Str: return !s.empty();
            case Seq: return !list->empty();
            case Obj: return !map->empty();
            default: return false;
        }
    }
    const Val* find(const std::string& key) const {
        if (k != Obj) return nullptr;
        for (const auto& kv : *map)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

std::string kind_name(const Val& v) {
    static const char* names[] = {"undefined", "none", "bool", "number", "number", "string", "sequence", "map"};
    return names[v.k];
}

std::string to_text(const Val& v);

std::string float_text(double f) {
    if (std::isnan(f)) return "NaN";
    if (std::isinf(f)) return f > 0 ? "inf" : "-inf";
    if (f == std::floor(f) && std::fabs(f) < 1e16) {
        char buf[64];
        snprintf(buf, sizeof buf, "%.1f", f);
        return buf;
    }
    char buf[64];
    for (int prec = 1; prec <= 17; ++prec) {  // shortest text that reads back to f
        snprintf(buf, sizeof buf, "%.*g", prec, f);
        if (strtod(buf, nullptr) == f) break;
    }
    return buf;
}

std::string to_text(const Val& v) {
    switch (v.k) {
        case Val::Undef: return "";
        case Val::None: return "none";
        case Val::Bool: return v.b ? "true" : "false";
        case Val::Int: return std::to_string(v.i);
        case Val::Float: return float_text(v.f);
        case Val::Str: return v.s;
        case Val::Seq: {
            std::string o = "[";
            for (size_t j = 0; j < v.list->size(); ++j) {
                const Val& e = (*v.list)[j];
                if (j) o += ", ";
                o += e.k == Val::Str ? "\"" + e.s + "\"" : to_text(e);
            }
            return o + "]";
        }
        case Val::Obj: {
            std::string o = "{";
            for (size_t j = 0; j < v.map->size(); ++j) {
                const auto& kv = (*v.map)[j];
                if (j) o += ", ";
                o += "\"" + kv.first + "\": ";
                o += kv.second.k == Val::Str ? "\"" + kv.second.s + "\"" : to_text(kv.second);
            }
            return o + "}";
        }
    }
    return "";
}

bool equal(const Val& a, const Val& b) {
    if (a.number() && b.number()) {
        if (a.k == Val::Int && b.k == Val::Int) return a.i == b.i;
        return a.as_double() == b.as_double();
    }
    if (a.k != b.k) return false;
    switch (a.k) {
        case Val::Undef:
        case Val::None: return true;
        case Val::Bool: return a.b == b.b;
        case Val::Str: return a.s == b.s;
        case Val::Seq:
            if (a.list->size() != b.list->size()) return false;
            for (size_t j = 0; j < a.list->size(); ++j)
                if (!equal((*a.list)[j], (*b.list)[j])) return false;
            return true;
        case Val::Obj:
            if (a.map->size() != b.map->size()) return false;
            for (const auto& kv : *a.map) {
                const Val* o = b.find(kv.first);
                if (!o || !equal(kv.second, *o)) return false;
            }
            return true;
        default: return false;
    }
}

// ------------------------------------------------------------------- lexer
struct Tok {
    enum Kind { Name, String, Integer, Real, Op, End } k;
    std::string s;
    int64_t i = 0;
    double f = 0.0;
};

std::vector<Tok> lex_expr(const std::string& src) {
    std::vector<Tok> out;
    size_t p = 0;
    const size_t n = src.size();
    while (p < n) {
        const char c = src[p];
        if (c == ' ' || c == '\t' || c == '\n' || c == '\r') {
            ++p;
        } else if (isalpha((unsigned char)c) || c == '_') {
            size_t q = p;
            while (q < n && (isalnum((unsigned char)src[q]) || src[q] == '_')) ++q;
            out.push_back(Tok{Tok::Name, src.substr(p, q - p)});
            p = q;
        } else if (isdigit((unsigned char)c)) {
            size_t q = p;
            while (q < n && (isdigit((unsigned char)src[q]) || src[q] == '_')) ++q;
            bool real = false;
            if (q + 1 < n && src[q] == '.' && isdigit((unsigned char)src[q + 1])) {
                real = true;
                ++q;
                while (q < n && isdigit((unsigned char)src[q])) ++q;
            }
            if (q < n && (src[q] == 'e' || src[q] == 'E')) {
                size_t r = q + 1;
                if (r < n && (src[r] == '+' || src[r] == '-')) ++r;
                if (r < n && isdigit((unsigned char)src[r])) {
                    real = true;
                    q = r;
                    while (q < n && isdigit((unsigned char)src[q])) ++q;
                }
            }
            std::string num;
            for (size_t j = p; j < q; ++j)
                if (src[j] != '_') num.push_back(src[j]);
            Tok t{real ? Tok::Real : Tok::Integer, num};
            if (real) t.f = strtod(num.c_str(), nullptr);
            else t.i = strtoll(num.c_str(), nullptr, 10);
            out.push_back(t);
            p = q;
        } else if (c == '\'' || c == '"') {
            std::string s;
            size_t q = p + 1;
            while (true) {
                if (q >= n) throw SyntaxError("unterminated string");
                if (src[q] == c) break;
                if (src[q] == '\\' && q + 1 < n) {
                    const char e = src[q + 1];
                    switch (e) {
                        case 'n': s.push_back('\n'); break;
                        case 't': s.push_back('\t'); break;
                        case 'r': s.push_back('\r'); break;
                        case '\\': s.push_back('\\'); break;
                        case '\'': s.push_back('\''); break;
                        case '"': s.push_back('"'); break;
                        default: s.push_back('\\'); s.push_back(e); break;
                    }
                    q += 2;
                } else {
                    s.push_back(src[q++]);
                }
            }
            out.push_back(Tok{Tok::String, s});
            p = q + 1;
        } else {
            static const char* ops2[] = {"==", "!=", "<=", ">=", "//", "**"};
            bool two = false;
            for (const char* o : ops2)
                if (src.compare(p, 2, o) == 0) {
                    out.push_back(Tok{Tok::Op, o});
                    p += 2;
                    two = true;
                    break;
                }
            if (two) continue;
            if (std::string("()[]{}.,|~+-*/%:<>=").find(c) == std::string::npos)
                throw SyntaxError(std::string("unexpected character '") + c + "'");
            out.push_back(Tok{Tok::Op, std::string(1, c)});
            ++p;
        }
    }
    out.push_back(Tok{Tok::End, ""});
    return out;
}

// Nesting limit of expressions and blocks: the parser recurses per level, so a
// hostile template must not be able to exhaust the stack.
constexpr int MAX_NEST = 100;
struct NestGuard {
    int& d;
    NestGuard(int& depth, const char* what) : d(depth) {
        if (++d > MAX_NEST) {
            --d;
            throw SyntaxError(std::string(what) + " nested too deeply");
        }
    }
    ~NestGuard() { --d; }
};

// ----------------------------------------------------------------- the tree
struct Expr;
using ExprP = std::shared_ptr<Expr>;
struct Expr {
    enum Kind { Lit, Var, ListLit, Attr, Item, Slice, Unary, Binary, Test, Filter, Call, Cond } k;
    Val lit;
    std::string name;           // Var / Attr / Test / Filter / Call / operator of Unary, Binary
    std::vector<ExprP> args;    // operands
    bool negate = false;        // "is not"
};

struct Node;
using NodeP = std::shared_ptr<Node>;
using Body = std::vector<NodeP>;
struct Node {
    enum Kind { Text, Out, If, For, Set } k;
    std::string text;
    ExprP expr;                                    // Out, For iterable, Set value
    std::vector<std::pair<ExprP, Body>> branches;  // If
    Body body, else_body;                          // For (and the If's else)
    std::vector<std::string> targets;              // For / Set
};

// ------------------------------------------------------------------ parser
class ExprParser {
   public:
    explicit ExprParser(std::vector<Tok> t) : t_(std::move(t)) {}

    ExprP parse_all() {
        ExprP e = expr();
        if (t_[p_].k != Tok::End) throw SyntaxError("unexpected '" + t_[p_].s + "'");
        return e;
    }
    // "a, b in expr" of a for statement
    void parse_for(std::vector<std::string>& targets, ExprP& iter) {
        do {
            if (t_[p_].k != Tok::Name) throw SyntaxError("expected a loop variable");
            targets.push_back(t_[p_++].s);
        } while (accept_op(","));
        if (!accept_name("in")) throw SyntaxError("expected 'in'");
        iter = expr_no_cond();
        if (t_[p_].k != Tok::End) throw SyntaxError("unsupported for-loop clause '" + t_[p_].s + "'");
    }
    void parse_set(std::string& name, ExprP& value) {
        if (t_[p_].k != Tok::Name) throw SyntaxError("expected a variable name");
        name = t_[p_++].s;
        if (!accept_op("=")) throw SyntaxError("expected '='");
        value = parse_all();
    }

   private:
    std::vector<Tok> t_;
    size_t p_ = 0;
    int depth_ = 0;

    bool is_op(const char* o) const { return t_[p_].k == Tok::Op && t_[p_].s == o; }
    bool is_name(const char* w) const { return t_[p_].k == Tok::Name && t_[p_].s == w; }
    bool accept_op(const char* o) {
        if (!is_op(o)) return false;
        ++p_;
        return true;
    }
    bool accept_name(const char* w) {
        if (!is_name(w)) return false;
        ++p_;
        return true;
    }
    void expect_op(const char* o) {
        if (!accept_op(o)) throw SyntaxError(std::string("expected '") + o + "'");
    }
    static ExprP mk(Expr::Kind k, std::string name, std::vector<ExprP> args) {
        auto e = std::make_shared<Expr>();
        e->k = k;
        e->name = std::move(name);
        e->args = std::move(args);
        return e;
    }

    ExprP expr() {  // a if cond else b
        NestGuard g(depth_, "expression");
        ExprP a = expr_no_cond();
        if (accept_name("if")) {
            ExprP c = or_expr();
            ExprP b;
            if (accept_name("else")) b = expr();
            else b = mk(Expr::Lit, "", {});  // undefined
            return mk(Expr::Cond, "", {c, a, b});
        }
        return a;
    }
    ExprP expr_no_cond() { return or_expr(); }
    ExprP or_expr() {
        ExprP a = and_expr();
        while (accept_name("or")) a = mk(Expr::Binary, "or", {a, and_expr()});
        return a;
    }
    ExprP and_expr() {
        ExprP a = not_expr();
        while (accept_name("and")) a = mk(Expr::Binary, "and", {a, not_expr()});
        return a;
    }
    ExprP not_expr() {
        if (accept_name("not")) {
            NestGuard g(depth_, "expression");
            return mk(Expr::Unary, "not", {not_expr()});
        }
        return compare();
    }
    ExprP compare() {
        ExprP a = concat();
        while (true) {
            static const char* cmp[] = {"==", "!=", "<=", ">=", "<", ">"};
            bool done = true;
            for (const char* o : cmp)
                if (accept_op(o)) {
                    a = mk(Expr::Binary, o, {a, concat()});
                    done = false;
                    break;
                }
            if (!done) continue;
            if (accept_name("in")) {
                a = mk(Expr::Binary, "in", {a, concat()});
            } else if (is_name("not") && t_[p_ + 1].k == Tok::Name && t_[p_ + 1].s == "in") {
                p_ += 2;
                a = mk(Expr::Unary, "not", {mk(Expr::Binary, "in", {a, concat()})});
            } else if (accept_name("is")) {
                const bool neg = accept_name("not");
                if (t_[p_].k != Tok::Name) throw SyntaxError("expected a test name");
                ExprP t = mk(Expr::Test, t_[p_++].s, {a});
                t->negate = neg;
                a = t;
            } else {
                return a;
            }
        }
    }
    ExprP concat() {
        ExprP a = additive();
        while (accept_op("~")) a = mk(Expr::Binary, "~", {a, additive()});
        return a;
    }
    ExprP additive() {
        ExprP a = multiplicative();
        while (true) {
            if (accept_op("+")) a = mk(Expr::Binary, "+", {a, multiplicative()});
            else if (accept_op("-")) a = mk(Expr::Binary, "-", {a, multiplicative()});
            else return a;
        }
    }
    ExprP multiplicative() {
        ExprP a = unary();
        while (true) {
            if (accept_op("*")) a = mk(Expr::Binary, "*", {a, unary()});
            else if (accept_op("//")) a = mk(Expr::Binary, "//", {a, unary()});
            else if (accept_op("/")) a = mk(Expr::Binary, "/", {a, unary()});
            else if (accept_op("%")) a = mk(Expr::Binary, "%", {a, unary()});
            else return a;
        }
    }
    ExprP unary() {
        if (accept_op("-")) {
            NestGuard g(depth_, "expression");
            return mk(Expr::Unary, "-", {unary()});
        }
        if (accept_op("+")) {
            NestGuard g(depth_, "expression");
            return unary();
        }
        return postfix(primary());
    }
    std::vector<ExprP> call_args() {  // after "("
        std::vector<ExprP> args;
        if (accept_op(")")) return args;
        do {
            if (t_[p_].k == Tok::Name && t_[p_ + 1].k == Tok::Op && t_[p_ + 1].s == "=")
                throw SyntaxError("keyword arguments are not supported");
            args.push_back(expr());
        } while (accept_op(","));
        expect_op(")");
        return args;
    }
    ExprP postfix(ExprP a) {
        while (true) {
            if (accept_op(".")) {
                if (t_[p_].k == Tok::Name) {
                    a = mk(Expr::Attr, t_[p_++].s, {a});
                } else if (t_[p_].k == Tok::Integer) {
                    auto idx = mk(Expr::Lit, "", {});
                    idx->lit = Val::integer(t_[p_++].i);
                    a = mk(Expr::Item, "", {a, idx});
                } else {
                    throw SyntaxError("expected an attribute name");
                }
            } else if (accept_op("[")) {
                ExprP lo, hi;
                if (!is_op(":")) lo = expr();
                if (accept_op(":")) {
                    if (!is_op("]")) hi = expr();
                    expect_op("]");
                    a = mk(Expr::Slice, "", {a, lo, hi});
                } else {
                    expect_op("]");
                    a = mk(Expr::Item, "", {a, lo});
                }
            } else if (accept_op("|")) {
                if (t_[p_].k != Tok::Name) throw SyntaxError("expected a filter name");
                const std::string f = t_[p_++].s;
                std::vector<ExprP> args{a};
                if (accept_op("(")) {
                    auto more = call_args();
                    args.insert(args.end(), more.begin(), more.end());
                }
                a = mk(Expr::Filter, f, args);
            } else if (is_op("(")) {
                if (a->k != Expr::Var) throw SyntaxError("only named functions can be called");
                ++p_;
                a = mk(Expr::Call, a->name, call_args());
            } else {
                return a;
            }
        }
    }
    ExprP primary() {
        const Tok& t = t_[p_];
        auto lit = [&](Val v) {
            auto e = mk(Expr::Lit, "", {});
            e->lit = std::move(v);
            ++p_;
            return e;
        };
        switch (t.k) {
            case Tok::String: {
                std::string s = t.s;
                ++p_;
                while (t_[p_].k == Tok::String) s += t_[p_++].s;  // adjacent literals join
                auto e = mk(Expr::Lit, "", {});
                e->lit = Val::str(s);
                return e;
            }
            case Tok::Integer: return lit(Val::integer(t.i));
            case Tok::Real: return lit(Val::real(t.f));
            case Tok::Name:
                if (t.s == "true" || t.s == "True") return lit(Val::boolean(true));
                if (t.s == "false" || t.s == "False") return lit(Val::boolean(false));
                if (t.s == "none" || t.s == "None") return lit(Val::none());
                ++p_;
                return mk(Expr::Var, t.s, {});
            case Tok::Op:
                if (t.s == "(") {
                    ++p_;
                    ExprP e = expr();
                    expect_op(")");
                    return e;
                }
                if (t.s == "[") {
                    ++p_;
                    std::vector<ExprP> items;
                    if (!accept_op("]")) {
                        do {
                            if (is_op("]")) break;
                            items.push_back(expr());
                        } while (accept_op(","));
                        expect_op("]");
                    }
                    return mk(Expr::ListLit, "", items);
                }
                throw SyntaxError("unexpected '" + t.s + "'");
            default: throw SyntaxError("unexpected end of expression");
        }
    }
};

struct Piece {
    enum Kind { Text, Out, Stmt } k;
    std::string s;
};

// Cuts the source into text, {{ }} and {% %} pieces ({# #} dropped),
// applying "-" whitespace control.
std::vector<Piece> cut(std::string src) {
    if (!src.empty() && src.back() == '\n') {  // keep_trailing_newline = false
        src.pop_back();
        if (!src.empty() && src.back() == '\r') src.pop_back();
    }
    std::vector<Piece> out;
    size_t p = 0;
    bool strip_next = false;
    auto is_ws = [](char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; };
    while (p <= src.size()) {
        size_t q = src.find('{', p);
        while (q != std::string::npos && q + 1 < src.size() && src[q + 1] != '{' && src[q + 1] != '%' &&
               src[q + 1] != '#')
            q = src.find('{', q + 1);
        if (q != std::string::npos && q + 1 >= src.size()) q = std::string::npos;
        std::string text = src.substr(p, q == std::string::npos ? std::string::npos : q - p);
        if (strip_next) {
            size_t a = 0;
            while (a < text.size() && is_ws(text[a])) ++a;
            text.erase(0, a);
        }
        if (q == std::string::npos) {
            if (!text.empty()) out.push_back(Piece{Piece::Text, text});
            break;
        }
        const char kind = src[q + 1];
        const char* close = kind == '{' ? "}}" : kind == '%' ? "%}" : "#}";
        size_t body = q + 2;
        if (body < src.size() && src[body] == '-') {
            while (!text.empty() && is_ws(text.back())) text.pop_back();
            ++body;
        } else if (body < src.size() && src[body] == '+') {
            ++body;
        }
        if (!text.empty()) out.push_back(Piece{Piece::Text, text});
        size_t e = src.find(close, body);
        if (kind != '#') {  // a closing delimiter inside a string literal does not end the tag
            size_t r = body;
            char quote = 0;
            for (; r < src.size(); ++r) {
                const char c = src[r];
                if (quote) {
                    if (c == '\\') ++r;
                    else if (c == quote) quote = 0;
                } else if (c == '\'' || c == '"') {
                    quote = c;
                } else if (src.compare(r, 2, close) == 0) {
                    break;
                }
            }
            e = r < src.size() ? r : std::string::npos;
        }
        if (e == std::string::npos) throw SyntaxError(std::string("unclosed tag, expected '") + close + "'");
        size_t inner_end = e;
        strip_next = false;
        if (inner_end > body && src[inner_end - 1] == '-') {
            strip_next = true;
            --inner_end;
        } else if (inner_end > body && src[inner_end - 1] == '+') {
            --inner_end;
        }
        const std::string inner = src.substr(body, inner_end - body);
        if (kind == '{') out.push_back(Piece{Piece::Out, inner});
        else if (kind == '%') out.push_back(Piece{Piece::Stmt, inner});
        p = e + 2;
    }
    return out;
}

class TemplateParser {
   public:
    explicit TemplateParser(std::vector<Piece> pieces) : ps_(std::move(pieces)) {}
    Body parse() {
        std::string stop;
        Body b = body({}, stop);
        if (!stop.empty()) throw SyntaxError("unexpected '" + stop + "'");
        return b;
    }

   private:
    std::vector<Piece> ps_;
    size_t i_ = 0;
    int depth_ = 0;
    std::vector<Tok> rest_;  // tokens after the keyword of the statement that ended the last body

    static std::vector<Tok> tokens_after_keyword(const std::string& stmt, std::string& kw) {
        std::vector<Tok> t = lex_expr(stmt);
        if (t.empty() || t[0].k != Tok::Name) throw SyntaxError("expected a statement keyword");
        kw = t[0].s;
        t.erase(t.begin());
        return t;
    }
    // Parses nodes until one of the stop keywords; `stop` receives it ("" at
    // the end of input) and rest_ the tokens after it.
    Body body(const std::vector<std::string>& stops, std::string& stop) {
        NestGuard g(depth_, "block");
        Body out;
        while (i_ < ps_.size()) {
            const Piece& pc = ps_[i_++];
            if (pc.k == Piece::Text) {
                auto n = std::make_shared<Node>();
                n->k = Node::Text;
                n->text = pc.s;
                out.push_back(n);
            } else if (pc.k == Piece::Out) {
                auto n = std::make_shared<Node>();
                n->k = Node::Out;
                n->expr = ExprParser(lex_expr(pc.s)).parse_all();
                out.push_back(n);
            } else {
                std::string kw;
                std::vector<Tok> t = tokens_after_keyword(pc.s, kw);
                for (const auto& s : stops)
                    if (kw == s) {
                        stop = kw;
                        rest_ = std::move(t);
                        return out;
                    }
                if (kw == "if") {
                    out.push_back(parse_if(std::move(t)));
                } else if (kw == "for") {
                    out.push_back(parse_for(std::move(t)));
                } else if (kw == "set") {
                    auto n = std::make_shared<Node>();
                    n->k = Node::Set;
                    n->targets.emplace_back();
                    ExprParser(std::move(t)).parse_set(n->targets[0], n->expr);
                    out.push_back(n);
                } else {
                    throw SyntaxError("unknown or unsupported statement '" + kw + "'");
                }
            }
        }
        stop.clear();
        return out;
    }
    static void expect_empty(const std::vector<Tok>& t, const char* what) {
        if (t.empty() || t[0].k != Tok::End) throw SyntaxError(std::string("unexpected tokens after ") + what);
    }
    NodeP parse_if(std::vector<Tok> cond) {
        auto n = std::make_shared<Node>();
        n->k = Node::If;
        ExprP c = ExprParser(std::move(cond)).parse_all();
        while (true) {
            std::string stop;
            Body b = body({"elif", "else", "endif"}, stop);
            if (stop.empty()) throw SyntaxError("missing endif");
            n->branches.emplace_back(c, std::move(b));
            if (stop == "elif") {
                c = ExprParser(std::move(rest_)).parse_all();
                continue;
            }
            if (stop == "else") {
                expect_empty(rest_, "else");
                n->else_body = body({"endif"}, stop);
                if (stop.empty()) throw SyntaxError("missing endif");
            }
            expect_empty(rest_, "endif");
            return n;
        }
    }
    NodeP parse_for(std::vector<Tok> head) {
        auto n = std::make_shared<Node>();
        n->k = Node::For;
        ExprParser(std::move(head)).parse_for(n->targets, n->expr);
        std::string stop;
        n->body = body({"else", "endfor"}, stop);
        if (stop.empty()) throw SyntaxError("missing endfor");
        if (stop == "else") {
            expect_empty(rest_, "else");
            n->else_body = body({"endfor"}, stop);
            if (stop.empty()) throw SyntaxError("missing endfor");
        }
        expect_empty(rest_, "endfor");
        return n;
    }
};

// ---------------------------------------------------------------- renderer
class Renderer {
   public:
    explicit Renderer(std::vector<std::map<std::string, Val>> scopes) : scopes_(std::move(scopes)) {}

    void run(const Body& b, std::string& out) {
        for (const auto& n : b) node(*n, out);
    }

   private:
    std::vector<std::map<std::string, Val>> scopes_;
    int depth_ = 0;

    Val lookup(const std::string& name) const {
        for (auto it = scopes_.rbegin(); it != scopes_.rend(); ++it) {
            const auto f = it->find(name);
            if (f != it->end()) return f->second;
        }
        return Val();
    }

    void node(const Node& n, std::string& out) {
        switch (n.k) {
            case Node::Text: out += n.text; break;
            case Node::Out: out += to_text(eval(*n.expr)); break;
            case Node::Set: scopes_.back()[n.targets[0]] = eval(*n.expr); break;
            case Node::If:
                for (const auto& br : n.branches)
                    if (eval(*br.first).truthy()) {
                        run(br.second, out);
                        return;
                    }
                run(n.else_body, out);
                break;
            case Node::For: {
                if (++depth_ > 64) throw RenderError("loops nested too deep");
                const Val seq = eval(*n.expr);
                List items;
                if (seq.k == Val::Seq) items = *seq.list;
                else if (seq.k == Val::Obj)
                    for (const auto& kv : *seq.map) items.push_back(Val::str(kv.first));
                else if (seq.k == Val::Str)
                    items = chars(seq.s);
                else if (seq.k != Val::Undef && seq.k != Val::None)
                    throw RenderError(kind_name(seq) + " is not iterable");
                if (items.empty()) {
                    run(n.else_body, out);
                } else {
                    const int64_t len = (int64_t)items.size();
                    for (int64_t j = 0; j < len; ++j) {
                        std::map<std::string, Val> sc;
                        const Val& it = items[(size_t)j];
                        if (n.targets.size() == 1) {
                            sc[n.targets[0]] = it;
                        } else {
                            if (it.k != Val::Seq || it.list->size() != n.targets.size())
                                throw RenderError("cannot unpack loop item");
                            for (size_t t = 0; t < n.targets.size(); ++t) sc[n.targets[t]] = (*it.list)[t];
                        }
                        sc["loop"] = Val::obj(Map{{"index", Val::integer(j + 1)},
                                                  {"index0", Val::integer(j)},
                                                  {"revindex", Val::integer(len - j)},
                                                  {"revindex0", Val::integer(len - j - 1)},
                                                  {"first", Val::boolean(j == 0)},
                                                  {"last", Val::boolean(j == len - 1)},
                                                  {"length", Val::integer(len)}});
                        scopes_.push_back(std::move(sc));
                        run(n.body, out);
                        scopes_.pop_back();
                    }
                }
                --depth_;
                break;
            }
        }
    }

    static List chars(const std::string& s) {
        List l;
        for (size_t p = 0; p < s.size();) {
            size_t q = p + 1;
            while (q < s.size() && ((unsigned char)s[q] & 0xC0) == 0x80) ++q;
            l.push_back(Val::str(s.substr(p, q - p)));
            p = q;
        }
        return l;
    }
    static int64_t index_of(const Val& v, int64_t len) {
        if (v.k != Val::Int) throw RenderError("sequence index must be an integer");
        return v.i < 0 ? v.i + len : v.i;
    }

    Val item(const Val& obj, const Val& key) {
        if (obj.k == Val::Undef) throw RenderError("cannot look up an item of an undefined value");
        if (obj.k == Val::Obj) {
            if (key.k != Val::Str) return Val();
            const Val* v = obj.find(key.s);
            return v ? *v : Val();
        }
        if (obj.k == Val::Seq) {
            const int64_t j = index_of(key, (int64_t)obj.list->size());
            return j >= 0 && j < (int64_t)obj.list->size() ? (*obj.list)[(size_t)j] : Val();
        }
        if (obj.k == Val::Str) {
            const List c = chars(obj.s);
            const int64_t j = index_of(key, (int64_t)c.size());
            return j >= 0 && j < (int64_t)c.size() ? c[(size_t)j] : Val();
        }
        return Val();
    }

    Val slice(const Val& v, const Expr* lo, const Expr* hi) {
        List src;
        if (v.k == Val::Seq) src = *v.list;
        else if (v.k == Val::Str) src = chars(v.s);
        else throw RenderError("cannot slice " + kind_name(v));
        const int64_t len = (int64_t)src.size();
        auto bound = [&](const Expr* e, int64_t dflt) {
            if (!e) return dflt;
            const Val b = eval(*e);
            if (b.k == Val::None || b.k == Val::Undef) return dflt;
            int64_t x = index_of(b, len);
            return x < 0 ? (int64_t)0 : x > len ? len : x;
        };
        const int64_t a = bound(lo, 0), b = bound(hi, len);
        List out;
        for (int64_t j = a; j < b; ++j) out.push_back(src[(size_t)j]);
        if (v.k == Val::Str) {
            std::string s;
            for (const auto& c : out) s += c.s;
            return Val::str(s);
        }
        return Val::seq(std::move(out));
    }

    static Val arith(const std::string& op, const Val& a, const Val& b) {
        if (op == "+" && a.k == Val::Str && b.k == Val::Str) return Val::str(a.s + b.s);
        if (op == "+" && a.k == Val::Seq && b.k == Val::Seq) {
            List l = *a.list;
            l.insert(l.end(), b.list->begin(), b.list->end());
            return Val::seq(std::move(l));
        }
        if (!a.number() || !b.number())
            throw RenderError("unsupported operand types for " + op + ": " + kind_name(a) + " and " + kind_name(b));
        if (a.k == Val::Int && b.k == Val::Int && op != "/") {
            if (op == "+") return Val::integer(a.i + b.i);
            if (op == "-") return Val::integer(a.i - b.i);
            if (op == "*") return Val::integer(a.i * b.i);
            if (b.i == 0) throw RenderError("division by zero");
            if (op == "//") {
                int64_t q = a.i / b.i;
                if ((a.i % b.i != 0) && ((a.i < 0) != (b.i < 0))) --q;
                return Val::integer(q);
            }
            int64_t r = a.i % b.i;
            if (r != 0 && ((r < 0) != (b.i < 0))) r += b.i;
            return Val::integer(r);
        }
        const double x = a.as_double(), y = b.as_double();
        if (op == "+") return Val::real(x + y);
        if (op == "-") return Val::real(x - y);
        if (op == "*") return Val::real(x * y);
        if (op == "/") return Val::real(x / y);
        if (op == "//") return Val::real(std::floor(x / y));
        return Val::real(std::fmod(x, y));
    }

    static bool contains(const Val& hay, const Val& needle) {
        if (hay.k == Val::Str) {
            if (needle.k != Val::Str) throw RenderError("'in' on a string needs a string");
            return hay.s.find(needle.s) != std::string::npos;
        }
        if (hay.k == Val::Seq) {
            for (const auto& e : *hay.list)
                if (equal(e, needle)) return true;
            return false;
        }
        if (hay.k == Val::Obj) return needle.k == Val::Str && hay.find(needle.s) != nullptr;
        if (hay.k == Val::Undef) return false;
        throw RenderError("cannot test membership in " + kind_name(hay));
    }

    static int compare_vals(const Val& a, const Val& b, const std::string& op) {
        if (a.number() && b.number()) {
            const double x = a.as_double(), y = b.as_double();
            return x < y ? -1 : x > y ? 1 : 0;
        }
        if (a.k == Val::Str && b.k == Val::Str) return a.s < b.s ? -1 : a.s > b.s ? 1 : 0;
        throw RenderError("cannot compare " + kind_name(a) + " " + op + " " + kind_name(b));
    }

    Val test(const Expr& e) {
        const Val v = eval(*e.args[0]);
        const std::string& t = e.name;
        bool r;
        if (t == "defined") r = v.k != Val::Undef;
        else if (t == "undefined") r = v.k == Val::Undef;
        else if (t == "none") r = v.k == Val::None;
        else if (t == "string") r = v.k == Val::Str;
        else if (t == "number") r = v.number();
        else if (t == "integer") r = v.k == Val::Int;
        else if (t == "float") r = v.k == Val::Float;
        else if (t == "boolean") r = v.k == Val::Bool;
        else if (t == "true") r = v.k == Val::Bool && v.b;
        else if (t == "false") r = v.k == Val::Bool && !v.b;
        else if (t == "mapping") r = v.k == Val::Obj;
        else if (t == "sequence") r = v.k == Val::Seq || v.k == Val::Str;
        else if (t == "iterable") r = v.k == Val::Seq || v.k == Val::Str || v.k == Val::Obj;
        else if (t == "odd" || t == "even") {
            if (v.k != Val::Int) throw RenderError("test " + t + " needs an integer");
            r = ((v.i % 2) != 0) == (t == "odd");
        } else {
            throw RenderError("unknown test '" + t + "'");
        }
        return Val::boolean(r != e.negate);
    }

    static std::string trim(const std::string& s) {
        size_t a = 0, b = s.size();
        while (a < b && isspace((unsigned char)s[a])) ++a;
        while (b > a && isspace((unsigned char)s[b - 1])) --b;
        return s.substr(a, b - a);
    }

    Val filter(const Expr& e) {
        const Val v = eval(*e.args[0]);
        const std::string& f = e.name;
        auto arg = [&](size_t j) { return j < e.args.size() ? eval(*e.args[j]) : Val(); };
        auto need_str = [&]() {
            if (v.k != Val::Str) throw RenderError("filter " + f + " needs a string, got " + kind_name(v));
        };
        if (f == "length" || f == "count") {
            if (v.k == Val::Str) return Val::integer((int64_t)chars(v.s).size());
            if (v.k == Val::Seq) return Val::integer((int64_t)v.list->size());
            if (v.k == Val::Obj) return Val::integer((int64_t)v.map->size());
            throw RenderError("filter length on " + kind_name(v));
        }
        if (f == "trim") { need_str(); return Val::str(trim(v.s)); }
        if (f == "upper" || f == "lower") {
            need_str();
            std::string s = v.s;
            for (char& c : s)
                if ((unsigned char)c < 128) c = (char)(f == "upper" ? toupper(c) : tolower(c));
            return Val::str(s);
        }
        if (f == "capitalize") {
            need_str();
            std::string s = v.s;
            for (size_t j = 0; j < s.size(); ++j)
                if ((unsigned char)s[j] < 128) s[j] = (char)(j == 0 ? toupper(s[j]) : tolower(s[j]));
            return Val::str(s);
        }
        if (f == "default" || f == "d") {
            const Val d = arg(1);
            const bool boolean = e.args.size() > 2 && eval(*e.args[2]).truthy();
            if (v.k == Val::Undef || (boolean && !v.truthy())) return d.k == Val::Undef ? Val::str("") : d;
            return v;
        }
        if (f == "first" || f == "last") {
            List l = v.k == Val::Str ? chars(v.s) : v.k == Val::Seq ? *v.list : List();
            if (v.k != Val::Str && v.k != Val::Seq) throw RenderError("filter " + f + " on " + kind_name(v));
            if (l.empty()) return Val();
            return f == "first" ? l.front() : l.back();
        }
        if (f == "string") return Val::str(to_text(v));
        if (f == "int") {
            if (v.k == Val::Int) return v;
            if (v.k == Val::Float) return Val::integer((int64_t)v.f);
            if (v.k == Val::Bool) return Val::integer(v.b ? 1 : 0);
            if (v.k == Val::Str) {
                char* end = nullptr;
                const std::string s = trim(v.s);
                const long long x = strtoll(s.c_str(), &end, 10);
                if (!s.empty() && end == s.c_str() + s.size()) return Val::integer(x);
                throw RenderError("cannot convert '" + v.s + "' to an integer");
            }
            throw RenderError("filter int on " + kind_name(v));
        }
        if (f == "join") {
            const Val sep = arg(1);
            List l = v.k == Val::Str ? chars(v.s) : v.k == Val::Seq ? *v.list : List();
            if (v.k != Val::Str && v.k != Val::Seq) throw RenderError("filter join on " + kind_name(v));
            std::string s;
            for (size_t j = 0; j < l.size(); ++j) {
                if (j) s += sep.k == Val::Str ? sep.s : to_text(sep);
                s += to_text(l[j]);
            }
            return Val::str(s);
        }
        if (f == "list") {
            if (v.k == Val::Seq) return v;
            if (v.k == Val::Str) return Val::seq(chars(v.s));
            if (v.k == Val::Obj) {
                List l;
                for (const auto& kv : *v.map) l.push_back(Val::str(kv.first));
                return Val::seq(l);
            }
            throw RenderError("filter list on " + kind_name(v));
        }
        if (f == "reverse") {
            if (v.k == Val::Seq) return Val::seq(List(v.list->rbegin(), v.list->rend()));
            if (v.k == Val::Str) {
                List c = chars(v.s);
                std::string s;
                for (auto it = c.rbegin(); it != c.rend(); ++it) s += it->s;
                return Val::str(s);
            }
            throw RenderError("filter reverse on " + kind_name(v));
        }
        throw RenderError("unknown filter '" + f + "'");
    }

    Val call(const Expr& e) {
        std::vector<Val> a;
        for (const auto& x : e.args) a.push_back(eval(*x));
        if (e.name == "raise_exception") throw RenderError(a.empty() ? "raise_exception" : to_text(a[0]));
        if (e.name == "range") {
            int64_t lo = 0, hi = 0, st = 1;
            for (const auto& x : a)
                if (x.k != Val::Int) throw RenderError("range() needs integers");
            if (a.size() == 1) hi = a[0].i;
            else if (a.size() >= 2) { lo = a[0].i; hi = a[1].i; }
            if (a.size() >= 3) st = a[2].i;
            if (a.empty() || a.size() > 3 || st == 0) throw RenderError("bad range() arguments");
            List l;
            for (int64_t x = lo; st > 0 ? x < hi : x > hi; x += st) {
                l.push_back(Val::integer(x));
                if (l.size() > 100000) throw RenderError("range() too large");
            }
            return Val::seq(std::move(l));
        }
        throw RenderError("unknown function '" + e.name + "'");
    }

    Val eval(const Expr& e) {
        switch (e.k) {
            case Expr::Lit: return e.lit;
            case Expr::Var: return lookup(e.name);
            case Expr::ListLit: {
                List l;
                for (const auto& x : e.args) l.push_back(eval(*x));
                return Val::seq(std::move(l));
            }
            case Expr::Attr: {
                const Val o = eval(*e.args[0]);
                if (o.k == Val::Undef) throw RenderError("cannot look up '" + e.name + "' of an undefined value");
                const Val* v = o.find(e.name);
                return v ? *v : Val();
            }
            case Expr::Item: return item(eval(*e.args[0]), eval(*e.args[1]));
            case Expr::Slice: return slice(eval(*e.args[0]), e.args[1].get(), e.args[2].get());
            case Expr::Unary: {
                const Val v = eval(*e.args[0]);
                if (e.name == "not") return Val::boolean(!v.truthy());
                if (v.k == Val::Int) return Val::integer(-v.i);
                if (v.k == Val::Float) return Val::real(-v.f);
                throw RenderError("cannot negate " + kind_name(v));
            }
            case Expr::Binary: {
                const std::string& op = e.name;
                if (op == "and") {
                    const Val a = eval(*e.args[0]);
                    return a.truthy() ? eval(*e.args[1]) : a;
                }
                if (op == "or") {
                    const Val a = eval(*e.args[0]);
                    return a.truthy() ? a : eval(*e.args[1]);
                }
                const Val a = eval(*e.args[0]), b = eval(*e.args[1]);
                if (op == "==") return Val::boolean(equal(a, b));
                if (op == "!=") return Val::boolean(!equal(a, b));
                if (op == "~") return Val::str(to_text(a) + to_text(b));
                if (op == "in") return Val::boolean(contains(b, a));
                if (op == "<") return Val::boolean(compare_vals(a, b, op) < 0);
                if (op == ">") return Val::boolean(compare_vals(a, b, op) > 0);
                if (op == "<=") return Val::boolean(compare_vals(a, b, op) <= 0);
                if (op == ">=") return Val::boolean(compare_vals(a, b, op) >= 0);
                return arith(op, a, b);
            }
            case Expr::Test: return test(e);
            case Expr::Filter: return filter(e);
            case Expr::Call: return call(e);
            case Expr::Cond: return eval(*e.args[0]).truthy() ? eval(*e.args[1]) : eval(*e.args[2]);
        }
        return Val();
    }
};

}  // namespace

bool render_chat_template(const std::string& source, const std::vector<ChatMessage>& messages,
                          bool add_generation_prompt, std::string& out, std::string& err) {
    Body tree;
    try {
        tree = TemplateParser(cut(source)).parse();
    } catch (const SyntaxError& e) {
        err = std::string("Failed to parse Jinja chat template: ") + e.what();
        return false;
    }
    List msgs;
    for (const auto& m : messages)
        msgs.push_back(Val::obj(Map{{"role", Val::str(m.role)}, {"content", Val::str(m.content)}}));
    std::map<std::string, Val> ctx;
    ctx["messages"] = Val::seq(std::move(msgs));
    ctx["add_generation_prompt"] = Val::boolean(add_generation_prompt);
    try {
        std::string o;
        Renderer({ctx}).run(tree, o);
        out = std::move(o);
    } catch (const RenderError& e) {
        err = std::string("Failed to render Jinja chat template: ") + e.what();
        return false;
    }
    return true;
}

}  // namespace krk
