// Jinja-subset chat template renderer (the semantics of minja, the engine the
// reference renders chat templates with; see chat_template.hpp for the scope).
#include "chat_template.hpp"

#include <algorithm>
#include <cctype>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <map>
#include <stdexcept>

namespace minfer {

// ---------------------------------------------------------------------------
// values

Value Value::array(Arr a) {
    Value v;
    v.k_ = ARR;
    v.a_ = std::make_shared<Arr>(std::move(a));
    return v;
}
Value Value::object() {
    Value v;
    v.k_ = OBJ;
    v.o_ = std::make_shared<Obj>();
    return v;
}
Value Value::function(Fn f) {
    // a callable is also an (empty) object: it prints as {}, counts as a
    // mapping, is true, and can carry attributes (a loop's cycle, ...)
    Value v = object();
    v.fn_ = std::make_shared<Fn>(std::move(f));
    return v;
}

int64_t Value::i() const {
    switch (k_) {
        case INT: return i_;
        case FLOAT: return (int64_t)f_;
        default: throw std::runtime_error("type must be number: " + dump());
    }
}
double Value::f() const {
    switch (k_) {
        case INT: return (double)i_;
        case FLOAT: return f_;
        default: throw std::runtime_error("type must be number: " + dump());
    }
}
const std::string& Value::str() const {
    if (k_ != STR) throw std::runtime_error("not a string: " + dump());
    return s_;
}
Value::Arr& Value::arr() const {
    if (k_ != ARR) throw std::runtime_error("Value is not an array: " + dump());
    return *a_;
}
Value::Obj& Value::obj() const {
    if (k_ != OBJ) throw std::runtime_error("Value is not an object: " + dump());
    return *o_;
}
Value Value::call(CallArgs& a) const {
    if (!fn_) throw std::runtime_error("Value is not callable: " + dump());
    return (*fn_)(a);
}
void Value::push(Value v) { arr().push_back(std::move(v)); }
void Value::set(const std::string& key, Value v) {
    for (auto& kv : obj())
        if (kv.first == key) {
            kv.second = std::move(v);
            return;
        }
    o_->emplace_back(key, std::move(v));
}
const Value* Value::find(const std::string& key) const {
    if (k_ != OBJ) return nullptr;
    for (const auto& kv : *o_)
        if (kv.first == key) return &kv.second;
    return nullptr;
}
void Value::erase(const std::string& key) {
    auto& o = obj();
    for (size_t i = 0; i < o.size(); ++i)
        if (o[i].first == key) {
            o.erase(o.begin() + (long)i);
            return;
        }
}
size_t Value::size() const {
    switch (k_) {
        case OBJ: return o_->size();
        case ARR: return a_->size();
        case STR: return s_.size();  // bytes
        default: throw std::runtime_error("Value is not an array or object: " + dump());
    }
}

bool Value::truthy() const {
    switch (k_) {
        case NUL: return false;
        case BOOL: return b_;
        case INT: return i_ != 0;
        case FLOAT: return f_ != 0;
        case STR: return !s_.empty();
        case ARR: return !a_->empty();
        default: return true;  // objects (even empty) and functions
    }
}

namespace {

// Well-formed UTF-8 (no overlong forms, surrogates or code points past
// U+10FFFF): what a JSON writer accepts.
bool valid_utf8(const std::string& s) {
    const auto* p = reinterpret_cast<const unsigned char*>(s.data());
    const size_t n = s.size();
    for (size_t i = 0; i < n;) {
        const unsigned c = p[i];
        size_t len;
        unsigned lo = 0x80, hi = 0xBF;
        if (c < 0x80) {
            ++i;
            continue;
        } else if (c >= 0xC2 && c <= 0xDF) {
            len = 2;
        } else if (c >= 0xE0 && c <= 0xEF) {
            len = 3;
            if (c == 0xE0) lo = 0xA0;
            if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            len = 4;
            if (c == 0xF0) lo = 0x90;
            if (c == 0xF4) hi = 0x8F;
        } else {
            return false;
        }
        if (i + len > n || p[i + 1] < lo || p[i + 1] > hi) return false;
        for (size_t k = 2; k < len; ++k)
            if ((p[i + k] & 0xC0) != 0x80) return false;
        i += len;
    }
    return true;
}

// JSON text of a string: quotes, backslash and control characters escaped
// (\b \f \n \r \t, others as \u00xx); other bytes unchanged. Text that is
// not UTF-8 cannot be written as JSON (the reference's engine throws too).
std::string json_quote(const std::string& s) {
    if (!valid_utf8(s)) throw std::runtime_error("invalid UTF-8 in a string written as JSON");
    std::string out = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\b': out += "\\b"; break;
            case '\f': out += "\\f"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            default:
                if (c < 0x20) {
                    char buf[8];
                    std::snprintf(buf, sizeof(buf), "\\u%04x", c);
                    out += buf;
                } else {
                    out += (char)c;
                }
        }
    }
    return out + "\"";
}

// Python-style repr: single quotes unless the text holds one
std::string py_quote(const std::string& s) {
    const std::string j = json_quote(s);
    if (s.find('\'') != std::string::npos) return j;
    std::string out = "'";
    for (size_t i = 1; i + 1 < j.size(); ++i) {
        if (j[i] == '\\' && j[i + 1] == '"') {
            out += '"';
            ++i;
        } else {
            out += j[i];
        }
    }
    return out + "'";
}

// Shortest decimal that reads back as x, laid out as JSON writers commonly do:
// fixed notation with a ".0" for integral values while the decimal point sits
// within 15 digits (and 0.000ddd down to 1e-4), else d.ddde+XX.
std::string fmt_double(double x) {
    if (!std::isfinite(x)) return "null";
    if (x == 0) return std::signbit(x) ? "-0.0" : "0.0";
    char buf[40];
    int prec = 1;
    for (; prec <= 17; ++prec) {
        std::snprintf(buf, sizeof(buf), "%.*e", prec - 1, x);
        if (std::strtod(buf, nullptr) == x) break;
    }
    // buf = [-]d.ddddde[+-]XX: digits and decimal exponent
    std::string s(buf), sign;
    if (s[0] == '-') {
        sign = "-";
        s = s.substr(1);
    }
    const size_t epos = s.find('e');
    const int e10 = std::atoi(s.c_str() + epos + 1);
    std::string digits;
    for (size_t i = 0; i < epos; ++i)
        if (s[i] != '.') digits += s[i];
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    const int k = (int)digits.size(), n = e10 + 1;  // value = 0.digits * 10^n
    std::string out;
    if (k <= n && n <= 15) {
        out = digits + std::string(n - k, '0') + ".0";
    } else if (0 < n && n <= 15) {
        out = digits.substr(0, n) + "." + digits.substr(n);
    } else if (-4 < n && n <= 0) {
        out = "0." + std::string(-n, '0') + digits;
    } else {
        out = digits.substr(0, 1);
        if (k > 1) out += "." + digits.substr(1);
        char eb[16];
        std::snprintf(eb, sizeof(eb), "e%c%02d", n - 1 < 0 ? '-' : '+', std::abs(n - 1));
        out += eb;
    }
    return sign + out;
}

}  // namespace

void Value::dump_to(std::string& out, int indent, int level, bool json) const {
    auto nl = [&](int lv) {
        if (indent > 0) {
            out += '\n';
            out.append((size_t)lv * indent, ' ');
        }
    };
    auto sep = [&]() {
        out += ',';
        if (indent < 0)
            out += ' ';
        else
            nl(level + 1);
    };
    switch (k_) {
        case NUL: out += "null"; break;
        case BOOL: out += json ? (b_ ? "true" : "false") : (b_ ? "True" : "False"); break;
        case INT: out += std::to_string(i_); break;
        case FLOAT: out += fmt_double(f_); break;
        case STR: out += json ? json_quote(s_) : py_quote(s_); break;
        case ARR:
            out += '[';
            nl(level + 1);
            for (size_t i = 0; i < a_->size(); ++i) {
                if (i) sep();
                (*a_)[i].dump_to(out, indent, level + 1, json);
            }
            nl(level);
            out += ']';
            break;
        case OBJ:
            out += '{';
            nl(level + 1);
            for (size_t i = 0; i < o_->size(); ++i) {
                if (i) sep();
                out += json ? json_quote((*o_)[i].first) : py_quote((*o_)[i].first);
                out += ": ";
                (*o_)[i].second.dump_to(out, indent, level + 1, json);
            }
            nl(level);
            out += '}';
            break;
    }
}

std::string Value::json_text(int indent) const {
    std::string out;
    std::function<void(const Value&, int)> put = [&](const Value& v, int level) {
        auto pad = [&](int lv) {
            out += '\n';
            out.append((size_t)lv * indent, ' ');
        };
        switch (v.k_) {
            case ARR:
                if (v.a_->empty()) {
                    out += "[]";
                    return;
                }
                out += '[';
                for (size_t i = 0; i < v.a_->size(); ++i) {
                    if (i) out += ',';
                    if (indent >= 0) pad(level + 1);
                    put((*v.a_)[i], level + 1);
                }
                if (indent >= 0) pad(level);
                out += ']';
                return;
            case OBJ:
                if (v.o_->empty()) {
                    out += "{}";
                    return;
                }
                out += '{';
                for (size_t i = 0; i < v.o_->size(); ++i) {
                    if (i) out += ',';
                    if (indent >= 0) pad(level + 1);
                    out += json_quote((*v.o_)[i].first);
                    out += indent >= 0 ? ": " : ":";
                    put((*v.o_)[i].second, level + 1);
                }
                if (indent >= 0) pad(level);
                out += '}';
                return;
            default: v.dump_to(out, -1, 0, true);
        }
    };
    put(*this, 0);
    return out;
}

std::string Value::dump(int indent, bool json) const {
    std::string out;
    dump_to(out, indent, 0, json);
    return out;
}

std::string Value::to_str() const {
    switch (k_) {
        case STR: return s_;
        case INT: return std::to_string(i_);
        case FLOAT: return std::to_string(f_);
        case BOOL: return b_ ? "True" : "False";
        case NUL: return "None";
        default: return dump();
    }
}

bool Value::equals(const Value& o) const {
    if ((fn_ || o.fn_) && fn_ != o.fn_) return false;  // (the same callable: compared as objects below)
    if (k_ == ARR) {
        if (o.k_ != ARR || a_->size() != o.a_->size()) return false;
        for (size_t i = 0; i < a_->size(); ++i) {
            const Value &x = (*a_)[i], &y = (*o.a_)[i];
            if (!x.truthy() || !y.truthy() || !x.equals(y)) return false;  // (falsy elements never compare equal)
        }
        return true;
    }
    if (k_ == OBJ) {
        if (o.k_ != OBJ || o_->size() != o.o_->size()) return false;
        for (const auto& kv : *o_) {
            const Value* y = o.find(kv.first);
            if (!kv.second.truthy() || !y || !kv.second.equals(*y)) return false;
        }
        return true;
    }
    // a scalar against a container compares the container's (null) scalar part
    if (o.k_ == ARR || o.k_ == OBJ) return k_ == NUL;
    if (is_number() && o.is_number()) {
        if (k_ == INT && o.k_ == INT) return i_ == o.i_;
        return f() == o.f();
    }
    if (k_ != o.k_) return false;
    switch (k_) {
        case NUL: return true;
        case BOOL: return b_ == o.b_;
        case STR: return s_ == o.s_;
        default: return false;
    }
}

// ---------------------------------------------------------------------------
// JSON input

namespace {

struct JsonParser {
    const std::string& s;
    size_t p = 0;
    [[noreturn]] void fail(const char* what) {
        throw std::invalid_argument(std::string("JSON: ") + what + " at offset " + std::to_string(p));
    }
    void ws() {
        while (p < s.size() && (s[p] == ' ' || s[p] == '\t' || s[p] == '\n' || s[p] == '\r')) ++p;
    }
    static void put_utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += (char)cp;
        } else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (p + 4 > s.size()) fail("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = s[p++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else fail("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        ++p;  // opening quote
        std::string out;
        while (true) {
            if (p >= s.size()) fail("unterminated string");
            const char c = s[p++];
            if (c == '"') return out;
            if ((unsigned char)c < 0x20) fail("control character in string");
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p >= s.size()) fail("unterminated escape");
            const char e = s[p++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp <= 0xDBFF) {
                        if (p + 2 > s.size() || s[p] != '\\' || s[p + 1] != 'u') fail("lone surrogate");
                        p += 2;
                        const uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo > 0xDFFF) fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
                        fail("lone surrogate");
                    }
                    put_utf8(out, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
    }
    Value value(int depth) {
        if (depth > 512) fail("nesting too deep");
        ws();
        if (p >= s.size()) fail("unexpected end");
        const char c = s[p];
        if (c == '{') {
            ++p;
            Value o = Value::object();
            ws();
            if (p < s.size() && s[p] == '}') {
                ++p;
                return o;
            }
            while (true) {
                ws();
                if (p >= s.size() || s[p] != '"') fail("expected key");
                std::string k = string();
                ws();
                if (p >= s.size() || s[p] != ':') fail("expected ':'");
                ++p;
                o.set(k, value(depth + 1));
                ws();
                if (p < s.size() && s[p] == ',') {
                    ++p;
                    continue;
                }
                if (p < s.size() && s[p] == '}') {
                    ++p;
                    return o;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p;
            Value a = Value::array();
            ws();
            if (p < s.size() && s[p] == ']') {
                ++p;
                return a;
            }
            while (true) {
                a.push(value(depth + 1));
                ws();
                if (p < s.size() && s[p] == ',') {
                    ++p;
                    continue;
                }
                if (p < s.size() && s[p] == ']') {
                    ++p;
                    return a;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') return Value(string());
        if (s.compare(p, 4, "true") == 0) {
            p += 4;
            return Value(true);
        }
        if (s.compare(p, 5, "false") == 0) {
            p += 5;
            return Value(false);
        }
        if (s.compare(p, 4, "null") == 0) {
            p += 4;
            return Value();
        }
        const size_t b = p;
        if (s[p] == '-') ++p;
        if (p >= s.size() || !std::isdigit((unsigned char)s[p])) fail("bad value");
        bool is_float = false;
        while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
        if (p < s.size() && s[p] == '.') {
            is_float = true;
            ++p;
            while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
        }
        if (p < s.size() && (s[p] == 'e' || s[p] == 'E')) {
            is_float = true;
            ++p;
            if (p < s.size() && (s[p] == '+' || s[p] == '-')) ++p;
            while (p < s.size() && std::isdigit((unsigned char)s[p])) ++p;
        }
        const std::string num = s.substr(b, p - b);
        if (!is_float) {
            errno = 0;
            const long long v = std::strtoll(num.c_str(), nullptr, 10);
            if (errno != ERANGE) return Value((int64_t)v);
        }
        return Value(std::strtod(num.c_str(), nullptr));
    }
};

}  // namespace

Value parse_json(const std::string& text) {
    JsonParser jp{text};
    Value v = jp.value(0);
    jp.ws();
    if (jp.p != text.size()) jp.fail("trailing characters");
    return v;
}

// ---------------------------------------------------------------------------
// expressions

namespace {

struct Context {
    std::map<std::string, Value> vars;
    std::shared_ptr<Context> parent;
    const Value* lookup(const std::string& n) const {
        for (const Context* c = this; c; c = c->parent.get()) {
            auto it = c->vars.find(n);
            if (it != c->vars.end()) return &it->second;
        }
        return nullptr;
    }
    Value get(const std::string& n) const {
        const Value* v = lookup(n);
        return v ? *v : Value();
    }
    void set(const std::string& n, Value v) { vars[n] = std::move(v); }
};
using Ctx = std::shared_ptr<Context>;

struct LoopControl {
    bool brk;
};

struct Expr;
using ExprP = std::shared_ptr<Expr>;
struct Expr {
    enum Kind { LIT, VAR, ARRAY, DICT, SUB, SLICE, ATTR_CALL, CALL, FILTER, UNARY, BIN, IS, IFX } kind;
    Value lit;
    std::string name;                 // VAR name, method name, IS test, operator
    std::vector<ExprP> items;         // ARRAY elements, FILTER parts, DICT keys/values interleaved
    ExprP a, b, c;                    // operands; SLICE start/end/step; IFX cond/then/else
    std::vector<ExprP> args;          // call arguments
    std::vector<std::pair<std::string, ExprP>> kwargs;
    bool negate = false;              // IS NOT
    explicit Expr(Kind k) : kind(k) {}
};

Value eval(const Expr& e, const Ctx& ctx);

// The context of the expression that calls a callable (a macro evaluates
// its parameters' defaults there).
thread_local const Ctx* g_caller = nullptr;
struct CallerScope {
    const Ctx* saved;
    explicit CallerScope(const Ctx& c) : saved(g_caller) { g_caller = &c; }
    ~CallerScope() { g_caller = saved; }
};

Value::Arr::size_type wrap_index(int64_t i, size_t n) { return (size_t)(i < 0 ? i + (int64_t)n : i); }

bool contains_value(const Value& item, const Value& container) {
    if (container.is_array()) {
        for (const Value& x : container.arr())
            if (x.truthy() && x.equals(item)) return true;
        return false;
    }
    if (container.is_object()) {
        if (item.is_array() || item.is_object() || item.is_callable())
            throw std::runtime_error("Unhashable type: " + item.dump());
        return item.is_string() && container.find(item.str()) != nullptr;
    }
    return item.is_string() && container.is_string() && container.str().find(item.str()) != std::string::npos;
}

Value get_item(const Value& t, const Value& key) {
    if (t.is_array()) {
        if (key.kind() != Value::INT) return Value();
        const size_t i = wrap_index(key.i(), t.arr().size());
        if (i >= t.arr().size()) throw std::out_of_range("array index out of range");
        return t.arr()[i];
    }
    if (t.is_object()) {
        if (key.is_array() || key.is_object() || key.is_callable())
            throw std::runtime_error("Unhashable type: " + t.dump());
        if (!key.is_string()) return Value();
        const Value* v = t.find(key.str());
        return v ? *v : Value();
    }
    return Value();
}

bool less(const Value& l, const Value& r) {
    if (l.is_null()) throw std::runtime_error("Undefined value or reference");
    if (l.is_number() && r.is_number()) return l.f() < r.f();
    if (l.is_string() && r.is_string()) return l.str() < r.str();
    throw std::runtime_error("Cannot compare values: " + l.dump() + " < " + r.dump());
}
bool greater(const Value& l, const Value& r) {
    if (l.is_null()) throw std::runtime_error("Undefined value or reference");
    if (l.is_number() && r.is_number()) return l.f() > r.f();
    if (l.is_string() && r.is_string()) return l.str() > r.str();
    throw std::runtime_error("Cannot compare values: " + l.dump() + " > " + r.dump());
}

Value binary(const std::string& op, const Value& l, const Value& r) {
    const bool ii = l.kind() == Value::INT && r.kind() == Value::INT;
    if (op == "~") return Value(l.to_str() + r.to_str());
    if (op == "+") {
        if (l.is_string() || r.is_string()) return Value(l.to_str() + r.to_str());
        if (ii) return Value(l.i() + r.i());
        if (l.is_array() && r.is_array()) {
            Value::Arr a = l.arr();
            a.insert(a.end(), r.arr().begin(), r.arr().end());
            return Value::array(std::move(a));
        }
        return Value(l.f() + r.f());
    }
    if (op == "-") return ii ? Value(l.i() - r.i()) : Value(l.f() - r.f());
    if (op == "*") {
        if (l.is_string() && r.kind() == Value::INT) {
            std::string out;
            for (int64_t i = 0; i < r.i(); ++i) out += l.to_str();
            return Value(out);
        }
        return ii ? Value(l.i() * r.i()) : Value(l.f() * r.f());
    }
    if (op == "/") {
        if (ii) {
            if (r.i() == 0) throw std::runtime_error("division by zero");
            return Value(l.i() / r.i());
        }
        return Value(l.f() / r.f());
    }
    if (op == "**") return Value(std::pow(l.f(), r.f()));
    if (op == "//" || op == "%") {
        const int64_t a = l.i(), b = r.i();
        if (b == 0) throw std::runtime_error("division by zero");
        return Value(op == "//" ? a / b : a % b);
    }
    if (op == "==") return Value(l.equals(r));
    if (op == "!=") return Value(!l.equals(r));
    if (op == "<") return Value(less(l, r));
    if (op == ">") return Value(greater(l, r));
    if (op == "<=") return Value(!greater(l, r));
    if (op == ">=") return Value(!less(l, r));
    if (op == "in") return Value(contains_value(l, r));
    if (op == "not in") return Value(!contains_value(l, r));
    throw std::runtime_error("Unknown binary operator " + op);
}

bool is_test(const std::string& t, const Value& v) {
    if (t == "none") return v.is_null();
    if (t == "boolean") return v.kind() == Value::BOOL;
    if (t == "integer") return v.kind() == Value::INT;
    if (t == "float") return v.kind() == Value::FLOAT;
    if (t == "number") return v.is_number();
    if (t == "string") return v.is_string();
    if (t == "mapping") return v.is_object();
    if (t == "iterable") return v.is_array() || v.is_object() || v.is_string();
    if (t == "sequence") return v.is_array();
    if (t == "defined") return !v.is_null();
    if (t == "true") return v.truthy();
    if (t == "false") return !v.truthy();
    throw std::runtime_error("Unknown type for 'is' operator: " + t);
}

CallArgs eval_args(const Expr& e, const Ctx& ctx) {
    CallArgs a;
    for (const auto& x : e.args) {
        if (x->kind == Expr::UNARY && x->name == "*") {  // *list: its items as positional arguments
            Value v = eval(*x->a, ctx);
            if (!v.is_array()) throw std::runtime_error("Expansion operator only supported on arrays");
            for (const Value& item : v.arr()) a.pos.push_back(item);
            continue;
        }
        if (x->kind == Expr::UNARY && x->name == "**") {  // **dict: its entries as keyword arguments
            Value v = eval(*x->a, ctx);
            if (!v.is_object()) throw std::runtime_error("ExpansionDict operator only supported on objects");
            for (const auto& kv : v.obj()) a.kw.emplace_back(kv.first, kv.second);
            continue;
        }
        a.pos.push_back(eval(*x, ctx));
    }
    for (const auto& kv : e.kwargs) a.kw.emplace_back(kv.first, eval(*kv.second, ctx));
    return a;
}

void expect_args(const CallArgs& a, const char* name, size_t pmin, size_t pmax, size_t kmin, size_t kmax) {
    if (a.pos.size() < pmin || a.pos.size() > pmax || a.kw.size() < kmin || a.kw.size() > kmax)
        throw std::runtime_error(std::string(name) + ": wrong number of arguments");
}

std::string strip_chars(const std::string& s, const std::string& chars, bool left, bool right) {
    const std::string set = chars.empty() ? " \t\n\r" : chars;
    const size_t b = left ? s.find_first_not_of(set) : 0;
    if (b == std::string::npos) return "";
    const size_t e = right ? s.find_last_not_of(set) : s.size() - 1;
    return s.substr(b, e - b + 1);
}

Value method_call(const Value& obj, const std::string& m, CallArgs& a) {
    if (obj.is_null()) throw std::runtime_error("Trying to call method '" + m + "' on null");
    if (obj.is_array()) {
        auto& arr = obj.arr();
        if (m == "append") {
            expect_args(a, "append", 1, 1, 0, 0);
            arr.push_back(a.pos[0]);
            return Value();
        }
        if (m == "pop") {
            expect_args(a, "pop", 0, 1, 0, 0);
            if (arr.empty()) throw std::runtime_error("pop from empty list");
            if (a.pos.empty()) {
                Value v = arr.back();
                arr.pop_back();
                return v;
            }
            const size_t i = wrap_index(a.pos[0].i(), arr.size());
            if (i >= arr.size()) throw std::runtime_error("pop index out of range");
            Value v = arr[i];
            arr.erase(arr.begin() + (long)i);
            return v;
        }
        if (m == "insert") {
            expect_args(a, "insert", 2, 2, 0, 0);
            const int64_t i = a.pos[0].i();
            if (i < 0 || i > (int64_t)arr.size()) throw std::runtime_error("Index out of range for insert method");
            arr.insert(arr.begin() + i, a.pos[1]);
            return Value();
        }
    } else if (obj.is_object()) {
        if (m == "items") {
            expect_args(a, "items", 0, 0, 0, 0);
            Value r = Value::array();
            for (const auto& kv : obj.obj()) r.push(Value::array({Value(kv.first), kv.second}));
            return r;
        }
        if (m == "keys") {
            expect_args(a, "keys", 0, 0, 0, 0);
            Value r = Value::array();
            for (const auto& kv : obj.obj()) r.push(Value(kv.first));
            return r;
        }
        if (m == "get") {
            expect_args(a, "get", 1, 2, 0, 0);
            const Value* v = a.pos[0].is_string() ? obj.find(a.pos[0].str()) : nullptr;
            return v ? *v : (a.pos.size() == 2 ? a.pos[1] : Value());
        }
        if (m == "pop") {
            expect_args(a, "pop", 1, 1, 0, 0);
            auto& o = obj.obj();
            for (size_t i = 0; i < o.size(); ++i)
                if (a.pos[0].is_string() && o[i].first == a.pos[0].str()) {
                    Value v = o[i].second;
                    o.erase(o.begin() + (long)i);
                    return v;
                }
            throw std::runtime_error("key not found: " + a.pos[0].dump());
        }
        if (const Value* f = obj.find(m)) {
            if (!f->is_callable()) throw std::runtime_error("Property '" + m + "' is not callable");
            return f->call(a);
        }
    } else if (obj.is_string()) {
        std::string s = obj.str();
        auto chars = [&]() { return a.pos.empty() ? std::string() : a.pos[0].str(); };
        if (m == "strip" || m == "lstrip" || m == "rstrip") {
            expect_args(a, m.c_str(), 0, 1, 0, 0);
            return Value(strip_chars(s, chars(), m != "rstrip", m != "lstrip"));
        }
        if (m == "split") {
            expect_args(a, "split", 1, 1, 0, 0);
            const std::string sep = a.pos[0].str();
            Value r = Value::array();
            size_t start = 0, end;
            while ((end = s.find(sep, start)) != std::string::npos) {
                r.push(Value(s.substr(start, end - start)));
                start = end + sep.size();
                if (sep.empty()) throw std::runtime_error("empty separator");
            }
            r.push(Value(s.substr(start)));
            return r;
        }
        if (m == "capitalize") {
            expect_args(a, "capitalize", 0, 0, 0, 0);
            if (!s.empty()) s[0] = (char)std::toupper((unsigned char)s[0]);
            return Value(s);
        }
        if (m == "upper" || m == "lower") {
            expect_args(a, m.c_str(), 0, 0, 0, 0);
            for (char& c : s) c = (char)(m == "upper" ? std::toupper((unsigned char)c) : std::tolower((unsigned char)c));
            return Value(s);
        }
        if (m == "endswith" || m == "startswith") {
            expect_args(a, m.c_str(), 1, 1, 0, 0);
            const std::string& x = a.pos[0].str();
            if (x.size() > s.size()) return Value(false);
            return Value(m == "startswith" ? s.compare(0, x.size(), x) == 0
                                           : s.compare(s.size() - x.size(), x.size(), x) == 0);
        }
        if (m == "title") {
            expect_args(a, "title", 0, 0, 0, 0);
            for (size_t i = 0; i < s.size(); ++i)
                s[i] = (char)(i == 0 || std::isspace((unsigned char)s[i - 1]) ? std::toupper((unsigned char)s[i])
                                                                             : std::tolower((unsigned char)s[i]));
            return Value(s);
        }
        if (m == "replace") {
            expect_args(a, "replace", 2, 3, 0, 0);
            const std::string before = a.pos[0].str(), after = a.pos[1].str();
            int64_t count = a.pos.size() == 3 ? a.pos[2].i() : (int64_t)s.size();
            size_t pos = 0;
            while ((pos = s.find(before, pos)) != std::string::npos && count-- > 0) {
                s.replace(pos, before.size(), after);
                pos += after.size();
            }
            return Value(s);
        }
    }
    throw std::runtime_error("Unknown method: " + m);
}

// a binary operator or test whose left side is evaluated
Value apply_operator(const Expr& e, const Value& l, const Ctx& ctx) {
    if (e.kind == Expr::IS) {
        const bool r = is_test(e.name, l);
        return Value(e.negate ? !r : r);
    }
    if (e.name == "and") return l.truthy() ? Value(eval(*e.b, ctx).truthy()) : Value(false);
    if (e.name == "or") return l.truthy() ? l : eval(*e.b, ctx);
    return binary(e.name, l, eval(*e.b, ctx));
}

Value eval(const Expr& e, const Ctx& ctx) {
    switch (e.kind) {
        case Expr::LIT: return e.lit;
        case Expr::VAR: return ctx->get(e.name);
        case Expr::ARRAY: {
            Value r = Value::array();
            for (const auto& x : e.items) r.push(eval(*x, ctx));
            return r;
        }
        case Expr::DICT: {
            Value r = Value::object();
            for (size_t i = 0; i + 1 < e.items.size(); i += 2) {
                Value k = eval(*e.items[i], ctx);
                if (k.is_array() || k.is_object() || k.is_callable()) throw std::runtime_error("Unhashable type");
                r.set(k.to_str(), eval(*e.items[i + 1], ctx));
            }
            return r;
        }
        case Expr::SUB: {
            Value t = eval(*e.a, ctx);
            if (e.b->kind == Expr::SLICE) {
                const Expr& sl = *e.b;
                const int64_t len = (int64_t)t.size();
                auto wrap = [len](int64_t i) { return i < 0 ? i + len : i; };
                const int64_t step = sl.c ? eval(*sl.c, ctx).i() : 1;
                if (!step) throw std::runtime_error("slice step cannot be zero");
                const int64_t start = sl.a ? wrap(eval(*sl.a, ctx).i()) : (step < 0 ? len - 1 : 0);
                const int64_t end = sl.b ? wrap(eval(*sl.b, ctx).i()) : (step < 0 ? -1 : len);
                if (t.is_string()) {
                    const std::string& s = t.str();
                    if (start < end && step == 1) {
                        if (start > len) throw std::out_of_range("slice start out of range");
                        return Value(s.substr((size_t)start, (size_t)(end - start)));
                    }
                    std::string r;
                    for (int64_t i = start; step > 0 ? i < end : i > end; i += step) {
                        if (i < 0 || i >= len) throw std::out_of_range("string index out of range");
                        r += s[(size_t)i];
                    }
                    return Value(r);
                }
                if (t.is_array()) {
                    Value r = Value::array();
                    for (int64_t i = start; step > 0 ? i < end : i > end; i += step) {
                        if (i < 0 || i >= len) throw std::out_of_range("array index out of range");
                        r.push(t.arr()[(size_t)i]);
                    }
                    return r;
                }
                throw std::runtime_error("Subscripting only supported on arrays and strings");
            }
            Value k = eval(*e.b, ctx);
            if (t.is_null()) {
                if (e.a->kind == Expr::VAR)
                    throw std::runtime_error("'" + e.a->name + "' is " +
                                             (ctx->lookup(e.a->name) ? "null" : "not defined"));
                throw std::runtime_error("Trying to access property '" + k.dump() + "' on null!");
            }
            return get_item(t, k);
        }
        case Expr::ATTR_CALL: {
            Value o = eval(*e.a, ctx);
            CallArgs a = eval_args(e, ctx);
            CallerScope cs(ctx);
            return method_call(o, e.name, a);
        }
        case Expr::CALL: {
            Value f = eval(*e.a, ctx);
            if (!f.is_callable()) throw std::runtime_error("Object is not callable: " + f.dump(2));
            CallArgs a = eval_args(e, ctx);
            CallerScope cs(ctx);
            return f.call(a);
        }
        case Expr::FILTER: {
            Value r = eval(*e.items[0], ctx);
            for (size_t i = 1; i < e.items.size(); ++i) {
                const Expr& p = *e.items[i];
                CallArgs a;
                Value f;
                if (p.kind == Expr::CALL) {
                    f = eval(*p.a, ctx);
                    a = eval_args(p, ctx);
                } else {
                    f = eval(p, ctx);
                }
                a.pos.insert(a.pos.begin(), r);
                CallerScope cs(ctx);
                r = f.call(a);
            }
            return r;
        }
        case Expr::UNARY: {
            if (e.name == "*" || e.name == "**")
                throw std::runtime_error("Expansion operator is only supported in function calls and collections");
            Value v = eval(*e.a, ctx);
            if (e.name == "not") return Value(!v.truthy());
            if (e.name == "-") return v.kind() == Value::INT ? Value(-v.i()) : Value(-v.f());
            return v;
        }
        case Expr::BIN:
        case Expr::IS: {
            Value l = eval(*e.a, ctx);
            if (l.is_callable()) {
                // an operator on a callable makes a callable: called, it calls
                // the left side and applies the operator to the result
                const Expr* ep = &e;
                Ctx c = ctx;
                return Value::function([l, ep, c](CallArgs& a) { return apply_operator(*ep, l.call(a), c); });
            }
            return apply_operator(e, l, ctx);
        }
        case Expr::IFX:
            if (eval(*e.a, ctx).truthy()) return eval(*e.b, ctx);
            return e.c ? eval(*e.c, ctx) : Value();
        case Expr::SLICE: throw std::runtime_error("SliceExpr not implemented");
    }
    return Value();
}

// ---- expression lexer / parser ----

struct Tok {
    enum K { ID, NUM, STR, OP, END } k;
    std::string s;
    Value v;
    size_t at = 0;  // offset in the expression source
};

std::vector<Tok> lex(const std::string& src) {
    std::vector<Tok> out;
    size_t p = 0;
    const size_t n = src.size();
    size_t marked = 0, start = 0;  // tokens whose offset is set; where the last one began
    auto mark = [&]() {
        if (marked < out.size()) {
            out.back().at = start;
            marked = out.size();
        }
    };
    while (p < n) {
        mark();
        start = p;
        const char c = src[p];
        if (std::isspace((unsigned char)c)) {
            ++p;
            continue;
        }
        if (std::isalpha((unsigned char)c) || c == '_') {
            size_t q = p;
            while (q < n && (std::isalnum((unsigned char)src[q]) || src[q] == '_')) ++q;
            out.push_back({Tok::ID, src.substr(p, q - p), Value()});
            p = q;
            continue;
        }
        if (std::isdigit((unsigned char)c)) {
            // the longest run of digits, one '.' and one e/E (no sign), which
            // must then read as a JSON number ("7." and "2.5e-3" do not)
            size_t q = p;
            bool dot = false, ex = false;
            while (q < n) {
                const char d = src[q];
                if (std::isdigit((unsigned char)d)) {
                    ++q;
                } else if (d == '.') {
                    if (dot) throw std::runtime_error("Multiple decimal points");
                    dot = true;
                    ++q;
                } else if (d == 'e' || d == 'E') {
                    if (ex) throw std::runtime_error("Multiple exponents");
                    ex = true;
                    ++q;
                } else {
                    break;
                }
            }
            const std::string t = src.substr(p, q - p);
            // JSON: (0 | [1-9][0-9]*) (. [0-9]+)? ([eE] [0-9]+)?
            size_t k = 0;
            bool good = t[0] != '0' || t.size() == 1 || !std::isdigit((unsigned char)t[1]);
            while (k < t.size() && std::isdigit((unsigned char)t[k])) ++k;
            if (good && k < t.size() && t[k] == '.') {
                const size_t b = ++k;
                while (k < t.size() && std::isdigit((unsigned char)t[k])) ++k;
                good = k > b;
            }
            if (good && k < t.size() && (t[k] == 'e' || t[k] == 'E')) {
                const size_t b = ++k;
                while (k < t.size() && std::isdigit((unsigned char)t[k])) ++k;
                good = k > b;
            }
            if (!good || k != t.size()) throw std::runtime_error("Failed to parse number: '" + t + "'");
            const bool fl = dot || ex;
            out.push_back({Tok::NUM, t,
                           fl ? Value(std::strtod(t.c_str(), nullptr)) : Value((int64_t)std::strtoll(t.c_str(), nullptr, 10))});
            p = q;
            continue;
        }
        if (c == '\'' || c == '"') {
            std::string s;
            size_t q = p + 1;
            while (q < n && src[q] != c) {
                if (src[q] == '\\' && q + 1 < n) {
                    const char x = src[++q];
                    switch (x) {
                        case 'n': s += '\n'; break;
                        case 't': s += '\t'; break;
                        case 'r': s += '\r'; break;
                        case 'b': s += '\b'; break;
                        case 'f': s += '\f'; break;
                        case 'v': s += '\v'; break;
                        default: s += x; break;
                    }
                    ++q;
                    continue;
                }
                s += src[q++];
            }
            if (q >= n) throw std::runtime_error("unterminated string literal");
            out.push_back({Tok::STR, s, Value(s)});
            p = q + 1;
            continue;
        }
        static const char* two[] = {"==", "!=", "<=", ">=", "**", "//"};
        bool done = false;
        for (const char* t : two)
            if (src.compare(p, 2, t) == 0) {
                out.push_back({Tok::OP, t, Value()});
                p += 2;
                done = true;
                break;
            }
        if (done) continue;
        if (std::strchr("<>+-*/%~|()[]{},:.=", c)) {
            out.push_back({Tok::OP, std::string(1, c), Value()});
            ++p;
            continue;
        }
        throw std::runtime_error(std::string("unexpected character '") + c + "' in expression");
    }
    mark();
    out.push_back({Tok::END, "", Value(), n});
    return out;
}

bool is_reserved(const std::string& s) {
    return s == "not" || s == "is" || s == "and" || s == "or" || s == "del";
}

struct ExprParser {
    std::vector<Tok> t;
    size_t p = 0;
    const Tok& peek(size_t o = 0) const { return t[std::min(p + o, t.size() - 1)]; }
    bool at_op(const char* s) const { return peek().k == Tok::OP && peek().s == s; }
    bool at_kw(const char* s) const { return peek().k == Tok::ID && peek().s == s; }
    bool eat_op(const char* s) {
        if (!at_op(s)) return false;
        ++p;
        return true;
    }
    bool eat_kw(const char* s) {
        if (!at_kw(s)) return false;
        ++p;
        return true;
    }
    void need_op(const char* s) {
        if (!eat_op(s)) throw std::runtime_error(std::string("expected '") + s + "' in expression");
    }
    bool at_end() const { return peek().k == Tok::END; }
    static ExprP mk(Expr::Kind k) { return std::make_shared<Expr>(k); }
    static ExprP bin(const std::string& op, ExprP l, ExprP r) {
        auto e = mk(Expr::BIN);
        e->name = op;
        e->a = std::move(l);
        e->b = std::move(r);
        return e;
    }

    ExprP expression(bool allow_if = true) {
        ExprP l = logical_or();
        if (!allow_if || !eat_kw("if")) return l;
        auto e = mk(Expr::IFX);
        e->b = l;
        e->a = logical_or();
        if (eat_kw("else")) e->c = expression();
        return e;
    }
    ExprP logical_or() {
        ExprP l = logical_and();
        while (eat_kw("or")) l = bin("or", l, logical_and());
        return l;
    }
    ExprP logical_and() {
        ExprP l = logical_not();
        while (eat_kw("and")) l = bin("and", l, logical_not());
        return l;
    }
    ExprP logical_not() {
        if (eat_kw("not")) {
            auto e = mk(Expr::UNARY);
            e->name = "not";
            e->a = logical_not();
            return e;
        }
        return compare();
    }
    ExprP compare() {
        ExprP l = concat();
        while (true) {
            std::string op;
            if (at_op("==") || at_op("!=") || at_op("<") || at_op("<=") || at_op(">") || at_op(">=")) {
                op = peek().s;
                ++p;
            } else if (at_kw("in")) {
                op = "in";
                ++p;
            } else if (at_kw("not") && peek(1).k == Tok::ID && peek(1).s == "in") {
                op = "not in";
                p += 2;
            } else if (eat_kw("is")) {
                auto e = mk(Expr::IS);
                e->negate = eat_kw("not");
                if (peek().k != Tok::ID || is_reserved(peek().s))
                    throw std::runtime_error("Expected identifier after 'is' keyword");
                e->name = peek().s;
                ++p;
                e->a = l;
                return e;  // (a test ends the comparison chain)
            } else {
                return l;
            }
            l = bin(op, l, concat());
        }
    }
    ExprP concat() {
        ExprP l = power();
        if (eat_op("~")) l = bin("~", l, logical_and());
        return l;
    }
    ExprP power() {
        ExprP l = additive();
        while (eat_op("**")) l = bin("**", l, additive());
        return l;
    }
    ExprP additive() {
        ExprP l = multiplicative();
        while (at_op("+") || at_op("-")) {
            const std::string op = peek().s;
            ++p;
            l = bin(op, l, multiplicative());
        }
        return l;
    }
    ExprP multiplicative() {
        ExprP l = unary();
        while (at_op("*") || at_op("**") || at_op("/") || at_op("//") || at_op("%")) {
            const std::string op = peek().s;
            ++p;
            l = bin(op, l, unary());
        }
        if (eat_op("|")) {
            ExprP r = multiplicative();
            if (r->kind == Expr::FILTER) {
                r->items.insert(r->items.begin(), l);
                return r;
            }
            auto f = mk(Expr::FILTER);
            f->items = {l, r};
            return f;
        }
        return l;
    }
    ExprP unary() {
        std::string op;
        if (at_op("+") || at_op("-")) {
            op = peek().s;
            ++p;
        }
        std::string exp;
        if (at_op("*") || at_op("**")) {
            exp = peek().s;
            ++p;
        }
        ExprP v = value();
        if (!exp.empty()) {
            auto e = mk(Expr::UNARY);
            e->name = exp;
            e->a = v;
            v = e;
        }
        if (!op.empty()) {
            auto e = mk(Expr::UNARY);
            e->name = op;
            e->a = v;
            v = e;
        }
        return v;
    }
    void call_args(Expr& e) {
        need_op("(");
        if (eat_op(")")) return;
        while (true) {
            if (peek().k == Tok::ID && !is_reserved(peek().s) && peek(1).k == Tok::OP && peek(1).s == "=") {
                const std::string k = peek().s;
                p += 2;
                e.kwargs.emplace_back(k, expression());
            } else {
                e.args.push_back(expression());
            }
            if (eat_op(",")) {
                if (eat_op(")")) return;
                continue;
            }
            need_op(")");
            return;
        }
    }
    ExprP primary() {
        const Tok& k = peek();
        if (k.k == Tok::OP && (k.s == "-" || k.s == "+")) {
            // a sign where a value starts belongs to a number literal (the
            // unary operator has taken the first one): "-3" right after it
            // reads as -3, anything else is not a number
            const Tok& nx = peek(1);
            if (k.s == "-" && nx.k == Tok::NUM && nx.at == k.at + 1) {
                p += 2;
                auto e = mk(Expr::LIT);
                e->lit = nx.v.kind() == Value::INT ? Value(-nx.v.i()) : Value(-nx.v.f());
                return e;
            }
            throw std::runtime_error("Failed to parse number: '" + k.s + (nx.k == Tok::NUM && nx.at == k.at + 1 ? nx.s : "") + "'");
        }
        if (k.k == Tok::NUM || k.k == Tok::STR) {
            ++p;
            auto e = mk(Expr::LIT);
            e->lit = k.v;
            return e;
        }
        if (k.k == Tok::ID) {
            const std::string& s = k.s;
            auto lit = [&](Value v) {
                ++p;
                auto e = mk(Expr::LIT);
                e->lit = std::move(v);
                return e;
            };
            if (s == "true" || s == "True") return lit(Value(true));
            if (s == "false" || s == "False") return lit(Value(false));
            if (s == "none" || s == "None" || s == "null") return lit(Value());
            if (is_reserved(s)) throw std::runtime_error("Expected value expression");
            ++p;
            auto e = mk(Expr::VAR);
            e->name = s;
            return e;
        }
        if (eat_op("(")) {
            ExprP first = expression();
            if (eat_op(")")) return first;
            auto arr = mk(Expr::ARRAY);
            arr->items.push_back(first);
            while (eat_op(",")) {
                if (at_op(")")) break;
                arr->items.push_back(expression());
            }
            need_op(")");
            return arr;
        }
        if (eat_op("[")) {
            auto arr = mk(Expr::ARRAY);
            if (eat_op("]")) return arr;
            while (true) {
                arr->items.push_back(expression());
                if (eat_op(",")) {
                    if (eat_op("]")) return arr;
                    continue;
                }
                need_op("]");
                return arr;
            }
        }
        if (eat_op("{")) {
            auto d = mk(Expr::DICT);
            if (eat_op("}")) return d;
            while (true) {
                d->items.push_back(expression());
                need_op(":");
                d->items.push_back(expression());
                if (eat_op(",")) {
                    if (eat_op("}")) return d;
                    continue;
                }
                need_op("}");
                return d;
            }
        }
        throw std::runtime_error("Expected value expression");
    }
    ExprP value() {
        ExprP v = primary();
        while (at_op("[") || at_op(".")) {
            if (eat_op("[")) {
                ExprP start, end, step, idx;
                bool c1 = false;
                if (!at_op(":")) start = expression();
                if (eat_op(":")) {
                    c1 = true;
                    if (!at_op(":") && !at_op("]")) end = expression();
                    if (eat_op(":") && !at_op("]")) step = expression();
                }
                if (c1) {
                    idx = mk(Expr::SLICE);
                    idx->a = start;
                    idx->b = end;
                    idx->c = step;
                } else {
                    idx = start;
                }
                if (!idx) throw std::runtime_error("Empty index in subscript");
                need_op("]");
                auto s = mk(Expr::SUB);
                s->a = v;
                s->b = idx;
                v = s;
            } else {
                ++p;  // '.'
                if (peek().k != Tok::ID || is_reserved(peek().s))
                    throw std::runtime_error("Expected identifier in subscript");
                const std::string name = peek().s;
                ++p;
                if (at_op("(")) {
                    auto m = mk(Expr::ATTR_CALL);
                    m->a = v;
                    m->name = name;
                    call_args(*m);
                    v = m;
                } else {
                    auto s = mk(Expr::SUB);
                    s->a = v;
                    auto key = mk(Expr::LIT);
                    key->lit = Value(name);
                    s->b = key;
                    v = s;
                }
            }
        }
        if (at_op("(")) {
            auto c = mk(Expr::CALL);
            c->a = v;
            call_args(*c);
            v = c;
        }
        return v;
    }
};

ExprP parse_expression(const std::string& src) {
    ExprParser ep{lex(src)};
    ExprP e = ep.expression();
    if (!ep.at_end()) throw std::runtime_error("unexpected '" + ep.peek().s + "' in expression: " + src);
    return e;
}

}  // namespace

// ---------------------------------------------------------------------------
// template nodes

struct TemplateNode {
    enum Kind { SEQ, TEXT, OUT, IF, FOR, SET, SET_BLOCK, BREAK, CONTINUE, MACRO, FILTER_BLOCK } kind;
    std::string text;                                  // TEXT
    ExprP expr;                                        // OUT, SET value, FOR iterable
    ExprP cond;                                        // FOR filter
    std::vector<std::string> names;                    // FOR / SET targets
    std::string ns;                                    // SET namespace
    std::vector<std::pair<ExprP, std::shared_ptr<TemplateNode>>> branches;  // IF (null cond: else)
    std::vector<std::shared_ptr<TemplateNode>> kids;   // SEQ
    std::shared_ptr<TemplateNode> body, else_body;     // FOR, SET_BLOCK, MACRO, FILTER_BLOCK
    std::vector<std::pair<std::string, ExprP>> params; // MACRO parameters (default or null)
    explicit TemplateNode(Kind k) : kind(k) {}
};

namespace {

using NodeP = std::shared_ptr<TemplateNode>;

void assign(const std::vector<std::string>& names, Context& ctx, const Value& v) {
    if (names.size() == 1) {
        ctx.set(names[0], v);
        return;
    }
    if (!v.is_array() || v.arr().size() != names.size())
        throw std::runtime_error("Mismatched number of variables and items in destructuring assignment");
    for (size_t i = 0; i < names.size(); ++i) ctx.set(names[i], v.arr()[i]);
}

void render_node(const TemplateNode& n, const Ctx& ctx, std::string& out) {
    switch (n.kind) {
        case TemplateNode::SEQ:
            for (const auto& k : n.kids) render_node(*k, ctx, out);
            return;
        case TemplateNode::TEXT: out += n.text; return;
        case TemplateNode::OUT: {
            Value v = eval(*n.expr, ctx);
            if (v.is_string())
                out += v.str();
            else if (v.kind() == Value::BOOL)
                out += v.b() ? "True" : "False";
            else if (!v.is_null())
                out += v.dump();
            return;
        }
        case TemplateNode::IF:
            for (const auto& br : n.branches)
                if (!br.first || eval(*br.first, ctx).truthy()) {
                    render_node(*br.second, ctx, out);
                    return;
                }
            return;
        case TemplateNode::FOR: {
            Value it = eval(*n.expr, ctx);
            std::vector<Value> items;
            if (!it.is_null()) {
                std::vector<Value> all;
                if (it.is_array())
                    all = it.arr();
                else if (it.is_object())
                    for (const auto& kv : it.obj()) all.emplace_back(kv.first);
                else if (it.is_string())
                    for (char c : it.str()) all.emplace_back(std::string(1, c));
                else
                    throw std::runtime_error("For loop iterable must be iterable: " + it.dump());
                for (const Value& x : all) {
                    assign(n.names, *ctx, x);  // (the targets stay set in the enclosing scope)
                    if (!n.cond || eval(*n.cond, ctx).truthy()) items.push_back(x);
                }
            }
            if (items.empty()) {
                if (n.else_body) render_node(*n.else_body, ctx, out);
                return;
            }
            Value loop = Value::object();
            const int64_t cnt = (int64_t)items.size();
            auto cycle_index = std::make_shared<size_t>(0);
            loop.set("length", Value(cnt));
            loop.set("cycle", Value::function([cycle_index](CallArgs& a) {
                         if (a.pos.empty() || !a.kw.empty())
                             throw std::runtime_error("cycle() expects at least 1 positional argument and no named arg");
                         Value v = a.pos[*cycle_index % a.pos.size()];
                         *cycle_index = (*cycle_index + 1) % a.pos.size();
                         return v;
                     }));
            auto lc = std::make_shared<Context>();
            lc->parent = ctx;
            lc->set("loop", loop);
            for (int64_t i = 0; i < cnt; ++i) {
                assign(n.names, *lc, items[(size_t)i]);
                loop.set("index", Value(i + 1));
                loop.set("index0", Value(i));
                loop.set("revindex", Value(cnt - i));
                loop.set("revindex0", Value(cnt - i - 1));
                loop.set("length", Value(cnt));
                loop.set("first", Value(i == 0));
                loop.set("last", Value(i == cnt - 1));
                loop.set("previtem", i > 0 ? items[(size_t)i - 1] : Value());
                loop.set("nextitem", i < cnt - 1 ? items[(size_t)i + 1] : Value());
                try {
                    render_node(*n.body, lc, out);
                } catch (const LoopControl& lcx) {
                    if (lcx.brk) break;
                }
            }
            return;
        }
        case TemplateNode::SET:
            if (!n.ns.empty()) {
                Value nsv = ctx->get(n.ns);
                if (!nsv.is_object()) throw std::runtime_error("Namespace '" + n.ns + "' is not an object");
                nsv.set(n.names[0], eval(*n.expr, ctx));
            } else {
                assign(n.names, *ctx, eval(*n.expr, ctx));
            }
            return;
        case TemplateNode::SET_BLOCK: {
            std::string s;
            render_node(*n.body, ctx, s);
            ctx->set(n.names[0], Value(s));
            return;
        }
        case TemplateNode::MACRO: {
            // a callable in the defining scope; a call binds its arguments in
            // that same scope (they stay set there), evaluates the defaults of
            // the parameters not passed in the caller's scope, and returns the
            // body's text
            const TemplateNode* node = &n;
            std::weak_ptr<Context> def = ctx;
            ctx->set(n.names[0], Value::function([node, def](CallArgs& a) {
                         Ctx c = def.lock();
                         if (!c) throw std::runtime_error("macro called outside its template");
                         const auto& ps = node->params;
                         std::vector<bool> given(ps.size(), false);
                         for (size_t i = 0; i < a.pos.size(); ++i) {
                             if (i >= ps.size())
                                 throw std::runtime_error("Too many positional arguments for macro " + node->names[0]);
                             c->set(ps[i].first, a.pos[i]);
                             given[i] = true;
                         }
                         for (auto& kv : a.kw) {
                             size_t k = 0;
                             while (k < ps.size() && ps[k].first != kv.first) ++k;
                             if (k == ps.size())
                                 throw std::runtime_error("Unknown parameter name for macro " + node->names[0] + ": " +
                                                          kv.first);
                             c->set(kv.first, kv.second);
                             given[k] = true;
                         }
                         const Ctx& caller = g_caller ? *g_caller : c;
                         for (size_t i = 0; i < ps.size(); ++i)
                             if (!given[i] && ps[i].second) c->set(ps[i].first, eval(*ps[i].second, caller));
                         std::string body;
                         render_node(*node->body, c, body);
                         return Value(body);
                     }));
            return;
        }
        case TemplateNode::FILTER_BLOCK: {
            Value f = eval(*n.expr, ctx);
            if (!f.is_callable()) throw std::runtime_error("Filter must be a callable: " + f.dump());
            std::string body;
            render_node(*n.body, ctx, body);
            CallArgs a;
            a.pos.emplace_back(body);
            CallerScope cs(ctx);
            out += f.call(a).to_str();
            return;
        }
        case TemplateNode::BREAK: throw LoopControl{true};
        case TemplateNode::CONTINUE: throw LoopControl{false};
    }
}

// ---- template lexer ----

struct TTok {
    enum K { TEXT, EXPR, STMT, COMMENT } k;
    std::string body;
    bool strip_before = false, strip_after = false;  // '-' after the opener / before the closer
    std::string word;                                // STMT keyword
    std::string rest;                                // STMT text after the keyword
};

size_t find_close(const std::string& s, size_t p, const char* close) {
    // the closer outside string literals
    char q = 0;
    for (; p + 1 < s.size(); ++p) {
        const char c = s[p];
        if (q) {
            if (c == '\\')
                ++p;
            else if (c == q)
                q = 0;
            continue;
        }
        if (c == '\'' || c == '"') {
            q = c;
            continue;
        }
        if (c == close[0] && s[p + 1] == close[1]) return p;
    }
    return std::string::npos;
}

std::vector<TTok> lex_template(const std::string& src) {
    std::vector<TTok> out;
    size_t p = 0;
    const size_t n = src.size();
    while (p < n) {
        size_t q = p;
        while (q + 1 < n && !(src[q] == '{' && (src[q + 1] == '{' || src[q + 1] == '%' || src[q + 1] == '#'))) ++q;
        if (q + 1 >= n) q = n;
        if (q > p) {
            TTok tt{TTok::TEXT, src.substr(p, q - p), false, false, "", ""};
            out.push_back(std::move(tt));
        }
        if (q >= n) break;
        const char kind = src[q + 1];
        size_t b = q + 2;
        TTok t{kind == '{' ? TTok::EXPR : kind == '%' ? TTok::STMT : TTok::COMMENT, "", false, false, "", ""};
        if (b < n && src[b] == '-') {
            t.strip_before = true;
            ++b;
        }
        const char* close = kind == '{' ? "}}" : kind == '%' ? "%}" : "#}";
        size_t e;
        if (kind == '#') {
            e = src.find("#}", b);
        } else {
            e = find_close(src, b, close);
        }
        if (e == std::string::npos) throw std::runtime_error("unterminated template tag");
        size_t be = e;
        if (be > b && src[be - 1] == '-') {
            t.strip_after = true;
            --be;
        }
        t.body = src.substr(b, be - b);
        if (t.k == TTok::STMT) {
            size_t i = 0;
            while (i < t.body.size() && std::isspace((unsigned char)t.body[i])) ++i;
            size_t j = i;
            while (j < t.body.size() && (std::isalnum((unsigned char)t.body[j]) || t.body[j] == '_')) ++j;
            t.word = t.body.substr(i, j - i);
            t.rest = t.body.substr(j);
        }
        out.push_back(std::move(t));
        p = e + 2;
    }
    return out;
}

bool is_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v'; }

// The whitespace rules of the reference's parser options (trim_blocks,
// lstrip_blocks, no trailing newline) and of the '-' markers, applied to
// every text token from its neighbours.
void apply_whitespace(std::vector<TTok>& toks) {
    for (size_t i = 0; i < toks.size(); ++i) {
        if (toks[i].k != TTok::TEXT) continue;
        std::string& t = toks[i].body;
        const bool has_prev = i > 0, has_next = i + 1 < toks.size();
        const bool strip_right = has_next && toks[i + 1].strip_before;
        const bool strip_left = has_prev && toks[i - 1].strip_after;
        if (strip_right) {
            size_t e = t.size();
            while (e > 0 && is_ws(t[e - 1])) --e;
            t.resize(e);
        } else if (has_next) {
            size_t e = t.size();
            while (e > 0 && (t[e - 1] == ' ' || t[e - 1] == '\t')) --e;
            if ((e == 0 && i == 0) || (e > 0 && t[e - 1] == '\n')) t.resize(e);
        }
        if (strip_left) {
            size_t b = 0;
            while (b < t.size() && is_ws(t[b])) ++b;
            t.erase(0, b);
        } else if (has_prev && toks[i - 1].k != TTok::EXPR) {
            if (!t.empty() && t[0] == '\n') t.erase(0, 1);
        }
        if (!has_next && !t.empty() && t.back() == '\n') {
            t.pop_back();
            if (!t.empty() && t.back() == '\r') t.pop_back();
        }
    }
}

std::vector<std::string> ident_list(ExprParser& ep) {
    std::vector<std::string> names;
    do {
        if (ep.peek().k != Tok::ID || is_reserved(ep.peek().s)) throw std::runtime_error("expected a variable name");
        names.push_back(ep.peek().s);
        ++ep.p;
    } while (ep.eat_op(","));
    return names;
}

struct TreeBuilder {
    std::vector<TTok>& toks;
    size_t i = 0;

    // parses nodes until a statement whose keyword is in `stops` (left unconsumed)
    NodeP sequence(std::initializer_list<const char*> stops) {
        auto seq = std::make_shared<TemplateNode>(TemplateNode::SEQ);
        while (i < toks.size()) {
            TTok& t = toks[i];
            if (t.k == TTok::STMT)
                for (const char* s : stops)
                    if (t.word == s) return seq;
            ++i;
            switch (t.k) {
                case TTok::TEXT:
                    if (!t.body.empty()) {
                        auto n = std::make_shared<TemplateNode>(TemplateNode::TEXT);
                        n->text = t.body;
                        seq->kids.push_back(n);
                    }
                    break;
                case TTok::COMMENT: break;
                case TTok::EXPR: {
                    auto n = std::make_shared<TemplateNode>(TemplateNode::OUT);
                    n->expr = parse_expression(t.body);
                    seq->kids.push_back(n);
                    break;
                }
                case TTok::STMT: seq->kids.push_back(statement(t)); break;
            }
        }
        if (stops.size()) throw std::runtime_error("unterminated block: expected {% " + std::string(*stops.begin()) + " %}");
        return seq;
    }
    void expect_end(const char* word) {
        if (i >= toks.size() || toks[i].k != TTok::STMT || toks[i].word != word)
            throw std::runtime_error(std::string("expected {% ") + word + " %}");
        ++i;
    }
    NodeP statement(TTok& t) {
        const std::string& w = t.word;
        if (w == "if") {
            auto n = std::make_shared<TemplateNode>(TemplateNode::IF);
            ExprP c = parse_expression(t.rest);
            while (true) {
                NodeP body = sequence({"elif", "else", "endif"});
                n->branches.emplace_back(c, body);
                if (i >= toks.size()) throw std::runtime_error("unterminated if");
                TTok& nt = toks[i++];
                if (nt.word == "elif") {
                    c = parse_expression(nt.rest);
                } else if (nt.word == "else") {
                    n->branches.emplace_back(nullptr, sequence({"endif"}));
                    expect_end("endif");
                    return n;
                } else {
                    return n;
                }
            }
        }
        if (w == "for") {
            auto n = std::make_shared<TemplateNode>(TemplateNode::FOR);
            ExprParser ep{lex(t.rest)};
            n->names = ident_list(ep);
            if (!ep.eat_kw("in")) throw std::runtime_error("expected 'in' in for statement");
            n->expr = ep.expression(false);
            if (ep.eat_kw("if")) n->cond = ep.expression();
            if (ep.at_kw("recursive")) throw std::domain_error("recursive loops are not supported");
            if (!ep.at_end()) throw std::runtime_error("unexpected tokens in for statement");
            n->body = sequence({"else", "endfor"});
            if (i < toks.size() && toks[i].word == "else") {
                ++i;
                n->else_body = sequence({"endfor"});
            }
            expect_end("endfor");
            return n;
        }
        if (w == "set") {
            ExprParser ep{lex(t.rest)};
            if (ep.peek().k == Tok::ID && ep.peek(1).k == Tok::OP && ep.peek(1).s == "." && ep.peek(2).k == Tok::ID) {
                auto n = std::make_shared<TemplateNode>(TemplateNode::SET);
                n->ns = ep.peek().s;
                n->names = {ep.peek(2).s};
                ep.p += 3;
                ep.need_op("=");
                n->expr = ep.expression();
                if (!ep.at_end()) throw std::runtime_error("unexpected tokens in set statement");
                return n;
            }
            std::vector<std::string> names = ident_list(ep);
            if (ep.at_end()) {
                if (names.size() != 1) throw std::runtime_error("Structural assignment not supported in set with template value");
                auto n = std::make_shared<TemplateNode>(TemplateNode::SET_BLOCK);
                n->names = names;
                n->body = sequence({"endset"});
                expect_end("endset");
                return n;
            }
            auto n = std::make_shared<TemplateNode>(TemplateNode::SET);
            n->names = names;
            ep.need_op("=");
            n->expr = ep.expression();
            if (!ep.at_end()) throw std::runtime_error("unexpected tokens in set statement");
            return n;
        }
        if (w == "break") return std::make_shared<TemplateNode>(TemplateNode::BREAK);
        if (w == "continue") return std::make_shared<TemplateNode>(TemplateNode::CONTINUE);
        if (w == "generation") {  // marks generated text for training masks: rendered as its body
            NodeP body = sequence({"endgeneration"});
            expect_end("endgeneration");
            return body;
        }
        if (w == "macro") {
            auto n = std::make_shared<TemplateNode>(TemplateNode::MACRO);
            ExprParser ep{lex(t.rest)};
            if (ep.peek().k != Tok::ID || is_reserved(ep.peek().s)) throw std::runtime_error("Expected macro name in macro block");
            n->names = {ep.peek().s};
            ++ep.p;
            ep.need_op("(");
            if (!ep.eat_op(")")) {
                while (true) {
                    if (ep.peek().k != Tok::ID || is_reserved(ep.peek().s))
                        throw std::domain_error("macro parameters other than names are not supported");
                    std::string pname = ep.peek().s;
                    ++ep.p;
                    ExprP dflt;
                    if (ep.eat_op("=")) dflt = ep.expression();
                    n->params.emplace_back(pname, dflt);
                    if (ep.eat_op(",")) {
                        if (ep.eat_op(")")) break;
                        continue;
                    }
                    ep.need_op(")");
                    break;
                }
            }
            if (!ep.at_end()) throw std::runtime_error("unexpected tokens in macro statement");
            n->body = sequence({"endmacro"});
            expect_end("endmacro");
            return n;
        }
        if (w == "filter") {
            auto n = std::make_shared<TemplateNode>(TemplateNode::FILTER_BLOCK);
            n->expr = parse_expression(t.rest);
            n->body = sequence({"endfilter"});
            expect_end("endfilter");
            return n;
        }
        throw std::domain_error("unsupported template statement: {% " + w + " %}");
    }
};

// ---- builtins ----

const Value& need(CallArgs& a, size_t i, const char* pname, const char* fname) {
    // positional i, or the keyword of that name
    if (i < a.pos.size()) return a.pos[i];
    for (auto& kv : a.kw)
        if (kv.first == pname) return kv.second;
    throw std::runtime_error(std::string(fname) + ": missing argument '" + pname + "'");
}
// Builtins with named parameters take them by position or by name; extra
// positional arguments and unknown names are errors.
void params(const CallArgs& a, const char* fname, std::initializer_list<const char*> names) {
    if (a.pos.size() > names.size()) throw std::runtime_error(std::string("Too many positional params for ") + fname);
    for (const auto& kv : a.kw) {
        bool known = false;
        for (const char* n : names) known = known || kv.first == n;
        if (!known) throw std::runtime_error("Unknown argument " + kv.first + " for function " + fname);
    }
}
const Value* opt(CallArgs& a, size_t i, const char* pname) {
    if (i < a.pos.size()) return &a.pos[i];
    for (auto& kv : a.kw)
        if (kv.first == pname) return &kv.second;
    return nullptr;
}

std::string html_escape(const std::string& s) {
    std::string r;
    for (char c : s) {
        switch (c) {
            case '&': r += "&amp;"; break;
            case '<': r += "&lt;"; break;
            case '>': r += "&gt;"; break;
            case '"': r += "&#34;"; break;
            case '\'': r += "&apos;"; break;
            default: r += c;
        }
    }
    return r;
}

Ctx builtins() {
    auto g = std::make_shared<Context>();
    auto def = [&](const char* name, Value::Fn f) { g->set(name, Value::function(std::move(f))); };
    def("raise_exception", [](CallArgs& a) -> Value {
        params(a, "raise_exception", {"message"});
        throw std::runtime_error(need(a, 0, "message", "raise_exception").str());
    });
    def("tojson", [](CallArgs& a) {
        params(a, "tojson", {"value", "indent"});
        const Value* ind = opt(a, 1, "indent");
        return Value(need(a, 0, "value", "tojson").dump(ind ? (int)ind->i() : -1, true));
    });
    def("items", [](CallArgs& a) {
        params(a, "items", {"object"});
        const Value& o = need(a, 0, "object", "items");
        if (!o.is_object()) throw std::runtime_error("Can only get item pairs from a mapping");
        Value r = Value::array();
        for (const auto& kv : o.obj()) r.push(Value::array({Value(kv.first), kv.second}));
        return r;
    });
    def("last", [](CallArgs& a) {
        params(a, "last", {"items"});
        const Value& v = need(a, 0, "items", "last");
        if (!v.is_array()) throw std::runtime_error("object is not a list");
        return v.arr().empty() ? Value() : v.arr().back();
    });
    def("trim", [](CallArgs& a) {
        params(a, "trim", {"text"});
        const Value& v = need(a, 0, "text", "trim");
        return v.is_null() ? v : Value(strip_chars(v.str(), "", true, true));
    });
    for (const char* nm : {"lower", "upper"}) {
        const bool up = nm[0] == 'u';
        def(nm, [up](CallArgs& a) {
            params(a, up ? "upper" : "lower", {"text"});
            const Value& v = need(a, 0, "text", up ? "upper" : "lower");
            if (v.is_null()) return v;
            std::string s = v.str();
            for (char& c : s) c = (char)(up ? std::toupper((unsigned char)c) : std::tolower((unsigned char)c));
            return Value(s);
        });
    }
    def("default", [](CallArgs& a) {
        expect_args(a, "default", 2, 3, 0, 1);
        auto as_bool = [](const Value& v) {
            if (v.kind() != Value::BOOL) throw std::runtime_error("type must be boolean: " + v.dump());
            return v.b();
        };
        bool boolean = false;
        if (a.pos.size() == 3)
            boolean = as_bool(a.pos[2]);
        else if (const Value* b = opt(a, 99, "boolean"))
            boolean = b->is_null() ? false : as_bool(*b);
        const Value &v = a.pos[0], &d = a.pos[1];
        return boolean ? (v.truthy() ? v : d) : (v.is_null() ? d : v);
    });
    auto esc = [](CallArgs& a) {
        params(a, "escape", {"text"});
        return Value(html_escape(need(a, 0, "text", "escape").str()));
    };
    def("e", esc);
    def("escape", esc);
    def("joiner", [](CallArgs& a) {
        params(a, "joiner", {"sep"});
        const Value* s = opt(a, 0, "sep");
        const std::string sep = s ? s->str() : "";
        auto first = std::make_shared<bool>(true);
        return Value::function([sep, first](CallArgs&) {
            if (*first) {
                *first = false;
                return Value("");
            }
            return Value(sep);
        });
    });
    def("count", [](CallArgs& a) {
        params(a, "count", {"items"});
        return Value((int64_t)need(a, 0, "items", "count").size());
    });
    def("dictsort", [](CallArgs& a) {
        params(a, "dictsort", {"value"});
        if (a.pos.size() + a.kw.size() != 1) throw std::runtime_error("dictsort expects exactly 1 argument");
        const Value& v = need(a, 0, "value", "dictsort");
        std::vector<std::string> keys;
        for (const auto& kv : v.obj()) keys.push_back(kv.first);
        std::sort(keys.begin(), keys.end());
        Value r = Value::array();
        for (const auto& k : keys) r.push(Value::array({Value(k), *v.find(k)}));
        return r;
    });
    def("join", [](CallArgs& a) {
        params(a, "join", {"items", "d"});
        const Value* d = opt(a, 1, "d");
        const std::string sep = d ? d->str() : "";
        const Value* items = opt(a, 0, "items");
        if (!items) throw std::domain_error("join without items is not supported");
        if (!items->is_array()) throw std::runtime_error("object is not iterable: " + items->dump());
        std::string r;
        for (size_t i = 0; i < items->arr().size(); ++i) {
            if (i) r += sep;
            r += items->arr()[i].to_str();
        }
        return Value(r);
    });
    def("namespace", [](CallArgs& a) {
        if (!a.pos.empty()) throw std::runtime_error("namespace: positional arguments are not allowed");
        Value ns = Value::object();
        for (auto& kv : a.kw) ns.set(kv.first, kv.second);
        return ns;
    });
    auto equalto = [](CallArgs& a) {
        params(a, "equalto", {"expected", "actual"});
        return Value(need(a, 1, "actual", "equalto").equals(need(a, 0, "expected", "equalto")));
    };
    def("equalto", equalto);
    def("==", equalto);
    def("length", [](CallArgs& a) {
        params(a, "length", {"items"});
        return Value((int64_t)need(a, 0, "items", "length").size());
    });
    def("safe", [](CallArgs& a) {
        params(a, "safe", {"value"});
        return Value(need(a, 0, "value", "safe").to_str());
    });
    def("string", [](CallArgs& a) {
        params(a, "string", {"value"});
        return Value(need(a, 0, "value", "string").to_str());
    });
    def("int", [](CallArgs& a) {
        params(a, "int", {"value"});
        const Value& v = need(a, 0, "value", "int");
        if (v.is_null()) return Value((int64_t)0);
        if (v.is_string()) {
            char* end = nullptr;
            const long long x = std::strtoll(v.str().c_str(), &end, 10);
            return Value((int64_t)(end == v.str().c_str() ? 0 : x));
        }
        if (v.kind() == Value::BOOL) return Value((int64_t)(v.b() ? 1 : 0));
        if (v.is_number()) return Value(v.i());
        return Value((int64_t)0);
    });
    def("list", [](CallArgs& a) {
        params(a, "list", {"items"});
        const Value& v = need(a, 0, "items", "list");
        if (!v.is_array()) throw std::runtime_error("object is not iterable");
        return v;
    });
    def("in", [](CallArgs& a) {
        params(a, "in", {"item", "items"});
        return Value(contains_value(need(a, 0, "item", "in"), need(a, 1, "items", "in")));
    });
    def("unique", [](CallArgs& a) {
        params(a, "unique", {"items"});
        const Value& v = need(a, 0, "items", "unique");
        if (!v.is_array()) throw std::runtime_error("object is not iterable");
        Value r = Value::array();
        for (const Value& x : v.arr()) {
            // a hash set of scalars: containers cannot be hashed, and values
            // of different JSON types (1 and 1.0) never collide
            if (x.is_array() || x.is_object() || x.is_callable())
                throw std::runtime_error("Unsupported type for hashing: " + x.dump());
            bool seen = false;
            for (const Value& y : r.arr())
                if (y.kind() == x.kind() && (x.is_null() || y.equals(x))) seen = true;
            if (!seen) r.push(x);
        }
        return r;
    });
    def("indent", [](CallArgs& a) {
        params(a, "indent", {"text", "indent", "first"});
        const std::string text = need(a, 0, "text", "indent").str();
        const Value* w = opt(a, 1, "indent");
        const Value* f = opt(a, 2, "first");
        if (f && f->kind() != Value::BOOL) throw std::runtime_error("indent: first must be a boolean");
        const bool first = f && f->b();
        const std::string pad(w ? (size_t)std::max<int64_t>(0, w->i()) : 0, ' ');
        // lines split at '\n' (a final newline ends the last line), each indented
        // but the first unless `first`; a final newline is kept
        std::string out;
        size_t b = 0;
        bool is_first = true;
        while (b < text.size()) {
            size_t e = text.find('\n', b);
            if (e == std::string::npos) e = text.size();
            if (!is_first) out += '\n';
            if (!is_first || first) out += pad;
            out.append(text, b, e - b);
            is_first = false;
            b = e + 1;
        }
        if (!text.empty() && text.back() == '\n') out += '\n';
        return Value(out);
    });
    def("range", [](CallArgs& a) {
        int64_t v[3] = {0, 0, 1};
        bool set[3] = {false, false, false};
        if (a.pos.size() == 1) {
            v[1] = a.pos[0].i();
            set[1] = true;
        } else {
            if (a.pos.size() > 3) throw std::runtime_error("range: too many arguments");
            for (size_t i = 0; i < a.pos.size(); ++i) {
                v[i] = a.pos[i].i();
                set[i] = true;
            }
        }
        for (auto& kv : a.kw) {
            const int i = kv.first == "start" ? 0 : kv.first == "end" ? 1 : kv.first == "step" ? 2 : -1;
            if (i < 0) throw std::runtime_error("Unknown argument " + kv.first + " for function range");
            if (set[i]) throw std::runtime_error("Duplicate argument " + kv.first + " for function range");
            v[i] = kv.second.i();
            set[i] = true;
        }
        if (!set[1]) throw std::runtime_error("range: missing end");
        if (v[2] == 0) throw std::runtime_error("range: step cannot be zero");
        Value r = Value::array();
        for (int64_t x = v[0]; v[2] > 0 ? x < v[1] : x > v[1]; x += v[2]) r.push(Value(x));
        return r;
    });
    return g;
}

// select/reject, selectattr/rejectattr and map look filters up by name, so
// they are defined over the builtins context
void add_lookup_filters(const Ctx& g) {
    std::weak_ptr<Context> wg = g;
    auto lookup = [wg](const Value& name) {
        auto c = wg.lock();
        Value f = c && name.is_string() ? c->get(name.str()) : Value();
        if (f.is_null()) throw std::runtime_error("Undefined filter: " + name.dump());
        return f;
    };
    for (const bool sel : {true, false}) {
        g->set(sel ? "select" : "reject", Value::function([lookup, sel](CallArgs& a) {
                   if (a.pos.size() < 2 || !a.kw.empty()) throw std::runtime_error("select/reject: bad arguments");
                   const Value& items = a.pos[0];
                   if (items.is_null()) return Value::array();
                   if (!items.is_array()) throw std::runtime_error("object is not iterable: " + items.dump());
                   Value f = lookup(a.pos[1]);
                   Value r = Value::array();
                   for (const Value& x : items.arr()) {
                       CallArgs fa;
                       fa.pos.push_back(x);
                       for (size_t i = 2; i < a.pos.size(); ++i) fa.pos.push_back(a.pos[i]);
                       if (f.call(fa).truthy() == sel) r.push(x);
                   }
                   return r;
               }));
        g->set(sel ? "selectattr" : "rejectattr", Value::function([lookup, sel](CallArgs& a) {
                   if (a.pos.size() < 2) throw std::runtime_error("selectattr/rejectattr: bad arguments");
                   const Value& items = a.pos[0];
                   if (items.is_null()) return Value::array();
                   if (!items.is_array()) throw std::runtime_error("object is not iterable: " + items.dump());
                   const std::string attr = a.pos[1].str();
                   const bool has_test = a.pos.size() >= 3;
                   Value f = has_test ? lookup(a.pos[2]) : Value();
                   Value r = Value::array();
                   for (const Value& x : items.arr()) {
                       Value v = get_item(x, Value(attr));
                       if (has_test) {
                           CallArgs fa;
                           fa.pos.push_back(v);
                           for (size_t i = 3; i < a.pos.size(); ++i) fa.pos.push_back(a.pos[i]);
                           fa.kw = a.kw;
                           if (f.call(fa).truthy() == sel) r.push(x);
                       } else {
                           r.push(v);
                       }
                   }
                   return r;
               }));
    }
    g->set("map", Value::function([lookup](CallArgs& a) {
               Value r = Value::array();
               const Value* attr = nullptr;
               const Value* dflt = nullptr;
               for (auto& kv : a.kw) {
                   if (kv.first == "attribute") attr = &kv.second;
                   if (kv.first == "default") dflt = &kv.second;
               }
               if (a.pos.size() == 1 && ((attr && a.kw.size() == 1) || (dflt && a.kw.size() == 2))) {
                   for (size_t i = 0; i < a.pos[0].size(); ++i) {
                       const Value& x = a.pos[0].arr()[i];
                       Value v = attr ? get_item(x, *attr) : Value();
                       r.push(v.is_null() ? (dflt ? *dflt : Value()) : v);
                   }
               } else if (a.kw.empty() && a.pos.size() >= 2) {
                   Value f = lookup(a.pos[1]);
                   for (size_t i = 0; i < a.pos[0].size(); ++i) {
                       CallArgs fa;
                       fa.pos.push_back(a.pos[0].arr()[i]);
                       for (size_t j = 2; j < a.pos.size(); ++j) fa.pos.push_back(a.pos[j]);
                       r.push(f.call(fa));
                   }
               } else {
                   throw std::runtime_error("Invalid or unsupported arguments for map");
               }
               return r;
           }));
}

}  // namespace

// ---------------------------------------------------------------------------
// chat template

ChatTemplate::ChatTemplate(const std::string& source, std::string bos_token, std::string eos_token)
    : bos_(std::move(bos_token)), eos_(std::move(eos_token)) {
    try {
        std::vector<TTok> toks = lex_template(source);
        apply_whitespace(toks);
        TreeBuilder tb{toks};
        root_ = tb.sequence({});
    } catch (const std::domain_error& e) {  // a construct that is not built
        parse_error_ = e.what();
        parse_unsupported_ = true;
        return;
    } catch (const std::exception& e) {
        parse_error_ = e.what();
        return;
    }
    // capability probes: renders of stand-in conversations, as the reference's
    // chat_template runs them (an error in a probe counts as an empty render)
    auto has = [](const std::string& s, const char* needle) { return s.find(needle) != std::string::npos; };
    auto msg = [](const char* role, Value content) {
        Value m = Value::object();
        m.set("role", Value(role));
        m.set("content", std::move(content));
        return m;
    };
    auto typed = [](const char* text) {
        Value part = Value::object();
        part.set("type", Value("text"));
        part.set("text", Value(text));
        return Value::array({part});
    };
    const char* user_needle = "<User Needle>";
    const char* sys_needle = "<System Needle>";
    const Value str_user = msg("user", Value(user_needle)), typed_user = msg("user", typed(user_needle));
    caps_.requires_typed_content = !has(try_raw_render(Value::array({str_user}), nullptr), user_needle) &&
                                   has(try_raw_render(Value::array({typed_user}), nullptr), user_needle);
    const Value user = caps_.requires_typed_content ? typed_user : str_user;
    const Value sys = msg("system", caps_.requires_typed_content ? typed(sys_needle) : Value(sys_needle));
    caps_.supports_system_role = has(try_raw_render(Value::array({sys, user}), nullptr), sys_needle);

    Value tool = parse_json(
        R"({"name": "some_tool", "type": "function", "function": {"name": "some_tool", "description": "Some tool.",)"
        R"( "parameters": {"type": "object", "properties": {"arg": {"type": "string", "description": "Some argument."}},)"
        R"( "required": ["arg"]}}})");
    const Value tools = Value::array({tool});
    caps_.supports_tools = has(try_raw_render(Value::array({user}), &tools), "some_tool");

    auto with_content = [&](Value c) {
        const Value a = msg("assistant", c);
        return try_raw_render(Value::array({user, a, user, a}), nullptr);
    };
    caps_.requires_non_null_content = has(with_content(Value("")), user_needle) && !has(with_content(Value()), user_needle);
    auto calls_msg = [&](Value calls) {
        Value m = msg("assistant", caps_.requires_non_null_content ? Value("") : Value());
        m.set("tool_calls", std::move(calls));
        return m;
    };
    auto call = [](const char* name, Value args) {
        Value f = Value::object();
        f.set("arguments", std::move(args));
        f.set("name", Value(name));
        Value c = Value::object();
        c.set("id", Value("call_1___"));
        c.set("type", Value("function"));
        c.set("function", f);
        return c;
    };
    const Value args_obj = parse_json(R"J({"argument_needle": "print('Hello, World!')"})J");
    const std::string args_text = R"J({"argument_needle":"print('Hello, World!')"})J";  // compact JSON text
    auto renders_args = [&](const std::string& s) {
        return has(s, "<parameter=argument_needle>") || has(s, "\"argument_needle\":") || has(s, "'argument_needle':");
    };
    const bool str_args =
        renders_args(try_raw_render(Value::array({user, calls_msg(Value::array({call("ipython", Value(args_text))}))}), nullptr));
    const bool obj_args =
        renders_args(try_raw_render(Value::array({user, calls_msg(Value::array({call("ipython", args_obj)}))}), nullptr));
    caps_.supports_tool_calls = str_args || obj_args;
    caps_.requires_object_arguments = !str_args && obj_args;
    if (caps_.supports_tool_calls) {
        const Value args = caps_.requires_object_arguments ? args_obj : Value(args_text);
        Value r2 = Value::object();
        r2.set("role", Value("tool"));
        r2.set("name", Value("test_tool1"));
        r2.set("content", Value("Some response!"));
        r2.set("tool_call_id", Value("call_911_"));
        caps_.supports_tool_responses = has(
            try_raw_render(Value::array({user, calls_msg(Value::array({call("test_tool1", args)})), r2}), nullptr),
            "Some response!");
    }
    // A template that cannot show tools gets them described in a system
    // message, with an example call inferred from what the template renders
    // for one: the text a tool-call turn adds after a plain prompt.
    if (!caps_.supports_tools) {
        try {
            const Value user_msg = msg("user", Value("Hey"));
            Value targs = Value::object();
            targs.set("arg1", Value("some_value"));
            Value f = Value::object();
            f.set("name", Value("tool_name"));
            f.set("arguments", caps_.requires_object_arguments ? targs : Value(targs.dump(-1, true)));
            Value tc = Value::object();
            tc.set("id", Value("call_1___"));
            tc.set("type", Value("function"));
            tc.set("function", f);
            Value tcm = msg("assistant", caps_.requires_non_null_content ? Value("") : Value());
            tcm.set("tool_calls", Value::array({tc}));
            const std::string prefix = render(Value::array({user_msg}), Value(), true);
            std::string full = render(Value::array({user_msg, tcm}), Value(), false);
            const size_t eos_last = full.rfind(eos_);
            if (eos_last == prefix.size() - eos_.size() ||
                (!full.empty() && full.back() == '\n' && eos_last == full.size() - eos_.size() - 1))
                full = full.substr(0, eos_last);
            size_t common = 0;
            for (size_t i = 0; i < prefix.size() && i < full.size(); ++i) {
                if (prefix[i] != full[i]) break;
                if (prefix[i] == '<') continue;  // (a divergence at a tag keeps the tag's '<')
                common = i + 1;
            }
            const std::string example = full.substr(common);
            if (example.find("tool_name") != std::string::npos || example.find("some_value") != std::string::npos)
                tool_call_example_ = example;
        } catch (const std::exception&) {
            // no example: the tools are described without one
        }
    }
}

ChatTemplate::~ChatTemplate() = default;

void ChatTemplate::check_parsed() const {
    if (root_) return;
    if (parse_unsupported_) throw std::domain_error("chat template uses " + parse_error_);
    throw std::runtime_error("chat template does not parse: " + parse_error_);
}

std::string ChatTemplate::raw_render(const Value& messages, const Value* tools, bool add_generation_prompt) const {
    check_parsed();
    Ctx g = builtins();
    add_lookup_filters(g);
    auto ctx = std::make_shared<Context>();
    ctx->parent = g;
    ctx->set("messages", messages);
    ctx->set("add_generation_prompt", Value(add_generation_prompt));
    ctx->set("bos_token", Value(bos_));
    ctx->set("eos_token", Value(eos_));
    const auto now = std::chrono::system_clock::now();
    ctx->set("strftime_now", Value::function([now](CallArgs& a) {
                 expect_args(a, "strftime_now", 1, 1, 0, 0);
                 const std::time_t t = std::chrono::system_clock::to_time_t(now);
                 std::tm tm{};
                 localtime_r(&t, &tm);
                 char buf[512];
                 const size_t n = std::strftime(buf, sizeof(buf), a.pos[0].str().c_str(), &tm);
                 return Value(std::string(buf, n));
             }));
    if (tools) ctx->set("tools", *tools);
    std::string out;
    render_node(*root_, ctx, out);
    return out;
}

std::string ChatTemplate::try_raw_render(const Value& messages, const Value* tools) const {
    try {
        return raw_render(messages, tools, false);
    } catch (const std::exception&) {
        return "";
    }
}

std::string ChatTemplate::render(const Value& messages, const Value& tools, bool add_generation_prompt) const {
    check_parsed();
    const Value* tools_var = tools.is_null() ? nullptr : &tools;
    const bool has_tools = tools.is_array() && !tools.arr().empty();
    bool has_tool_calls = false, has_tool_responses = false, has_string_content = false;
    for (const Value& m : messages.arr()) {
        const Value* tc = m.find("tool_calls");
        if (tc && !tc->is_null()) has_tool_calls = true;
        const Value* role = m.find("role");
        if (role && role->is_string() && role->str() == "tool") has_tool_responses = true;
        const Value* c = m.find("content");
        if (c && c->is_string()) has_string_content = true;
    }
    const bool poly_system = !caps_.supports_system_role;
    const bool poly_tools = has_tools && !caps_.supports_tools;
    const bool poly_calls = has_tool_calls && !caps_.supports_tool_calls;
    const bool poly_responses = has_tool_responses && !caps_.supports_tool_responses;
    const bool poly_obj_args = has_tool_calls && caps_.requires_object_arguments;
    const bool poly_typed = has_string_content && caps_.requires_typed_content;
    if (!(poly_system || poly_tools || poly_calls || poly_responses || poly_obj_args || poly_typed))
        return raw_render(messages, tools_var, add_generation_prompt);

    auto copy_obj = [](const Value& o) {
        Value c = Value::object();
        for (const auto& kv : o.obj()) c.set(kv.first, kv.second);
        return c;
    };
    auto role_of = [](const Value& m) -> std::string {
        const Value* r = m.find("role");
        if (!r) throw std::out_of_range("key 'role' not found");
        if (!r->is_string()) throw std::runtime_error("role must be a string");
        return r->str();
    };
    Value actual = Value::array();
    auto add = [&](const Value& m) {
        const Value* c = m.find("content");
        if (poly_typed && c && c->is_string()) {
            Value part = Value::object();
            part.set("type", Value("text"));
            part.set("text", *c);
            Value nm = Value::object();
            const Value* r = m.find("role");
            if (!r) throw std::out_of_range("key 'role' not found");
            nm.set("role", *r);
            nm.set("content", Value::array({part}));
            actual.push(nm);
        } else {
            actual.push(m);
        }
    };
    std::string pending;
    auto flush = [&]() {
        if (pending.empty()) return;
        Value m = Value::object();
        m.set("role", Value("user"));
        m.set("content", Value(pending));
        add(m);
        pending.clear();
    };

    // the tools, described in the (first) system message
    Value msgs = messages;
    if (poly_tools) {
        std::string prompt =
            "You can call any of the following tools to satisfy the user's requests: " + tools.dump(2, true);
        if (!tool_call_example_.empty()) prompt += "\n\nExample tool call syntax:\n\n" + tool_call_example_ + "\n\n";
        Value adj = Value::array();
        for (const Value& m : messages.arr()) adj.push(m);
        Value sys = Value::object();
        sys.set("role", Value("system"));
        const Value* r0 = adj.arr().empty() ? nullptr : adj.arr()[0].find("role");
        if (!adj.arr().empty() && !r0) throw std::out_of_range("key 'role' not found");
        if (r0 && r0->is_string() && r0->str() == "system") {
            const Value* c = adj.arr()[0].find("content");
            if (!c || !c->is_string()) throw std::runtime_error("system content must be a string");
            sys.set("content", Value(c->str() + "\n\n" + prompt));
            adj.arr()[0] = sys;
        } else {
            sys.set("content", Value(prompt));
            adj.arr().insert(adj.arr().begin(), sys);
        }
        msgs = adj;
    }

    for (const Value& m0 : msgs.arr()) {
        if (!m0.is_object() || !m0.find("role") || (!m0.find("content") && !m0.find("tool_calls")))
            throw std::runtime_error("message must have 'role' and one of 'content' or 'tool_calls' fields: " +
                                     m0.json_text());
        // a deep enough copy: the message and its tool calls are rewritten
        Value m = copy_obj(m0);
        const std::string role = role_of(m);
        if (const Value* tcs0 = m.find("tool_calls")) {
            if (poly_obj_args || poly_calls) {
                if (!tcs0->is_array()) throw std::runtime_error("tool_calls must be an array");
                Value tcs = Value::array();
                for (const Value& tc0 : tcs0->arr()) {
                    Value tc = tc0.is_object() ? copy_obj(tc0) : tc0;
                    if (tc.is_object()) {
                        if (!tc.find("type")) tc.set("type", Value());  // (a lookup that adds the key)
                        const Value* ty = tc.find("type");
                        if (ty->is_string() && ty->str() == "function") {
                            const Value* f0 = tc.find("function");
                            if (!f0) throw std::out_of_range("key 'function' not found");
                            Value f = f0->is_object() ? copy_obj(*f0) : *f0;
                            const Value* a = f.find("arguments");
                            if (!a) throw std::out_of_range("key 'arguments' not found");
                            if (a->is_string()) {
                                try {
                                    f.set("arguments", parse_json(a->str()));
                                } catch (const std::invalid_argument&) {
                                    // not JSON: the text stays
                                }
                            }
                            tc.set("function", f);
                        }
                    }
                    tcs.push(tc);
                }
                m.set("tool_calls", tcs);
            }
            if (poly_calls) {
                Value calls = Value::array();
                for (const Value& tc : m.find("tool_calls")->arr()) {
                    const Value* ty = tc.find("type");
                    if (!ty) throw std::out_of_range("key 'type' not found");
                    if (!(ty->is_string() && ty->str() == "function")) continue;
                    const Value* f = tc.find("function");
                    if (!f || !f->find("name") || !f->find("arguments"))
                        throw std::out_of_range("tool call function needs name and arguments");
                    Value c = Value::object();
                    c.set("name", *f->find("name"));
                    c.set("arguments", *f->find("arguments"));
                    if (const Value* id = tc.find("id")) c.set("id", *id);
                    calls.push(c);
                }
                Value o = Value::object();
                o.set("tool_calls", calls);
                if (const Value* c = m.find("content")) {
                    // (JSON emptiness: null, [] and {} are empty; "" is not)
                    const bool empty = c->is_null() || (c->is_array() && c->arr().empty()) ||
                                       (c->is_object() && c->obj().empty());
                    if (!empty) o.set("content", *c);
                }
                m.set("content", Value(o.json_text(2)));
                m.erase("tool_calls");
            }
        }
        if (poly_responses && role == "tool") {
            m.set("role", Value("user"));
            Value r = Value::object();
            if (const Value* n = m.find("name")) r.set("tool", *n);
            const Value* c = m.find("content");
            if (!c) throw std::out_of_range("key 'content' not found");
            r.set("content", *c);
            if (const Value* id = m.find("tool_call_id")) r.set("tool_call_id", *id);
            Value o = Value::object();
            o.set("tool_response", r);
            m.set("content", Value(o.json_text(2)));
            m.erase("name");
        }
        if (!m.find("content")) m.set("content", Value());  // (a lookup that adds the key)
        const Value content = *m.find("content");
        if (!content.is_null() && poly_system) {
            if (!content.is_string()) throw std::runtime_error("content must be a string");
            const std::string& text = content.str();
            if (role == "system") {
                if (!pending.empty()) pending += "\n";
                pending += text;
                continue;
            }
            if (role == "user") {
                if (!pending.empty()) {
                    m.set("content", Value(pending + (text.empty() ? "" : "\n" + text)));
                    pending.clear();
                }
            } else {
                flush();
            }
        }
        add(m);
    }
    flush();
    return raw_render(actual, tools_var, add_generation_prompt);
}

}  // namespace minfer
