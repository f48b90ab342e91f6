// dag_json.cuh -- a small JSON reader for the serialized Chelis DAG.
//
// The DAG crosses the boundary as the JSON that serde writes for
// crates/chelis-dag-core's `Dag` (dag.rs:2913-2920; node layout
// tests/wire_behavior.rs): objects, arrays, strings, integers that must stay
// exact (i64 payloads up to 2^63), and no floats in the graph itself (float
// constants travel as hex bit strings).  Integers without a fraction or
// exponent are kept as int64; other numbers as double.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

namespace chelis {
namespace json {

struct Value {
    enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    int64_t i = 0;
    double d = 0.0;
    std::string s;
    std::vector<Value> a;
    std::vector<std::pair<std::string, Value>> o;

    const Value *get(const char *key) const {
        if (kind != Obj) return nullptr;
        for (const auto &kv : o)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    bool is_null() const { return kind == Null; }
};

class Reader {
  public:
    Reader(const char *text, size_t len) : p_(text), end_(text + len) {}
    // false (with `error()` set) on malformed input or trailing bytes
    bool parse(Value *out) {
        skip();
        if (!value(out, 0)) return false;
        skip();
        if (p_ != end_) return fail("trailing bytes after the document");
        return true;
    }
    const std::string &error() const { return err_; }

  private:
    const char *p_;
    const char *end_;
    std::string err_;

    bool fail(const char *what) {
        if (err_.empty()) err_ = what;
        return false;
    }
    void skip() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool literal(const char *word) {
        const char *q = p_;
        for (; *word; ++word, ++q)
            if (q >= end_ || *q != *word) return false;
        p_ = q;
        return true;
    }
    bool value(Value *v, int depth) {
        if (depth > 256) return fail("nesting too deep");
        if (p_ >= end_) return fail("unexpected end of input");
        switch (*p_) {
            case '{': return object(v, depth);
            case '[': return array(v, depth);
            case '"': v->kind = Value::Str; return string(&v->s);
            case 't': v->kind = Value::Bool; v->b = true; return literal("true") || fail("bad literal");
            case 'f': v->kind = Value::Bool; v->b = false; return literal("false") || fail("bad literal");
            case 'n': v->kind = Value::Null; return literal("null") || fail("bad literal");
            default: return number(v);
        }
    }
    bool object(Value *v, int depth) {
        v->kind = Value::Obj;
        ++p_;
        skip();
        if (p_ < end_ && *p_ == '}') {
            ++p_;
            return true;
        }
        for (;;) {
            skip();
            if (p_ >= end_ || *p_ != '"') return fail("object key expected");
            std::string key;
            if (!string(&key)) return false;
            skip();
            if (p_ >= end_ || *p_ != ':') return fail("':' expected");
            ++p_;
            skip();
            v->o.emplace_back(std::move(key), Value());
            if (!value(&v->o.back().second, depth + 1)) return false;
            skip();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            return fail("',' or '}' expected");
        }
    }
    bool array(Value *v, int depth) {
        v->kind = Value::Arr;
        ++p_;
        skip();
        if (p_ < end_ && *p_ == ']') {
            ++p_;
            return true;
        }
        for (;;) {
            skip();
            v->a.emplace_back();
            if (!value(&v->a.back(), depth + 1)) return false;
            skip();
            if (p_ < end_ && *p_ == ',') {
                ++p_;
                continue;
            }
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            return fail("',' or ']' expected");
        }
    }
    static int hexval(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    void utf8(uint32_t cp, std::string *s) {
        if (cp < 0x80) {
            s->push_back(static_cast<char>(cp));
        } else if (cp < 0x800) {
            s->push_back(static_cast<char>(0xC0 | (cp >> 6)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            s->push_back(static_cast<char>(0xE0 | (cp >> 12)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else {
            s->push_back(static_cast<char>(0xF0 | (cp >> 18)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        }
    }
    bool string(std::string *s) {
        ++p_;  // opening quote
        while (p_ < end_ && *p_ != '"') {
            if (static_cast<unsigned char>(*p_) < 0x20) return fail("control byte in string");
            if (*p_ != '\\') {
                s->push_back(*p_++);
                continue;
            }
            if (++p_ >= end_) return fail("unterminated escape");
            const char c = *p_++;
            switch (c) {
                case '"': s->push_back('"'); break;
                case '\\': s->push_back('\\'); break;
                case '/': s->push_back('/'); break;
                case 'b': s->push_back('\b'); break;
                case 'f': s->push_back('\f'); break;
                case 'n': s->push_back('\n'); break;
                case 'r': s->push_back('\r'); break;
                case 't': s->push_back('\t'); break;
                case 'u': {
                    if (end_ - p_ < 4) return fail("short \\u escape");
                    uint32_t cp = 0;
                    for (int k = 0; k < 4; ++k) {
                        const int h = hexval(p_[k]);
                        if (h < 0) return fail("bad \\u escape");
                        cp = (cp << 4) | static_cast<uint32_t>(h);
                    }
                    p_ += 4;
                    utf8(cp, s);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p_ >= end_) return fail("unterminated string");
        ++p_;
        return true;
    }
    bool number(Value *v) {
        const char *start = p_;
        bool integral = true;
        if (p_ < end_ && *p_ == '-') ++p_;
        if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("value expected");
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        if (p_ < end_ && *p_ == '.') {
            integral = false;
            ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        const std::string text(start, p_);
        if (integral) {
            // exact int64 (overflow is an error, not a rounding)
            const bool neg = text[0] == '-';
            uint64_t mag = 0;
            for (size_t k = neg ? 1 : 0; k < text.size(); ++k) {
                const uint64_t digit = static_cast<uint64_t>(text[k] - '0');
                if (mag > (UINT64_MAX - digit) / 10) return fail("integer out of range");
                mag = mag * 10 + digit;
            }
            if ((!neg && mag > static_cast<uint64_t>(INT64_MAX)) ||
                (neg && mag > static_cast<uint64_t>(INT64_MAX) + 1))
                return fail("integer out of range");
            v->kind = Value::Int;
            v->i = neg ? static_cast<int64_t>(0 - mag) : static_cast<int64_t>(mag);
            v->d = static_cast<double>(v->i);
            return true;
        }
        v->kind = Value::Num;
        v->d = std::strtod(text.c_str(), nullptr);
        return true;
    }
};

}  // namespace json
}  // namespace chelis
