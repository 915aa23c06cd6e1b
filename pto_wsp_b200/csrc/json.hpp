// Minimal JSON reader for workload plans (objects, arrays, strings, integers
// kept exact as 64-bit, doubles, bools, null).  Plans are produced by
// pto_wsp_b200/plan.py; this parser only needs to read that output.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace ptowsp::json {

struct Value {
    enum class Type { Null, Bool, Int, Double, String, Array, Object };
    Type type = Type::Null;
    bool b = false;
    int64_t i = 0;        // Int (also holds u64 bit pattern when is_unsigned)
    bool is_unsigned = false;
    double d = 0.0;
    std::string s;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool is_null() const { return type == Type::Null; }
    bool is_obj() const { return type == Type::Object; }
    bool is_arr() const { return type == Type::Array; }
    bool has(const std::string& k) const { return type == Type::Object && obj.count(k) != 0; }
    const Value& at(const std::string& k) const {
        auto it = obj.find(k);
        if (type != Type::Object || it == obj.end()) throw std::runtime_error("plan: missing key '" + k + "'");
        return it->second;
    }
    const Value* get(const std::string& k) const {
        if (type != Type::Object) return nullptr;
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
    int64_t as_i64() const {
        if (type == Type::Int) return i;
        if (type == Type::Double) return static_cast<int64_t>(d);
        if (type == Type::Bool) return b ? 1 : 0;
        if (type == Type::String) return static_cast<int64_t>(std::stoull(s, nullptr, 0));
        throw std::runtime_error("plan: expected integer");
    }
    uint64_t as_u64() const {
        if (type == Type::String) return std::stoull(s, nullptr, 0);
        return static_cast<uint64_t>(as_i64());
    }
    double as_f64() const {
        if (type == Type::Double) return d;
        if (type == Type::Int) return is_unsigned ? static_cast<double>(static_cast<uint64_t>(i)) : static_cast<double>(i);
        if (type == Type::Bool) return b ? 1.0 : 0.0;
        throw std::runtime_error("plan: expected number");
    }
    const std::string& as_str() const {
        if (type != Type::String) throw std::runtime_error("plan: expected string");
        return s;
    }
};

class Parser {
public:
    Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
    Value parse() {
        Value v = value();
        ws();
        if (p_ != end_) throw std::runtime_error("plan: trailing characters after JSON value");
        return v;
    }

private:
    const char* p_;
    const char* end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r')) ++p_;
    }
    [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("plan: JSON ") + what); }
    char peek() {
        ws();
        if (p_ >= end_) fail("unexpected end");
        return *p_;
    }
    Value value() {
        char c = peek();
        if (c == '{') return object();
        if (c == '[') return array();
        if (c == '"') {
            Value v;
            v.type = Value::Type::String;
            v.s = string();
            return v;
        }
        if (c == 't' || c == 'f' || c == 'n') return literal();
        return number();
    }
    Value literal() {
        Value v;
        auto match = [&](const char* w) {
            size_t n = std::char_traits<char>::length(w);
            if (static_cast<size_t>(end_ - p_) >= n && std::equal(w, w + n, p_)) {
                p_ += n;
                return true;
            }
            return false;
        };
        if (match("true")) {
            v.type = Value::Type::Bool;
            v.b = true;
        } else if (match("false")) {
            v.type = Value::Type::Bool;
            v.b = false;
        } else if (match("null")) {
            v.type = Value::Type::Null;
        } else {
            fail("bad literal");
        }
        return v;
    }
    Value number() {
        const char* start = p_;
        bool is_float = false;
        if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
        while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' || *p_ == '+')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') is_float = true;
            ++p_;
        }
        std::string tok(start, p_);
        if (tok.empty()) fail("bad number");
        Value v;
        if (is_float) {
            v.type = Value::Type::Double;
            v.d = std::strtod(tok.c_str(), nullptr);
        } else {
            v.type = Value::Type::Int;
            if (tok[0] == '-') {
                v.i = std::strtoll(tok.c_str(), nullptr, 10);
            } else {
                uint64_t u = std::strtoull(tok.c_str(), nullptr, 10);
                v.i = static_cast<int64_t>(u);
                v.is_unsigned = u > static_cast<uint64_t>(INT64_MAX);
            }
        }
        return v;
    }
    std::string string() {
        if (*p_ != '"') fail("expected string");
        ++p_;
        std::string out;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c == '\\') {
                if (p_ >= end_) fail("bad escape");
                char e = *p_++;
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (end_ - p_ < 4) fail("bad unicode escape");
                        unsigned cp = static_cast<unsigned>(std::strtoul(std::string(p_, p_ + 4).c_str(), nullptr, 16));
                        p_ += 4;
                        if (cp < 0x80) {
                            out += static_cast<char>(cp);
                        } else if (cp < 0x800) {
                            out += static_cast<char>(0xC0 | (cp >> 6));
                            out += static_cast<char>(0x80 | (cp & 0x3F));
                        } else {
                            out += static_cast<char>(0xE0 | (cp >> 12));
                            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
                            out += static_cast<char>(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: out += e; break;
                }
            } else {
                out += c;
            }
        }
        if (p_ >= end_) fail("unterminated string");
        ++p_;
        return out;
    }
    Value array() {
        ++p_;
        Value v;
        v.type = Value::Type::Array;
        if (peek() == ']') {
            ++p_;
            return v;
        }
        for (;;) {
            v.arr.push_back(value());
            char c = peek();
            ++p_;
            if (c == ']') break;
            if (c != ',') fail("expected , or ]");
        }
        return v;
    }
    Value object() {
        ++p_;
        Value v;
        v.type = Value::Type::Object;
        if (peek() == '}') {
            ++p_;
            return v;
        }
        for (;;) {
            peek();
            std::string k = string();
            if (peek() != ':') fail("expected :");
            ++p_;
            v.obj[k] = value();
            char c = peek();
            ++p_;
            if (c == '}') break;
            if (c != ',') fail("expected , or }");
        }
        return v;
    }
};

inline Value parse(const char* p, size_t n) { return Parser(p, n).parse(); }

}  // namespace ptowsp::json
