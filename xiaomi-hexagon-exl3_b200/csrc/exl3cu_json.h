// Minimal JSON reader for the model loader: safetensors headers and the
// deployment manifest (RFC 8259 grammar).  Host code only.
//
// * Values: null, bool, integer (a number without fraction or exponent that
//   fits int64), real (every other number), string (UTF-8; escapes decoded,
//   \u surrogate pairs joined), array, object (keys in document order).
// * Strict: control characters inside strings, leading zeros, trailing
//   commas, trailing garbage and nesting deeper than kMaxDepth are errors.
//   A key that appears twice in one object is an error too.
// * parse() throws JsonError with the byte offset of the problem.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace exl3cu {
namespace json {

struct JsonError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

enum class Kind { Null, Bool, Int, Real, String, Array, Object };

struct Value {
    Kind kind = Kind::Null;
    bool b = false;
    int64_t i = 0;
    double d = 0.0;
    std::string s;
    std::vector<Value> items;                          // Array
    std::vector<std::pair<std::string, Value>> members;  // Object, document order

    bool is_int() const { return kind == Kind::Int; }
    bool is_number() const { return kind == Kind::Int || kind == Kind::Real; }
    bool is_string() const { return kind == Kind::String; }
    bool is_array() const { return kind == Kind::Array; }
    bool is_object() const { return kind == Kind::Object; }
    double number() const { return kind == Kind::Int ? double(i) : d; }

    // Member `key` of an object, or nullptr (also when this is not an object).
    const Value * find(const std::string & key) const {
        if (kind != Kind::Object) return nullptr;
        for (const auto & m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
    // Member `key`; throws JsonError naming the key when absent.
    const Value & at(const std::string & key) const {
        const Value * v = find(key);
        if (!v) throw JsonError("missing key \"" + key + "\"");
        return *v;
    }
    bool equals_string(const char * text) const { return kind == Kind::String && s == text; }
    bool equals_int(int64_t v) const { return (kind == Kind::Int && i == v) || (kind == Kind::Real && d == double(v)); }
};

class Parser {
public:
    static constexpr int kMaxDepth = 64;

    Parser(const char * begin, const char * end) : p_(begin), b_(begin), e_(end) {}

    Value parse_document() {
        Value v = value(0);
        ws();
        if (p_ != e_) fail("trailing characters after the JSON value");
        return v;
    }

private:
    const char * p_;
    const char * b_;
    const char * e_;

    [[noreturn]] void fail(const char * what) const {
        throw JsonError(std::string("JSON: ") + what + " at byte " + std::to_string(size_t(p_ - b_)));
    }
    void ws() {
        while (p_ != e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool literal(const char * word) {
        const size_t n = std::strlen(word);
        if (size_t(e_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
        p_ += n;
        return true;
    }

    Value value(int depth) {
        if (depth > kMaxDepth) fail("nesting too deep");
        ws();
        if (p_ == e_) fail("unexpected end of input");
        Value v;
        switch (*p_) {
            case '{': object(v, depth); return v;
            case '[': array(v, depth); return v;
            case '"': v.kind = Kind::String; v.s = string(); return v;
            case 't': if (!literal("true")) fail("invalid literal"); v.kind = Kind::Bool; v.b = true; return v;
            case 'f': if (!literal("false")) fail("invalid literal"); v.kind = Kind::Bool; return v;
            case 'n': if (!literal("null")) fail("invalid literal"); return v;
            default: number(v); return v;
        }
    }

    void object(Value & v, int depth) {
        v.kind = Kind::Object;
        ++p_;  // '{'
        ws();
        if (p_ != e_ && *p_ == '}') { ++p_; return; }
        for (;;) {
            ws();
            if (p_ == e_ || *p_ != '"') fail("expected a string key");
            std::string key = string();
            for (const auto & m : v.members)
                if (m.first == key) fail("duplicate key");
            ws();
            if (p_ == e_ || *p_ != ':') fail("expected ':'");
            ++p_;
            Value item = value(depth + 1);
            v.members.emplace_back(std::move(key), std::move(item));
            ws();
            if (p_ == e_) fail("unterminated object");
            if (*p_ == ',') { ++p_; continue; }
            if (*p_ == '}') { ++p_; return; }
            fail("expected ',' or '}'");
        }
    }

    void array(Value & v, int depth) {
        v.kind = Kind::Array;
        ++p_;  // '['
        ws();
        if (p_ != e_ && *p_ == ']') { ++p_; return; }
        for (;;) {
            v.items.push_back(value(depth + 1));
            ws();
            if (p_ == e_) fail("unterminated array");
            if (*p_ == ',') { ++p_; continue; }
            if (*p_ == ']') { ++p_; return; }
            fail("expected ',' or ']'");
        }
    }

    unsigned hex4() {
        if (e_ - p_ < 4) fail("truncated \\u escape");
        unsigned u = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = *p_++;
            u <<= 4;
            if (c >= '0' && c <= '9') u |= unsigned(c - '0');
            else if (c >= 'a' && c <= 'f') u |= unsigned(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') u |= unsigned(c - 'A' + 10);
            else fail("invalid \\u escape");
        }
        return u;
    }

    static void utf8(std::string & out, unsigned cp) {
        if (cp < 0x80) {
            out += char(cp);
        } else if (cp < 0x800) {
            out += char(0xc0 | (cp >> 6));
            out += char(0x80 | (cp & 0x3f));
        } else if (cp < 0x10000) {
            out += char(0xe0 | (cp >> 12));
            out += char(0x80 | ((cp >> 6) & 0x3f));
            out += char(0x80 | (cp & 0x3f));
        } else {
            out += char(0xf0 | (cp >> 18));
            out += char(0x80 | ((cp >> 12) & 0x3f));
            out += char(0x80 | ((cp >> 6) & 0x3f));
            out += char(0x80 | (cp & 0x3f));
        }
    }

    std::string string() {
        ++p_;  // opening quote
        std::string out;
        for (;;) {
            if (p_ == e_) fail("unterminated string");
            const unsigned char c = static_cast<unsigned char>(*p_++);
            if (c == '"') return out;
            if (c < 0x20) fail("control character in string");
            if (c != '\\') { out += char(c); continue; }
            if (p_ == e_) fail("unterminated escape");
            const char esc = *p_++;
            switch (esc) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    unsigned cp = hex4();
                    if (cp >= 0xd800 && cp < 0xdc00) {
                        if (e_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') fail("unpaired surrogate");
                        p_ += 2;
                        const unsigned lo = hex4();
                        if (lo < 0xdc00 || lo >= 0xe000) fail("invalid low surrogate");
                        cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                    } else if (cp >= 0xdc00 && cp < 0xe000) {
                        fail("unpaired surrogate");
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail("invalid escape");
            }
        }
    }

    void number(Value & v) {
        const char * start = p_;
        if (p_ != e_ && *p_ == '-') ++p_;
        if (p_ == e_ || *p_ < '0' || *p_ > '9') fail("invalid value");
        if (*p_ == '0') {
            ++p_;
            if (p_ != e_ && *p_ >= '0' && *p_ <= '9') fail("leading zero");
        } else {
            while (p_ != e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        bool integral = true;
        if (p_ != e_ && *p_ == '.') {
            integral = false;
            ++p_;
            if (p_ == e_ || *p_ < '0' || *p_ > '9') fail("digit expected after '.'");
            while (p_ != e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ != e_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ != e_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ == e_ || *p_ < '0' || *p_ > '9') fail("digit expected in exponent");
            while (p_ != e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        const std::string text(start, p_);
        if (integral) {
            // Accumulate with an overflow check; out-of-range integers become reals.
            const bool neg = text[0] == '-';
            uint64_t mag = 0;
            bool overflow = false;
            for (size_t k = neg ? 1 : 0; k < text.size(); ++k) {
                const uint64_t digit = uint64_t(text[k] - '0');
                if (mag > (UINT64_MAX - digit) / 10) { overflow = true; break; }
                mag = mag * 10 + digit;
            }
            const uint64_t limit = neg ? uint64_t(INT64_MAX) + 1 : uint64_t(INT64_MAX);
            if (!overflow && mag <= limit) {
                v.kind = Kind::Int;
                v.i = neg ? int64_t(0 - mag) : int64_t(mag);
                return;
            }
        }
        v.kind = Kind::Real;
        v.d = std::strtod(text.c_str(), nullptr);
    }
};

inline Value parse(const char * begin, const char * end) { return Parser(begin, end).parse_document(); }
inline Value parse(const std::string & text) { return parse(text.data(), text.data() + text.size()); }

}  // namespace json
}  // namespace exl3cu
