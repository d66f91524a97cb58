// Minimal JSON reader for the model files (graph.json, the weight manifest). The reference reads them with serde_json
// (crates/flyhigh-engine/src/model/mod.rs:38-82); this is a small recursive-descent parser of RFC 8259 JSON with the
// accessors the loader and the planner need. Errors throw std::runtime_error with the byte offset.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace fhjson {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;  // insertion order kept (graph op field order is irrelevant)

    bool is_null() const { return kind == Null; }
    bool is_string() const { return kind == String; }
    bool is_number() const { return kind == Number; }
    bool is_array() const { return kind == Array; }
    bool is_object() const { return kind == Object; }
    bool is_bool() const { return kind == Bool; }

    const Value* find(const std::string& k) const {
        if (kind != Object) return nullptr;
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    // missing keys and wrong kinds read as a shared null, like serde_json's `value["key"]`
    const Value& operator[](const std::string& k) const {
        static const Value null_value;
        const Value* v = find(k);
        return v ? *v : null_value;
    }
    const Value& operator[](size_t i) const {
        static const Value null_value;
        return (kind == Array && i < arr.size()) ? arr[i] : null_value;
    }
    size_t size() const { return kind == Array ? arr.size() : (kind == Object ? obj.size() : 0); }
    std::string as_str(const std::string& dflt = "") const { return kind == String ? str : dflt; }
    double as_num(double dflt = 0.0) const { return kind == Number ? num : dflt; }
    bool as_bool(bool dflt = false) const { return kind == Bool ? b : dflt; }
    // an unsigned integer (serde's as_u64): only non-negative integral numbers qualify
    bool is_u64() const { return kind == Number && num >= 0 && num < 18446744073709551616.0 && num == (double)(uint64_t)num; }
};

class Parser {
  public:
    Parser(const char* p, size_t n) : s_(p), n_(n) {}
    Value parse() {
        Value v = value();
        ws();
        if (i_ != n_) fail("trailing characters");
        return v;
    }

  private:
    const char* s_;
    size_t n_;
    size_t i_ = 0;
    int depth_ = 0;

    [[noreturn]] void fail(const char* what) {
        throw std::runtime_error(std::string("json: ") + what + " at byte " + std::to_string(i_));
    }
    void ws() {
        while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
    }
    bool lit(const char* w) {
        size_t k = 0;
        while (w[k]) {
            if (i_ + k >= n_ || s_[i_ + k] != w[k]) return false;
            k++;
        }
        i_ += k;
        return true;
    }
    Value value() {
        if (++depth_ > 256) fail("nesting too deep");
        ws();
        if (i_ >= n_) fail("unexpected end");
        Value v;
        char c = s_[i_];
        if (c == '{') {
            v.kind = Value::Object;
            i_++;
            ws();
            if (i_ < n_ && s_[i_] == '}') {
                i_++;
            } else {
                for (;;) {
                    ws();
                    if (i_ >= n_ || s_[i_] != '"') fail("expected a key");
                    std::string k = string();
                    ws();
                    if (i_ >= n_ || s_[i_] != ':') fail("expected ':'");
                    i_++;
                    v.obj.emplace_back(std::move(k), value());
                    ws();
                    if (i_ < n_ && s_[i_] == ',') { i_++; continue; }
                    if (i_ < n_ && s_[i_] == '}') { i_++; break; }
                    fail("expected ',' or '}'");
                }
            }
        } else if (c == '[') {
            v.kind = Value::Array;
            i_++;
            ws();
            if (i_ < n_ && s_[i_] == ']') {
                i_++;
            } else {
                for (;;) {
                    v.arr.push_back(value());
                    ws();
                    if (i_ < n_ && s_[i_] == ',') { i_++; continue; }
                    if (i_ < n_ && s_[i_] == ']') { i_++; break; }
                    fail("expected ',' or ']'");
                }
            }
        } else if (c == '"') {
            v.kind = Value::String;
            v.str = string();
        } else if (lit("true")) {
            v.kind = Value::Bool;
            v.b = true;
        } else if (lit("false")) {
            v.kind = Value::Bool;
        } else if (lit("null")) {
            v.kind = Value::Null;
        } else if (c == '-' || (c >= '0' && c <= '9')) {
            v.kind = Value::Number;
            size_t st = i_;
            if (s_[i_] == '-') i_++;
            while (i_ < n_ && ((s_[i_] >= '0' && s_[i_] <= '9') || s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E' ||
                               s_[i_] == '+' || s_[i_] == '-'))
                i_++;
            std::string t(s_ + st, i_ - st);
            char* end = nullptr;
            v.num = std::strtod(t.c_str(), &end);
            if (!end || *end) fail("bad number");
        } else {
            fail("unexpected character");
        }
        depth_--;
        return v;
    }
    static void utf8(std::string& o, uint32_t cp) {
        if (cp < 0x80) {
            o += (char)cp;
        } else if (cp < 0x800) {
            o += (char)(0xC0 | (cp >> 6));
            o += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += (char)(0xE0 | (cp >> 12));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        } else {
            o += (char)(0xF0 | (cp >> 18));
            o += (char)(0x80 | ((cp >> 12) & 0x3F));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (i_ + 4 > n_) fail("bad escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; k++) {
            char c = s_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= c - '0';
            else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
            else fail("bad hex digit");
        }
        return v;
    }
    std::string string() {
        i_++;  // opening quote
        std::string o;
        for (;;) {
            if (i_ >= n_) fail("unterminated string");
            char c = s_[i_++];
            if (c == '"') break;
            if ((unsigned char)c < 0x20) fail("control character in string");
            if (c != '\\') { o += c; continue; }
            if (i_ >= n_) fail("bad escape");
            char e = s_[i_++];
            switch (e) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && i_ + 1 < n_ && s_[i_] == '\\' && s_[i_ + 1] == 'u') {
                        i_ += 2;
                        uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(o, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
        return o;
    }
};

inline Value parse(const std::string& text) { return Parser(text.data(), text.size()).parse(); }
inline Value parse(const uint8_t* p, size_t n) { return Parser((const char*)p, n).parse(); }

// JSON string literal of `s` (for the report writers)
inline std::string quote(const std::string& s) {
    std::string o = "\"";
    for (char c : s) {
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c == '\n') o += "\\n";
        else if ((unsigned char)c < 0x20) {
            char b[8];
            snprintf(b, sizeof b, "\\u%04x", c);
            o += b;
        } else o += c;
    }
    return o + "\"";
}

}  // namespace fhjson
