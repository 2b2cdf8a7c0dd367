// Minimal JSON reader for bundle manifests (objects, arrays, strings with
// escapes, numbers, booleans, null).  Plays the role of the reference's
// JsonParser (Mac/cpu/src/json_parser.cpp) for manifest.json.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace socb {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    bool is_int = false;
    int64_t i64 = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    bool is_object() const { return kind == Object; }
    bool is_array() const { return kind == Array; }
    bool is_null() const { return kind == Null; }
    bool contains(const std::string& k) const {
        if (kind != Object) return false;
        for (auto& kv : obj)
            if (kv.first == k) return true;
        return false;
    }
    const Json& at(const std::string& k) const {
        if (kind != Object) throw std::runtime_error("json value is not an object (key " + k + ")");
        for (auto& kv : obj)
            if (kv.first == k) return kv.second;
        throw std::runtime_error("json object is missing key: " + k);
    }
    const std::string& as_string() const {
        if (kind != String) throw std::runtime_error("json value is not a string");
        return str;
    }
    double as_number() const {
        if (kind != Number) throw std::runtime_error("json value is not a number");
        return num;
    }
    int64_t as_int64() const {
        if (kind != Number) throw std::runtime_error("json value is not a number");
        return is_int ? i64 : static_cast<int64_t>(num);
    }
    bool as_bool() const {
        if (kind != Bool) throw std::runtime_error("json value is not a boolean");
        return b;
    }
    const std::vector<Json>& as_array() const {
        if (kind != Array) throw std::runtime_error("json value is not an array");
        return arr;
    }
};

class JsonReader {
public:
    explicit JsonReader(const std::string& text) : s_(text) {}
    Json parse() {
        Json v = value();
        ws();
        if (p_ != s_.size()) fail("trailing characters");
        return v;
    }

private:
    const std::string& s_;
    size_t p_ = 0;

    [[noreturn]] void fail(const char* what) {
        throw std::runtime_error(std::string("json parse error: ") + what + " at offset " + std::to_string(p_));
    }
    void ws() {
        while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\r' || s_[p_] == '\t')) ++p_;
    }
    bool lit(const char* w) {
        size_t n = std::char_traits<char>::length(w);
        if (s_.compare(p_, n, w) == 0) {
            p_ += n;
            return true;
        }
        return false;
    }
    Json value() {
        ws();
        if (p_ >= s_.size()) fail("unexpected end");
        char c = s_[p_];
        Json v;
        if (c == '{') {
            v.kind = Json::Object;
            ++p_;
            ws();
            if (p_ < s_.size() && s_[p_] == '}') {
                ++p_;
                return v;
            }
            for (;;) {
                ws();
                if (p_ >= s_.size() || s_[p_] != '"') fail("expected key");
                std::string k = string();
                ws();
                if (p_ >= s_.size() || s_[p_] != ':') fail("expected ':'");
                ++p_;
                v.obj.emplace_back(std::move(k), value());
                ws();
                if (p_ < s_.size() && s_[p_] == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < s_.size() && s_[p_] == '}') {
                    ++p_;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::Array;
            ++p_;
            ws();
            if (p_ < s_.size() && s_[p_] == ']') {
                ++p_;
                return v;
            }
            for (;;) {
                v.arr.push_back(value());
                ws();
                if (p_ < s_.size() && s_[p_] == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < s_.size() && s_[p_] == ']') {
                    ++p_;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::String;
            v.str = string();
            return v;
        }
        if (lit("true")) {
            v.kind = Json::Bool;
            v.b = true;
            return v;
        }
        if (lit("false")) {
            v.kind = Json::Bool;
            return v;
        }
        if (lit("null")) return v;
        if (lit("NaN") || lit("Infinity") || lit("-Infinity")) {
            v.kind = Json::Number;
            return v;
        }
        return number();
    }
    Json number() {
        size_t start = p_;
        bool integral = true;
        if (s_[p_] == '-') ++p_;
        while (p_ < s_.size()) {
            char c = s_[p_];
            if (c >= '0' && c <= '9') {
                ++p_;
            } else if (c == '.' || c == 'e' || c == 'E' || c == '+' || c == '-') {
                integral = false;
                ++p_;
            } else {
                break;
            }
        }
        if (p_ == start) fail("invalid value");
        std::string tok = s_.substr(start, p_ - start);
        Json v;
        v.kind = Json::Number;
        v.num = std::strtod(tok.c_str(), nullptr);
        if (integral) {
            v.is_int = true;
            v.i64 = std::strtoll(tok.c_str(), nullptr, 10);
        }
        return v;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (p_ + 4 > s_.size()) fail("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            char c = s_[p_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
            else fail("bad hex digit");
        }
        return v;
    }
    std::string string() {
        ++p_;  // opening quote
        std::string out;
        while (p_ < s_.size()) {
            char c = s_[p_++];
            if (c == '"') return out;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (p_ >= s_.size()) break;
            char e = s_[p_++];
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
                    if (cp >= 0xD800 && cp <= 0xDBFF && p_ + 6 <= s_.size() && s_[p_] == '\\' && s_[p_ + 1] == 'u') {
                        p_ += 2;
                        uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
        fail("unterminated string");
    }
};

}  // namespace socb
