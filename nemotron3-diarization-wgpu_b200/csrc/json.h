// Minimal JSON reader for config.json, processor_config.json and the
// safetensors header (objects, arrays, numbers, strings, true/false/null).
#pragma once

#include <charconv>
#include <cmath>
#include <cstdlib>
#include <stdexcept>
#include <system_error>
#include <string>
#include <utility>
#include <vector>

namespace n3d {
namespace json {

struct Value {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;

    const Value* get(const std::string& key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class Parser {
  public:
    explicit Parser(const std::string& s) : s_(s) {}
    Value parse_document() {
        Value v = value();
        ws();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

  private:
    // Deeper nesting is an error: the files read here are three levels deep, and the
    // recursion below must not be driven into a stack overflow by a damaged file.
    static constexpr int kMaxDepth = 128;
    struct Nest {
        Parser& p;
        explicit Nest(Parser& q) : p(q) {
            if (++p.depth_ > kMaxDepth) p.fail("nesting too deep");
        }
        ~Nest() { p.depth_--; }
    };

    [[noreturn]] void fail(const char* what) {
        throw std::runtime_error(std::string(what) + " at byte " + std::to_string(i_));
    }
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
    }
    bool lit(const char* w) {
        size_t n = 0;
        while (w[n]) n++;
        if (s_.compare(i_, n, w) == 0) {
            i_ += n;
            return true;
        }
        return false;
    }
    Value value() {
        ws();
        if (i_ >= s_.size()) fail("unexpected end");
        const char c = s_[i_];
        Value v;
        if (c == '{') {
            const Nest nest(*this);
            v.kind = Value::Obj;
            i_++;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') {
                i_++;
                return v;
            }
            for (;;) {
                ws();
                if (i_ >= s_.size() || s_[i_] != '"') fail("expected key");
                std::string k = string();
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
                i_++;
                v.obj.emplace_back(std::move(k), value());
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    i_++;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') {
                    i_++;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            const Nest nest(*this);
            v.kind = Value::Arr;
            i_++;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') {
                i_++;
                return v;
            }
            for (;;) {
                v.arr.push_back(value());
                ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    i_++;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') {
                    i_++;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Value::Str;
            v.str = string();
            return v;
        }
        if (lit("true")) {
            v.kind = Value::Bool;
            v.b = true;
            return v;
        }
        if (lit("false")) {
            v.kind = Value::Bool;
            return v;
        }
        if (lit("null")) return v;
        // from_chars reads the C number format whatever locale the host process has set
        // (strtod would stop at the '.' under a locale with a decimal comma)
        const char* start = s_.data() + i_;
        const std::from_chars_result r = std::from_chars(start, s_.data() + s_.size(), v.num);
        if (r.ec == std::errc::result_out_of_range) fail("number out of range");
        if (r.ec != std::errc() || r.ptr == start || !std::isfinite(v.num)) fail("bad value");  // no nan / inf
        v.kind = Value::Num;
        i_ += (size_t)(r.ptr - start);
        return v;
    }
    std::string string() {
        std::string out;
        i_++;  // opening quote
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) fail("bad escape");
                const char e = s_[i_++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (i_ + 4 > s_.size()) fail("bad \\u escape");
                        const unsigned cp = (unsigned)std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16);
                        i_ += 4;
                        if (cp < 0x80) {
                            out += (char)cp;
                        } else if (cp < 0x800) {
                            out += (char)(0xC0 | (cp >> 6));
                            out += (char)(0x80 | (cp & 0x3F));
                        } else {
                            out += (char)(0xE0 | (cp >> 12));
                            out += (char)(0x80 | ((cp >> 6) & 0x3F));
                            out += (char)(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i_ >= s_.size()) fail("unterminated string");
        i_++;
        return out;
    }
    const std::string& s_;
    size_t i_ = 0;
    int depth_ = 0;
};

inline Value parse(const std::string& s) { return Parser(s).parse_document(); }

}  // namespace json
}  // namespace n3d
