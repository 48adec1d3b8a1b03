// tl_json.h -- minimal JSON reader for the model binary header.
//
// The header written by export_mistral.py (json.dumps of metadata, tensors
// and tokenizer; export_mistral.py:143-150) only uses objects, arrays,
// strings, integers and floats.  This parser builds a small DOM, keeps object
// member order, decodes string escapes (\uXXXX to UTF-8, surrogate pairs
// included) and keeps integers exact as int64.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace tl {

struct JValue {
    enum Type { Null, Bool, Int, Float, Str, Arr, Obj } type = Null;
    bool b = false;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;

    const JValue* get(const char* key) const {
        if (type != Obj) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
    bool is_num() const { return type == Int || type == Float; }
};

class JsonParser {
  public:
    JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}

    bool parse(JValue& out, std::string& err) {
        if (!value(out, 0)) {
            err = err_.empty() ? "invalid JSON" : err_;
            return false;
        }
        ws();
        if (p_ != end_) {
            err = "trailing characters after JSON value";
            return false;
        }
        return true;
    }

  private:
    const char* p_;
    const char* end_;
    std::string err_;

    bool fail(const char* m) {
        if (err_.empty()) err_ = m;
        return false;
    }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return fail("bad literal");
        p_ += n;
        return true;
    }
    static void utf8(std::string& o, uint32_t c) {
        if (c < 0x80) {
            o += static_cast<char>(c);
        } else if (c < 0x800) {
            o += static_cast<char>(0xC0 | (c >> 6));
            o += static_cast<char>(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            o += static_cast<char>(0xE0 | (c >> 12));
            o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
            o += static_cast<char>(0x80 | (c & 0x3F));
        } else {
            o += static_cast<char>(0xF0 | (c >> 18));
            o += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
            o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
            o += static_cast<char>(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& c) {
        if (end_ - p_ < 4) return fail("short \\u escape");
        c = 0;
        for (int k = 0; k < 4; k++) {
            const char h = *p_++;
            c <<= 4;
            if (h >= '0' && h <= '9') c |= h - '0';
            else if (h >= 'a' && h <= 'f') c |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') c |= h - 'A' + 10;
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string& o) {
        if (p_ >= end_ || *p_ != '"') return fail("expected string");
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (p_ >= end_) return fail("unterminated escape");
            c = *p_++;
            switch (c) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp <= 0xDBFF && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        uint32_t lo;
                        if (!hex4(lo)) return false;
                        if (lo >= 0xDC00 && lo <= 0xDFFF) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        else { utf8(o, cp); cp = lo; }
                    }
                    utf8(o, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p_ >= end_) return fail("unterminated string");
        ++p_;
        return true;
    }
    bool number(JValue& v) {
        const char* s = p_;
        bool is_float = false;
        if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
        while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                             *p_ == '-' || *p_ == '+')) {
            if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') is_float = true;
            ++p_;
        }
        std::string tok(s, p_);
        if (tok.empty() || tok == "-") return fail("bad number");
        char* e = nullptr;
        if (!is_float) {
            v.type = JValue::Int;
            v.i = std::strtoll(tok.c_str(), &e, 10);
            v.f = static_cast<double>(v.i);
        } else {
            v.type = JValue::Float;
            v.f = std::strtod(tok.c_str(), &e);
            v.i = static_cast<int64_t>(v.f);
        }
        if (!e || *e != '\0') return fail("bad number");
        return true;
    }
    bool value(JValue& v, int depth) {
        if (depth > 64) return fail("JSON nested too deeply");
        ws();
        if (p_ >= end_) return fail("unexpected end of JSON");
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.type = JValue::Obj;
            ws();
            if (p_ < end_ && *p_ == '}') { ++p_; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
                ++p_;
                v.obj.emplace_back(std::move(k), JValue());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == '}') { ++p_; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p_;
            v.type = JValue::Arr;
            ws();
            if (p_ < end_ && *p_ == ']') { ++p_; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == ']') { ++p_; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.type = JValue::Str;
            return string(v.s);
        }
        if (c == 't') { v.type = JValue::Bool; v.b = true; return lit("true"); }
        if (c == 'f') { v.type = JValue::Bool; v.b = false; return lit("false"); }
        if (c == 'n') { v.type = JValue::Null; return lit("null"); }
        return number(v);
    }
};

}  // namespace tl
