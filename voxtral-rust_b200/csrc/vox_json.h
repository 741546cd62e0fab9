// vox_json.h -- a small JSON reader for the host-side file formats the
// decoder path reads: the safetensors header and tekken.json.  Parses into a
// DOM of Json values; strings are decoded to UTF-8 (\uXXXX escapes and
// surrogate pairs included); integers without a fraction or exponent keep
// their exact 64-bit value next to the double.  Errors carry the byte offset.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace vox {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    bool is_int = false;       // the literal had no fraction or exponent
    int64_t i64 = 0;           // exact value when is_int (and in range)
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;  // in file order

    const Json* get(const std::string& key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
  public:
    JsonParser(const char* p, size_t n) : s_(p), n_(n) {}

    // Parses one value spanning the whole input (trailing whitespace allowed).
    bool parse(Json* out, std::string* err) {
        pos_ = 0;
        err_.clear();
        bool ok = value(out, 0);
        if (ok) {
            ws();
            if (pos_ != n_) ok = fail("trailing characters");
        }
        if (!ok && err) *err = err_;
        return ok;
    }

  private:
    const char* s_;
    size_t n_, pos_ = 0;
    std::string err_;

    bool fail(const char* what) {
        err_ = std::string(what) + " at byte " + std::to_string(pos_);
        return false;
    }
    void ws() {
        while (pos_ < n_ && (s_[pos_] == ' ' || s_[pos_] == '\t' || s_[pos_] == '\n' || s_[pos_] == '\r')) ++pos_;
    }
    bool lit(const char* w) {
        const size_t k = std::strlen(w);
        if (pos_ + k > n_ || std::memcmp(s_ + pos_, w, k) != 0) return fail("invalid literal");
        pos_ += k;
        return true;
    }
    bool value(Json* out, int depth) {
        if (depth > 256) return fail("nesting too deep");
        ws();
        if (pos_ >= n_) return fail("unexpected end");
        const char c = s_[pos_];
        if (c == '{') return object(out, depth);
        if (c == '[') return array(out, depth);
        if (c == '"') {
            out->kind = Json::String;
            return string(&out->str);
        }
        if (c == 't') { out->kind = Json::Bool; out->b = true; return lit("true"); }
        if (c == 'f') { out->kind = Json::Bool; out->b = false; return lit("false"); }
        if (c == 'n') { out->kind = Json::Null; return lit("null"); }
        return number(out);
    }
    bool object(Json* out, int depth) {
        out->kind = Json::Object;
        ++pos_;
        ws();
        if (pos_ < n_ && s_[pos_] == '}') { ++pos_; return true; }
        for (;;) {
            ws();
            if (pos_ >= n_ || s_[pos_] != '"') return fail("expected a key");
            std::string key;
            if (!string(&key)) return false;
            ws();
            if (pos_ >= n_ || s_[pos_] != ':') return fail("expected ':'");
            ++pos_;
            out->obj.emplace_back(std::move(key), Json{});
            if (!value(&out->obj.back().second, depth + 1)) return false;
            ws();
            if (pos_ < n_ && s_[pos_] == ',') { ++pos_; continue; }
            if (pos_ < n_ && s_[pos_] == '}') { ++pos_; return true; }
            return fail("expected ',' or '}'");
        }
    }
    bool array(Json* out, int depth) {
        out->kind = Json::Array;
        ++pos_;
        ws();
        if (pos_ < n_ && s_[pos_] == ']') { ++pos_; return true; }
        for (;;) {
            out->arr.emplace_back();
            if (!value(&out->arr.back(), depth + 1)) return false;
            ws();
            if (pos_ < n_ && s_[pos_] == ',') { ++pos_; continue; }
            if (pos_ < n_ && s_[pos_] == ']') { ++pos_; return true; }
            return fail("expected ',' or ']'");
        }
    }
    static void put_utf8(std::string* o, uint32_t cp) {
        if (cp < 0x80) {
            o->push_back((char)cp);
        } else if (cp < 0x800) {
            o->push_back((char)(0xC0 | (cp >> 6)));
            o->push_back((char)(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            o->push_back((char)(0xE0 | (cp >> 12)));
            o->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o->push_back((char)(0x80 | (cp & 0x3F)));
        } else {
            o->push_back((char)(0xF0 | (cp >> 18)));
            o->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
            o->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
            o->push_back((char)(0x80 | (cp & 0x3F)));
        }
    }
    bool hex4(uint32_t* v) {
        if (pos_ + 4 > n_) return fail("short \\u escape");
        uint32_t x = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = s_[pos_ + i];
            x <<= 4;
            if (c >= '0' && c <= '9') x |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') x |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') x |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        pos_ += 4;
        *v = x;
        return true;
    }
    bool string(std::string* o) {
        ++pos_;  // opening quote
        o->clear();
        while (pos_ < n_) {
            const char c = s_[pos_];
            if (c == '"') { ++pos_; return true; }
            if ((unsigned char)c < 0x20) return fail("control character in string");
            if (c != '\\') { o->push_back(c); ++pos_; continue; }
            if (++pos_ >= n_) break;
            const char e = s_[pos_++];
            switch (e) {
                case '"': o->push_back('"'); break;
                case '\\': o->push_back('\\'); break;
                case '/': o->push_back('/'); break;
                case 'b': o->push_back('\b'); break;
                case 'f': o->push_back('\f'); break;
                case 'n': o->push_back('\n'); break;
                case 'r': o->push_back('\r'); break;
                case 't': o->push_back('\t'); break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: needs a low one
                        uint32_t lo;
                        if (pos_ + 2 > n_ || s_[pos_] != '\\' || s_[pos_ + 1] != 'u') return fail("lone surrogate");
                        pos_ += 2;
                        if (!hex4(&lo)) return false;
                        if (lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return fail("lone surrogate");
                    }
                    put_utf8(o, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        return fail("unterminated string");
    }
    bool number(Json* out) {
        const size_t b = pos_;
        if (pos_ < n_ && s_[pos_] == '-') ++pos_;
        if (pos_ >= n_ || s_[pos_] < '0' || s_[pos_] > '9') return fail("invalid value");
        if (s_[pos_] == '0') ++pos_;
        else while (pos_ < n_ && s_[pos_] >= '0' && s_[pos_] <= '9') ++pos_;
        bool integral = true;
        if (pos_ < n_ && s_[pos_] == '.') {
            integral = false;
            ++pos_;
            if (pos_ >= n_ || s_[pos_] < '0' || s_[pos_] > '9') return fail("bad fraction");
            while (pos_ < n_ && s_[pos_] >= '0' && s_[pos_] <= '9') ++pos_;
        }
        if (pos_ < n_ && (s_[pos_] == 'e' || s_[pos_] == 'E')) {
            integral = false;
            ++pos_;
            if (pos_ < n_ && (s_[pos_] == '+' || s_[pos_] == '-')) ++pos_;
            if (pos_ >= n_ || s_[pos_] < '0' || s_[pos_] > '9') return fail("bad exponent");
            while (pos_ < n_ && s_[pos_] >= '0' && s_[pos_] <= '9') ++pos_;
        }
        const std::string text(s_ + b, pos_ - b);
        out->kind = Json::Number;
        out->num = std::strtod(text.c_str(), nullptr);
        out->is_int = false;
        if (integral && text.size() < 20) {
            out->is_int = true;
            out->i64 = std::strtoll(text.c_str(), nullptr, 10);
        }
        return true;
    }
};

}  // namespace vox
