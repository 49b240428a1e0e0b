// json.h -- a strict JSON reader (RFC 8259) for headers and configuration files (internal): UTF-8 validated up
// front by the caller, \u escapes decoded to UTF-8 and required to form valid Unicode, objects kept in file order
// (duplicates are the caller's to refuse), numbers kept as their literal text, nesting depth bounded.
#pragma once

#include <stdint.h>
#include <string.h>

#include <string>
#include <utility>
#include <vector>

namespace lrm {
namespace json {

struct Error {
    std::string msg;
};

// Strict UTF-8: well-formed sequences of 1-4 bytes, shortest form, no surrogates, at most U+10FFFF.
inline bool valid_utf8(const uint8_t *p, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = p[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int len;
        uint32_t cp;
        if (c >= 0xC2 && c <= 0xDF) {
            len = 2;
            cp = c & 0x1F;
        } else if (c >= 0xE0 && c <= 0xEF) {
            len = 3;
            cp = c & 0x0F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            len = 4;
            cp = c & 0x07;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (int k = 1; k < len; ++k) {
            if ((p[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + k] & 0x3F);
        }
        if ((len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF) return false;
        if (cp >= 0xD800 && cp <= 0xDFFF) return false;
        i += len;
    }
    return true;
}

inline void put_utf8(std::string &s, uint32_t cp) {
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xC0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
        s += (char)(0xE0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    } else {
        s += (char)(0xF0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3F));
        s += (char)(0x80 | ((cp >> 6) & 0x3F));
        s += (char)(0x80 | (cp & 0x3F));
    }
}

// A JSON value of the header: objects keep their members in file order.
struct JValue {
    enum Kind { OBJECT, ARRAY, STRING, NUMBER, LITERAL } kind = LITERAL;
    std::string text;  // STRING: decoded UTF-8; NUMBER: the literal; LITERAL: true / false / null
    std::vector<std::pair<std::string, JValue>> members;
    std::vector<JValue> items;
};

class Parser {
  public:
    Parser(const uint8_t *p, size_t n, int max_depth = 8) : p_(p), end_(p + n), max_depth_(max_depth) {}

    JValue document() {
        JValue v = value(1);
        ws();
        if (p_ != end_) bad("content after the root value");
        return v;
    }

  private:
    const uint8_t *p_, *end_;
    int max_depth_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    [[noreturn]] void bad(const char *what) { throw Error{std::string("not valid JSON: ") + what}; }

    JValue value(int depth) {
        if (depth > max_depth_) bad("nesting too deep");
        ws();
        if (p_ == end_) bad("unexpected end");
        JValue v;
        const uint8_t c = *p_;
        if (c == '{') {
            v.kind = JValue::OBJECT;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return v;
            }
            for (;;) {
                ws();
                if (p_ == end_ || *p_ != '"') bad("expected a member name");
                std::string key = string_body();
                ws();
                if (p_ == end_ || *p_ != ':') bad("expected ':'");
                ++p_;
                v.members.emplace_back(std::move(key), value(depth + 1));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return v;
                }
                bad("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = JValue::ARRAY;
            ++p_;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return v;
            }
            for (;;) {
                v.items.push_back(value(depth + 1));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return v;
                }
                bad("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = JValue::STRING;
            v.text = string_body();
            return v;
        }
        if (c == '-' || (c >= '0' && c <= '9')) {
            v.kind = JValue::NUMBER;
            const uint8_t *s = p_;
            if (*p_ == '-') ++p_;
            if (p_ == end_ || !(*p_ >= '0' && *p_ <= '9')) bad("bad number");
            if (*p_ == '0') {
                ++p_;
            } else {
                while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
            }
            if (p_ < end_ && *p_ == '.') {
                ++p_;
                if (p_ == end_ || !(*p_ >= '0' && *p_ <= '9')) bad("bad number");
                while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
            }
            if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
                ++p_;
                if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
                if (p_ == end_ || !(*p_ >= '0' && *p_ <= '9')) bad("bad number");
                while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
            }
            v.text.assign((const char *)s, (size_t)(p_ - s));
            return v;
        }
        for (const char *lit : {"true", "false", "null"}) {
            const size_t n = strlen(lit);
            if ((size_t)(end_ - p_) >= n && memcmp(p_, lit, n) == 0) {
                p_ += n;
                v.kind = JValue::LITERAL;
                v.text = lit;
                return v;
            }
        }
        bad("unexpected character");
    }

    uint32_t hex4() {
        if (end_ - p_ < 4) bad("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const uint8_t c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9')
                v |= c - '0';
            else if (c >= 'a' && c <= 'f')
                v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F')
                v |= c - 'A' + 10;
            else
                bad("bad \\u escape");
        }
        return v;
    }

    // After the opening quote: the decoded string (escapes resolved; the raw bytes were checked as UTF-8 already).
    std::string string_body() {
        ++p_;  // the quote
        std::string s;
        for (;;) {
            if (p_ == end_) bad("unterminated string");
            const uint8_t c = *p_++;
            if (c == '"') return s;
            if (c < 0x20) bad("control character in a string");
            if (c != '\\') {
                s += (char)c;
                continue;
            }
            if (p_ == end_) bad("unterminated escape");
            const uint8_t e = *p_++;
            switch (e) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xDC00 && cp <= 0xDFFF) bad("a lone low surrogate");
                    if (cp >= 0xD800 && cp <= 0xDBFF) {
                        if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') bad("a high surrogate without its low half");
                        p_ += 2;
                        const uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo > 0xDFFF) bad("a high surrogate without its low half");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(s, cp);
                    break;
                }
                default: bad("unknown escape");
            }
        }
    }
};

}  // namespace json
}  // namespace lrm
