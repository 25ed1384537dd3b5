// json.cuh - a small JSON reader for the files the library reads itself: the tuned-plan
// cache and safetensors checkpoint headers.  Objects keep their keys in file order;
// numbers are doubles (checkpoint offsets stay exact below 2^53); \u escapes (surrogate
// pairs included) become UTF-8.  Anything malformed fails the whole parse.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace bybycu {

struct JVal {
    enum Type { kNull, kNum, kStr, kObj, kArr, kBool } type = kNull;
    double num = 0;
    bool boolean = false;
    std::string str;
    std::vector<std::pair<std::string, JVal>> obj;
    std::vector<JVal> arr;
    const JVal* get(const char* k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

namespace json_detail {

struct Parser {
    const char* p;
    const char* end;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool hex4(uint32_t* v) {
        if (end - p < 4) return false;
        *v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p++;
            const int d = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                        : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
            if (d < 0) return false;
            *v = *v * 16 + static_cast<uint32_t>(d);
        }
        return true;
    }
    static void utf8(std::string* s, uint32_t cp) {
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
    bool str(std::string* s) {
        if (p >= end || *p != '"') return false;
        ++p;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) return false;
                const char e = *p++;
                switch (e) {
                    case 'n': c = '\n'; break;
                    case 't': c = '\t'; break;
                    case 'r': c = '\r'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'u': {
                        uint32_t cp;
                        if (!hex4(&cp)) return false;
                        if (cp >= 0xD800 && cp < 0xDC00) {   // a surrogate pair
                            uint32_t lo;
                            if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return false;
                            p += 2;
                            if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        }
                        utf8(s, cp);
                        continue;
                    }
                    case '"': case '\\': case '/': c = e; break;
                    default: return false;
                }
            }
            s->push_back(c);
        }
        if (p >= end) return false;
        ++p;
        return true;
    }
    bool value(JVal* v, int depth) {
        if (depth > 32) return false;
        ws();
        if (p >= end) return false;
        if (*p == '"') {
            v->type = JVal::kStr;
            return str(&v->str);
        }
        if (*p == '{' || *p == '[') {
            const bool is_obj = *p == '{';
            const char close = is_obj ? '}' : ']';
            v->type = is_obj ? JVal::kObj : JVal::kArr;
            ++p;
            ws();
            if (p < end && *p == close) { ++p; return true; }
            for (;;) {
                std::string k;
                if (is_obj) {
                    ws();
                    if (!str(&k)) return false;
                    ws();
                    if (p >= end || *p != ':') return false;
                    ++p;
                }
                JVal child;
                if (!value(&child, depth + 1)) return false;
                if (is_obj) v->obj.emplace_back(std::move(k), std::move(child));
                else v->arr.push_back(std::move(child));
                ws();
                if (p < end && *p == ',') { ++p; continue; }
                if (p < end && *p == close) { ++p; return true; }
                return false;
            }
        }
        if (*p == '-' || (*p >= '0' && *p <= '9')) {
            const std::string tok(p, static_cast<size_t>(std::min<ptrdiff_t>(end - p, 64)));
            char* q = nullptr;
            v->num = strtod(tok.c_str(), &q);
            if (q == tok.c_str()) return false;
            p += q - tok.c_str();
            v->type = JVal::kNum;
            return true;
        }
        static const struct { const char* lit; JVal::Type type; bool b; } lits[] = {
            {"true", JVal::kBool, true}, {"false", JVal::kBool, false}, {"null", JVal::kNull, false}};
        for (const auto& l : lits) {
            const size_t n = strlen(l.lit);
            if (static_cast<size_t>(end - p) >= n && !strncmp(p, l.lit, n)) {
                p += n;
                v->type = l.type;
                v->boolean = l.b;
                return true;
            }
        }
        return false;
    }
};

}  // namespace json_detail

// Parses the whole text as one JSON value (trailing whitespace allowed).
inline bool json_parse(const std::string& text, JVal* out) {
    json_detail::Parser jp{text.data(), text.data() + text.size()};
    if (!jp.value(out, 0)) return false;
    jp.ws();
    return jp.p == jp.end;
}

}  // namespace bybycu
