// json.h -- a small JSON reader for the host side (safetensors headers, tokenizer.json):
// objects, arrays, strings with \u escapes (surrogate pairs joined), numbers, true / false /
// null.  Errors throw std::runtime_error with the given context prefix.
#pragma once
#include <cstdint>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace xdna {
namespace json {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;
};

struct JsonParser {
    const char *p, *end;
    const char *context = "JSON";
    [[noreturn]] void fail(const char *what) { throw std::runtime_error(std::string(context) + ": " + what); }
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
    }
    void put_utf8(std::string &o, uint32_t cp) {
        if (cp < 0x80) o += (char)cp;
        else if (cp < 0x800) { o += (char)(0xc0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3f)); }
        else if (cp < 0x10000) {
            o += (char)(0xe0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
        } else {
            o += (char)(0xf0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3f));
            o += (char)(0x80 | ((cp >> 6) & 0x3f)); o += (char)(0x80 | (cp & 0x3f));
        }
    }
    uint32_t hex4() {
        if (end - p < 4) fail("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; i++, p++) {
            const char c = *p;
            v = v * 16 + (c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                          : c >= 'A' && c <= 'F' ? c - 'A' + 10 : (fail("bad \\u escape"), 0));
        }
        return v;
    }
    std::string string() {
        if (p >= end || *p != '"') fail("expected a string");
        p++;
        std::string o;
        while (p < end && *p != '"') {
            if (*p != '\\') { o += *p++; continue; }
            if (++p >= end) fail("bad escape");
            const char c = *p++;
            switch (c) {
            case 'n': o += '\n'; break;
            case 't': o += '\t'; break;
            case 'r': o += '\r'; break;
            case 'b': o += '\b'; break;
            case 'f': o += '\f'; break;
            case 'u': {
                uint32_t cp = hex4();
                if (cp >= 0xd800 && cp < 0xdc00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                    p += 2;
                    cp = 0x10000 + ((cp - 0xd800) << 10) + (hex4() - 0xdc00);
                }
                put_utf8(o, cp);
                break;
            }
            default: o += c;
            }
        }
        if (p >= end) fail("unterminated string");
        p++;
        return o;
    }
    Json value(int depth = 0) {
        if (depth > 16) fail("nested too deeply");
        ws();
        if (p >= end) fail("unexpected end");
        Json j;
        if (*p == '{') {
            j.kind = Json::Obj;
            p++;
            ws();
            if (p < end && *p == '}') { p++; return j; }
            while (true) {
                ws();
                std::string k = string();
                ws();
                if (p >= end || *p != ':') fail("expected ':'");
                p++;
                j.obj[k] = value(depth + 1);
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == '}') { p++; return j; }
                fail("expected ',' or '}'");
            }
        }
        if (*p == '[') {
            j.kind = Json::Arr;
            p++;
            ws();
            if (p < end && *p == ']') { p++; return j; }
            while (true) {
                j.arr.push_back(value(depth + 1));
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == ']') { p++; return j; }
                fail("expected ',' or ']'");
            }
        }
        if (*p == '"') { j.kind = Json::Str; j.str = string(); return j; }
        if (end - p >= 4 && !std::strncmp(p, "true", 4)) { p += 4; j.kind = Json::Bool; j.b = true; return j; }
        if (end - p >= 5 && !std::strncmp(p, "false", 5)) { p += 5; j.kind = Json::Bool; return j; }
        if (end - p >= 4 && !std::strncmp(p, "null", 4)) { p += 4; return j; }
        const char *s = p;
        while (p < end && (std::strchr("+-.eE", *p) || (*p >= '0' && *p <= '9'))) p++;
        if (p == s) fail("unexpected character");
        j.kind = Json::Num;
        j.num = std::stod(std::string(s, p));
        return j;
    }
};


}  // namespace json
}  // namespace xdna
