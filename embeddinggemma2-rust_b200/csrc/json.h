// Minimal JSON reader for config.json and safetensors headers: objects, arrays, strings (with the
// standard escapes), numbers, true / false / null. Parse errors throw std::runtime_error.
#pragma once
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace eg2 {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string& k) const { return kind == Obj && obj.count(k); }
    const Json& at(const std::string& k) const {
        auto it = obj.find(k);
        if (kind != Obj || it == obj.end()) throw std::runtime_error("missing key `" + k + "`");
        return it->second;
    }
    double number() const {
        if (kind != Num) throw std::runtime_error("expected a number");
        return num;
    }
    long integer() const { return (long)number(); }
    const std::string& string() const {
        if (kind != Str) throw std::runtime_error("expected a string");
        return str;
    }

    static Json parse(const char* p, size_t n) {
        size_t i = 0;
        Json j = value(p, n, i);
        ws(p, n, i);
        if (i != n) throw std::runtime_error("trailing characters in JSON");
        return j;
    }

   private:
    static void ws(const char* p, size_t n, size_t& i) {
        while (i < n && (p[i] == ' ' || p[i] == '\n' || p[i] == '\r' || p[i] == '\t')) i++;
    }
    static void expect(const char* p, size_t n, size_t& i, char c) {
        ws(p, n, i);
        if (i >= n || p[i] != c) throw std::runtime_error(std::string("JSON: expected '") + c + "'");
        i++;
    }
    static std::string parse_str(const char* p, size_t n, size_t& i) {
        expect(p, n, i, '"');
        std::string s;
        while (i < n && p[i] != '"') {
            char c = p[i++];
            if (c == '\\') {
                if (i >= n) break;
                char e = p[i++];
                switch (e) {
                    case 'n': s += '\n'; break;
                    case 't': s += '\t'; break;
                    case 'r': s += '\r'; break;
                    case 'b': s += '\b'; break;
                    case 'f': s += '\f'; break;
                    case 'u': {
                        if (i + 4 > n) throw std::runtime_error("JSON: bad \\u escape");
                        unsigned cp = (unsigned)strtoul(std::string(p + i, 4).c_str(), nullptr, 16);
                        i += 4;
                        if (cp < 0x80) s += (char)cp;
                        else if (cp < 0x800) { s += (char)(0xC0 | (cp >> 6)); s += (char)(0x80 | (cp & 0x3F)); }
                        else { s += (char)(0xE0 | (cp >> 12)); s += (char)(0x80 | ((cp >> 6) & 0x3F)); s += (char)(0x80 | (cp & 0x3F)); }
                        break;
                    }
                    default: s += e;
                }
            } else {
                s += c;
            }
        }
        if (i >= n) throw std::runtime_error("JSON: unterminated string");
        i++;
        return s;
    }
    static Json value(const char* p, size_t n, size_t& i) {
        ws(p, n, i);
        if (i >= n) throw std::runtime_error("JSON: unexpected end");
        Json j;
        char c = p[i];
        if (c == '{') {
            j.kind = Obj;
            i++;
            ws(p, n, i);
            if (i < n && p[i] == '}') { i++; return j; }
            while (true) {
                std::string k = parse_str(p, n, i);
                expect(p, n, i, ':');
                j.obj[k] = value(p, n, i);
                ws(p, n, i);
                if (i < n && p[i] == ',') { i++; continue; }
                expect(p, n, i, '}');
                return j;
            }
        }
        if (c == '[') {
            j.kind = Arr;
            i++;
            ws(p, n, i);
            if (i < n && p[i] == ']') { i++; return j; }
            while (true) {
                j.arr.push_back(value(p, n, i));
                ws(p, n, i);
                if (i < n && p[i] == ',') { i++; continue; }
                expect(p, n, i, ']');
                return j;
            }
        }
        if (c == '"') {
            j.kind = Str;
            j.str = parse_str(p, n, i);
            return j;
        }
        if (n - i >= 4 && std::string(p + i, 4) == "true") { j.kind = Bool; j.b = true; i += 4; return j; }
        if (n - i >= 5 && std::string(p + i, 5) == "false") { j.kind = Bool; i += 5; return j; }
        if (n - i >= 4 && std::string(p + i, 4) == "null") { i += 4; return j; }
        size_t st = i;
        while (i < n && (isdigit((unsigned char)p[i]) || p[i] == '-' || p[i] == '+' || p[i] == '.' || p[i] == 'e' || p[i] == 'E')) i++;
        if (st == i) throw std::runtime_error("JSON: unexpected character");
        j.kind = Num;
        j.num = strtod(std::string(p + st, i - st).c_str(), nullptr);
        return j;
    }
};

}  // namespace eg2
