// toml.h -- the TOML subset the reference's scenario manifests and engine config use
// (rust/npu-engine/src/config.rs, rust/npu-runtime/src/config.rs:6-24): `[table]` and
// `[[array]]` headers, `key = value` lines with strings (basic escapes), integers, floats and
// booleans, `#` comments outside strings.  Keys are flattened to "table.key"; the i-th entry of
// an array of tables is the table "array[i]".
#pragma once

#include <cstdlib>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>

namespace xdna {

struct Toml {
    std::map<std::string, std::string> kv;   // "table.key" -> value (strings unquoted)
    std::map<std::string, bool> is_str;
    std::map<std::string, int> arrays;       // array-of-tables name -> entries

    static std::string trim(const std::string &s) {
        size_t a = s.find_first_not_of(" \t\r"), b = s.find_last_not_of(" \t\r");
        return a == std::string::npos ? "" : s.substr(a, b - a + 1);
    }
    // parse; returns "" or an error message
    std::string parse(const std::string &text) {
        std::istringstream in(text);
        std::string line, table;
        int ln = 0;
        while (std::getline(in, line)) {
            ln++;
            // strip a comment that is not inside a string
            bool q = false;
            for (size_t i = 0; i < line.size(); i++) {
                if (line[i] == '"' && (i == 0 || line[i - 1] != '\\')) q = !q;
                if (line[i] == '#' && !q) { line.resize(i); break; }
            }
            line = trim(line);
            if (line.empty()) continue;
            if (line[0] == '[') {
                if (line.size() >= 5 && line[1] == '[' && line.compare(line.size() - 2, 2, "]]") == 0) {
                    const std::string name = trim(line.substr(2, line.size() - 4));
                    if (name.empty()) return "line " + std::to_string(ln) + ": empty table name";
                    table = name + "[" + std::to_string(arrays[name]++) + "]";
                    continue;
                }
                if (line.back() != ']' || line.size() < 3 || line[1] == '[')
                    return "line " + std::to_string(ln) + ": unsupported table header";
                table = trim(line.substr(1, line.size() - 2));
                continue;
            }
            const size_t eq = line.find('=');
            if (eq == std::string::npos) return "line " + std::to_string(ln) + ": expected key = value";
            const std::string key = trim(line.substr(0, eq));
            std::string val = trim(line.substr(eq + 1));
            const std::string full = table.empty() ? key : table + "." + key;
            if (!val.empty() && val[0] == '"') {
                std::string out;
                size_t i = 1;
                for (; i < val.size() && val[i] != '"'; i++) {
                    if (val[i] == '\\' && i + 1 < val.size()) {
                        const char e = val[++i];
                        out += e == 'n' ? '\n' : e == 't' ? '\t' : e;
                    } else {
                        out += val[i];
                    }
                }
                if (i >= val.size()) return "line " + std::to_string(ln) + ": unterminated string";
                kv[full] = out;
                is_str[full] = true;
            } else {
                kv[full] = val;
                is_str[full] = false;
            }
        }
        return "";
    }
    bool has(const std::string &k) const { return kv.count(k) != 0; }
    int count(const std::string &array) const {
        auto it = arrays.find(array);
        return it == arrays.end() ? 0 : it->second;
    }
    // true if any key of `table` is present
    bool has_table(const std::string &table) const {
        auto it = kv.lower_bound(table + ".");
        return it != kv.end() && it->first.compare(0, table.size() + 1, table + ".") == 0;
    }
    std::string str(const std::string &k, const std::string &dflt = "") const {
        auto it = kv.find(k);
        return it == kv.end() ? dflt : it->second;
    }
    // a required string field (serde's messages: missing field / invalid type)
    std::string req_str(const std::string &k) const {
        auto it = kv.find(k);
        if (it == kv.end()) throw std::runtime_error("missing field `" + k.substr(k.rfind('.') + 1) + "`");
        if (!is_str.at(k)) throw std::runtime_error("invalid type for `" + k + "`: expected a string");
        return it->second;
    }
    long integer(const std::string &k) const {
        auto it = kv.find(k);
        if (it == kv.end()) throw std::runtime_error("missing field `" + k.substr(k.rfind('.') + 1) + "`");
        char *end = nullptr;
        const long v = std::strtol(it->second.c_str(), &end, 10);
        if (is_str.at(k) || !end || *end) throw std::runtime_error("invalid type for `" + k + "`: expected an integer");
        return v;
    }
    bool boolean(const std::string &k, bool dflt) const {
        auto it = kv.find(k);
        if (it == kv.end()) return dflt;
        if (it->second == "true") return true;
        if (it->second == "false") return false;
        throw std::runtime_error("invalid type for `" + k + "`: expected a boolean");
    }
};

}  // namespace xdna
