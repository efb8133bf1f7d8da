// A small JSON reader for manifest.json (objects, arrays, strings, numbers,
// booleans, null).  Numbers are kept as double; the manifest's integers (offsets,
// sizes) stay exact up to 2^53 bytes.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace webyiq {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string& key) const { return kind == Object && obj.count(key) != 0; }
    // Member `key` of an object, or a Null value.
    const Json& operator[](const std::string& key) const;
    const Json& operator[](size_t i) const { return arr.at(i); }
    size_t size() const { return kind == Array ? arr.size() : kind == Object ? obj.size() : 0; }
};

// Parses `text`; on failure returns false and sets `err` (with the byte offset).
bool parse_json(const std::string& text, Json& out, std::string& err);

}  // namespace webyiq
