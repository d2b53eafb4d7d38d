// A small JSON reader for HF-style config.json files (objects, arrays,
// numbers, strings, booleans, null). Enough for Config::from_json; not a
// general-purpose library.
#pragma once
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace omg {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool is_null() const { return kind == Null; }
  const Json& operator[](const std::string& k) const {
    static const Json null_json;
    if (kind != Object) return null_json;
    auto it = obj.find(k);
    return it == obj.end() ? null_json : it->second;
  }
  bool has(const std::string& k) const { return kind == Object && obj.count(k) > 0; }
  // as_u64 / as_f64 / as_str: present and of the right kind, else false.
  bool as_u64(uint64_t* out) const {
    if (kind != Number || num < 0 || num != static_cast<double>(static_cast<uint64_t>(num)))
      return false;
    *out = static_cast<uint64_t>(num);
    return true;
  }
  bool as_f64(double* out) const {
    if (kind != Number) return false;
    *out = num;
    return true;
  }
  const std::string* as_str() const { return kind == String ? &str : nullptr; }

  static Json parse(const std::string& text) {
    size_t i = 0;
    Json j = parse_value(text, i);
    skip_ws(text, i);
    if (i != text.size()) throw std::runtime_error("config.json: trailing characters");
    return j;
  }

 private:
  static void skip_ws(const std::string& s, size_t& i) {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  static void expect(const std::string& s, size_t& i, char c) {
    skip_ws(s, i);
    if (i >= s.size() || s[i] != c)
      throw std::runtime_error(std::string("config.json: expected '") + c + "'");
    ++i;
  }
  static std::string parse_string(const std::string& s, size_t& i) {
    expect(s, i, '"');
    std::string out;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\' && i < s.size()) {
        char e = s[i++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i + 4 > s.size()) throw std::runtime_error("config.json: bad escape");
            unsigned cp = std::stoul(s.substr(i, 4), nullptr, 16);
            i += 4;
            if (cp < 0x80) {
              out += static_cast<char>(cp);
            } else if (cp < 0x800) {
              out += static_cast<char>(0xC0 | (cp >> 6));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            } else {
              out += static_cast<char>(0xE0 | (cp >> 12));
              out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i >= s.size()) throw std::runtime_error("config.json: unterminated string");
    ++i;
    return out;
  }
  static Json parse_value(const std::string& s, size_t& i) {
    skip_ws(s, i);
    if (i >= s.size()) throw std::runtime_error("config.json: unexpected end");
    Json j;
    const char c = s[i];
    if (c == '{') {
      j.kind = Object;
      ++i;
      skip_ws(s, i);
      if (i < s.size() && s[i] == '}') {
        ++i;
        return j;
      }
      while (true) {
        std::string k = parse_string(s, i);
        expect(s, i, ':');
        j.obj[k] = parse_value(s, i);
        skip_ws(s, i);
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        expect(s, i, '}');
        return j;
      }
    }
    if (c == '[') {
      j.kind = Array;
      ++i;
      skip_ws(s, i);
      if (i < s.size() && s[i] == ']') {
        ++i;
        return j;
      }
      while (true) {
        j.arr.push_back(parse_value(s, i));
        skip_ws(s, i);
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        expect(s, i, ']');
        return j;
      }
    }
    if (c == '"') {
      j.kind = String;
      j.str = parse_string(s, i);
      return j;
    }
    if (s.compare(i, 4, "true") == 0) {
      i += 4;
      j.kind = Bool;
      j.b = true;
      return j;
    }
    if (s.compare(i, 5, "false") == 0) {
      i += 5;
      j.kind = Bool;
      return j;
    }
    if (s.compare(i, 4, "null") == 0) {
      i += 4;
      return j;
    }
    const char* start = s.c_str() + i;
    char* end = nullptr;
    j.num = std::strtod(start, &end);
    if (end == start) throw std::runtime_error("config.json: bad value");
    j.kind = Number;
    i += static_cast<size_t>(end - start);
    return j;
  }
};

}  // namespace omg
