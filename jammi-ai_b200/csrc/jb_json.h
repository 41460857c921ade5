// Minimal JSON reader for HF config.json, open_clip_config.json and the
// safetensors header.  Numbers are kept as double; no streaming.
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace jb {

struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  const Json* get(const std::string& k) const {
    if (kind != Obj) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
  double num_or(const std::string& k, double d) const {
    const Json* j = get(k);
    return (j && j->kind == Num) ? j->num : d;
  }
  bool bool_or(const std::string& k, bool d) const {
    const Json* j = get(k);
    return (j && j->kind == Bool) ? j->b : d;
  }
  std::string str_or(const std::string& k, const std::string& d) const {
    const Json* j = get(k);
    return (j && j->kind == Str) ? j->str : d;
  }

  static Json parse(const std::string& text) {
    size_t i = 0;
    Json j = parse_value(text, i);
    skip_ws(text, i);
    if (i != text.size()) throw std::runtime_error("json: trailing characters");
    return j;
  }

 private:
  static void skip_ws(const std::string& s, size_t& i) {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  static void expect(const std::string& s, size_t& i, char c) {
    skip_ws(s, i);
    if (i >= s.size() || s[i] != c) throw std::runtime_error(std::string("json: expected '") + c + "'");
    ++i;
  }
  static std::string parse_string(const std::string& s, size_t& i) {
    expect(s, i, '"');
    std::string out;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) break;
        char e = s[i++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i + 4 > s.size()) throw std::runtime_error("json: bad \\u escape");
            unsigned cp = std::stoul(s.substr(i, 4), nullptr, 16);
            i += 4;
            if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
              const unsigned lo = std::stoul(s.substr(i + 2, 4), nullptr, 16);
              if (lo >= 0xDC00 && lo < 0xE000) {  // surrogate pair
                cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                i += 6;
              }
            }
            if (cp < 0x80) {
              out += static_cast<char>(cp);
            } else if (cp < 0x800) {
              out += static_cast<char>(0xC0 | (cp >> 6));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            } else if (cp < 0x10000) {
              out += static_cast<char>(0xE0 | (cp >> 12));
              out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            } else {
              out += static_cast<char>(0xF0 | (cp >> 18));
              out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
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
    if (i >= s.size()) throw std::runtime_error("json: unterminated string");
    ++i;
    return out;
  }
  static Json parse_value(const std::string& s, size_t& i) {
    skip_ws(s, i);
    if (i >= s.size()) throw std::runtime_error("json: unexpected end");
    Json j;
    const char c = s[i];
    if (c == '{') {
      j.kind = Obj;
      ++i;
      skip_ws(s, i);
      if (i < s.size() && s[i] == '}') { ++i; return j; }
      while (true) {
        std::string k = parse_string(s, i);
        expect(s, i, ':');
        j.obj[k] = parse_value(s, i);
        skip_ws(s, i);
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        expect(s, i, '}');
        return j;
      }
    }
    if (c == '[') {
      j.kind = Arr;
      ++i;
      skip_ws(s, i);
      if (i < s.size() && s[i] == ']') { ++i; return j; }
      while (true) {
        j.arr.push_back(parse_value(s, i));
        skip_ws(s, i);
        if (i < s.size() && s[i] == ',') { ++i; continue; }
        expect(s, i, ']');
        return j;
      }
    }
    if (c == '"') {
      j.kind = Str;
      j.str = parse_string(s, i);
      return j;
    }
    if (s.compare(i, 4, "true") == 0) { j.kind = Bool; j.b = true; i += 4; return j; }
    if (s.compare(i, 5, "false") == 0) { j.kind = Bool; j.b = false; i += 5; return j; }
    if (s.compare(i, 4, "null") == 0) { i += 4; return j; }
    const char* start = s.c_str() + i;
    char* end = nullptr;
    j.num = std::strtod(start, &end);
    if (end == start) throw std::runtime_error("json: bad value");
    j.kind = Num;
    i += static_cast<size_t>(end - start);
    return j;
  }
};

}  // namespace jb
