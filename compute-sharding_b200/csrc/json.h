// json.h — the small JSON reader and writer of the host side: packed-stage indexes, GGUF shard
// manifests and runtime bundles (the reference writes them with serde_json, crates/stage-forward-lab/
// src/gguf.rs:636-751 and lib.rs:3512-3613).
//
// The writer reproduces serde_json's pretty printer (two-space indent, `"key": value`, one array
// element per line, `[]` / `{}` when empty, no trailing newline) so that files written here are
// byte-identical to the reference's for the same content.
#pragma once

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <utility>
#include <vector>

namespace sfc {

struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json *get(const char *k) const {
    for (auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

inline void utf8_append(std::string &out, uint32_t cp) {
  if (cp < 0x80) {
    out += char(cp);
  } else if (cp < 0x800) {
    out += char(0xC0 | (cp >> 6));
    out += char(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += char(0xE0 | (cp >> 12));
    out += char(0x80 | ((cp >> 6) & 0x3F));
    out += char(0x80 | (cp & 0x3F));
  } else {
    out += char(0xF0 | (cp >> 18));
    out += char(0x80 | ((cp >> 12) & 0x3F));
    out += char(0x80 | ((cp >> 6) & 0x3F));
    out += char(0x80 | (cp & 0x3F));
  }
}

struct JsonParser {
  const char *p, *e;  // the text must be followed by a NUL (std::string storage is)
  bool ok = true;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(const char *s) {
    size_t n = strlen(s);
    if (size_t(e - p) >= n && !memcmp(p, s, n)) {
      p += n;
      return true;
    }
    return false;
  }
  bool hex4(uint32_t &v) {
    if (e - p < 4) return false;
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = p[i];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
      else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
      else return false;
    }
    p += 4;
    return true;
  }
  std::string string() {
    std::string out;
    ++p;  // opening quote
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) {
        ++p;
        const char c = *p++;
        switch (c) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            uint32_t v = 0;
            if (!hex4(v)) {
              ok = false;
              return out;
            }
            if (v >= 0xD800 && v < 0xDC00) {  // surrogate pair
              uint32_t lo = 0;
              if (e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                p += 2;
                if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) {
                  ok = false;
                  return out;
                }
                v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
              } else {
                ok = false;
                return out;
              }
            }
            utf8_append(out, v);
            break;
          }
          default: out += c;  // '"', '\\', '/'
        }
      } else {
        out += *p++;
      }
    }
    if (p >= e) ok = false;
    ++p;
    return out;
  }
  Json value() {
    Json j;
    ws();
    if (p >= e) {
      ok = false;
      return j;
    }
    if (*p == '{') {
      j.kind = Json::Obj;
      ++p;
      ws();
      if (p < e && *p == '}') {
        ++p;
        return j;
      }
      while (ok) {
        ws();
        if (p >= e || *p != '"') {
          ok = false;
          break;
        }
        std::string k = string();
        ws();
        if (p >= e || *p != ':') {
          ok = false;
          break;
        }
        ++p;
        j.obj.emplace_back(k, value());
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == '}') {
          ++p;
          break;
        }
        ok = false;
      }
    } else if (*p == '[') {
      j.kind = Json::Arr;
      ++p;
      ws();
      if (p < e && *p == ']') {
        ++p;
        return j;
      }
      while (ok) {
        j.arr.push_back(value());
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        if (p < e && *p == ']') {
          ++p;
          break;
        }
        ok = false;
      }
    } else if (*p == '"') {
      j.kind = Json::Str;
      j.str = string();
    } else if (lit("true")) {
      j.kind = Json::Bool;
      j.b = true;
    } else if (lit("false")) {
      j.kind = Json::Bool;
    } else if (lit("null")) {
      j.kind = Json::Null;
    } else {
      char *end = nullptr;
      j.num = strtod(p, &end);
      if (end == p) ok = false;
      j.kind = Json::Num;
      p = end;
    }
    return j;
  }
};

// Parses a whole document (trailing whitespace allowed).
inline bool json_parse(const std::string &text, Json &out) {
  JsonParser jp{text.data(), text.data() + text.size()};
  out = jp.value();
  jp.ws();
  return jp.ok && jp.p == jp.e;
}

inline bool read_file(const std::string &path, std::string &out) {
  FILE *f = fopen(path.c_str(), "rb");
  if (!f) return false;
  if (fseek(f, 0, SEEK_END) != 0) {
    fclose(f);
    return false;
  }
  const long n = ftell(f);
  if (n < 0 || fseek(f, 0, SEEK_SET) != 0) {
    fclose(f);
    return false;
  }
  out.resize(size_t(n));
  const size_t got = n > 0 ? fread(&out[0], 1, size_t(n), f) : 0;
  fclose(f);
  return got == size_t(n);
}

inline bool write_file(const std::string &path, const std::string &bytes) {
  FILE *f = fopen(path.c_str(), "wb");
  if (!f) return false;
  const size_t put = bytes.empty() ? 0 : fwrite(bytes.data(), 1, bytes.size(), f);
  const bool ok = put == bytes.size();
  return fclose(f) == 0 && ok;
}

// serde_json's string escaping: quote, backslash and control characters; everything else
// (including non-ASCII UTF-8) as is.
inline void json_escape(std::string &out, const std::string &s) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          snprintf(buf, sizeof(buf), "\\u%04x", unsigned(c));
          out += buf;
        } else {
          out += char(c);
        }
    }
  }
  out += '"';
}

// Pretty writer in serde_json's layout.  Usage: begin_obj(); key("a"); num(1); ... end_obj().
class JsonWriter {
 public:
  std::string out;
  void begin_obj() { open('{'); }
  void end_obj() { close('}'); }
  void begin_arr() { open('['); }
  void end_arr() { close(']'); }
  void key(const char *k) {
    item();
    json_escape(out, k);
    out += ": ";
    after_key_ = true;
  }
  void str(const std::string &s) {
    item();
    json_escape(out, s);
  }
  void num(uint64_t v) {
    item();
    out += std::to_string(v);
  }
  void null() {
    item();
    out += "null";
  }
  void str_array(const std::vector<std::string> &v) {
    begin_arr();
    for (auto &s : v) str(s);
    end_arr();
  }
  void num_array(const std::vector<uint64_t> &v) {
    begin_arr();
    for (auto x : v) num(x);
    end_arr();
  }

 private:
  std::vector<int> count_;  // elements written so far in each open container
  bool after_key_ = false;
  void indent() {
    out += '\n';
    out.append(2 * count_.size(), ' ');
  }
  void item() {  // position for a value or a key
    if (after_key_) {
      after_key_ = false;
      return;
    }
    if (count_.empty()) return;
    if (count_.back()++ > 0) out += ',';
    indent();
  }
  void open(char c) {
    item();
    out += c;
    count_.push_back(0);
  }
  void close(char c) {
    const int n = count_.back();
    count_.pop_back();
    if (n > 0) indent();
    out += c;
  }
};

}  // namespace sfc
