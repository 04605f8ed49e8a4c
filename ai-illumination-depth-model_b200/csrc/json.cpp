// A small strict JSON reader for container headers (objects keep key order,
// later duplicate keys win on lookup, as JSON.parse does).
#include <cmath>
#include <cstdlib>

#include "host.h"

namespace illumina {

const Json *Json::get(const std::string &k) const {
  if (type != Object) return nullptr;
  const Json *found = nullptr;
  for (const auto &kv : obj)
    if (kv.first == k) found = &kv.second;
  return found;
}

namespace {

struct Parser {
  const std::string &s;
  size_t i = 0;
  int depth = 0;
  explicit Parser(const std::string &t) : s(t) {}

  [[noreturn]] void fail(const std::string &what) {
    throw std::runtime_error(what + " at position " + std::to_string(i));
  }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) i++;
  }
  bool lit(const char *w) {
    size_t n = std::char_traits<char>::length(w);
    if (s.compare(i, n, w) == 0) {
      i += n;
      return true;
    }
    return false;
  }
  static void utf8(std::string &o, unsigned cp) {
    if (cp < 0x80) o += (char)cp;
    else if (cp < 0x800) o += (char)(0xc0 | (cp >> 6)), o += (char)(0x80 | (cp & 0x3f));
    else if (cp < 0x10000)
      o += (char)(0xe0 | (cp >> 12)), o += (char)(0x80 | ((cp >> 6) & 0x3f)), o += (char)(0x80 | (cp & 0x3f));
    else
      o += (char)(0xf0 | (cp >> 18)), o += (char)(0x80 | ((cp >> 12) & 0x3f)),
          o += (char)(0x80 | ((cp >> 6) & 0x3f)), o += (char)(0x80 | (cp & 0x3f));
  }
  unsigned hex4() {
    if (i + 4 > s.size()) fail("truncated \\u escape");
    unsigned v = 0;
    for (int k = 0; k < 4; k++) {
      char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string str() {
    if (s[i] != '"') fail("expected string");
    i++;
    std::string o;
    while (true) {
      if (i >= s.size()) fail("unterminated string");
      char c = s[i++];
      if (c == '"') break;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') {
        o += c;
        continue;
      }
      if (i >= s.size()) fail("unterminated escape");
      char e = s[i++];
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          unsigned cp = hex4();
          if (cp >= 0xd800 && cp < 0xdc00 && i + 1 < s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            i += 2;
            unsigned lo = hex4();
            cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
          }
          utf8(o, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return o;
  }
  Json value() {
    ws();
    if (i >= s.size()) fail("unexpected end of input");
    if (++depth > 256) fail("nesting too deep");
    Json j;
    char c = s[i];
    if (c == '{') {
      j.type = Json::Object;
      i++;
      ws();
      if (i < s.size() && s[i] == '}') {
        i++;
      } else {
        while (true) {
          ws();
          if (i >= s.size()) fail("unexpected end of input");
          std::string k = str();
          ws();
          if (i >= s.size() || s[i] != ':') fail("expected ':'");
          i++;
          j.obj.emplace_back(k, value());
          ws();
          if (i < s.size() && s[i] == ',') {
            i++;
            continue;
          }
          if (i < s.size() && s[i] == '}') {
            i++;
            break;
          }
          fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      j.type = Json::Array;
      i++;
      ws();
      if (i < s.size() && s[i] == ']') {
        i++;
      } else {
        while (true) {
          j.arr.push_back(value());
          ws();
          if (i < s.size() && s[i] == ',') {
            i++;
            continue;
          }
          if (i < s.size() && s[i] == ']') {
            i++;
            break;
          }
          fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      j.type = Json::String;
      j.str = str();
    } else if (lit("true")) {
      j.type = Json::Bool, j.b = true;
    } else if (lit("false")) {
      j.type = Json::Bool, j.b = false;
    } else if (lit("null")) {
      j.type = Json::Null;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      size_t st = i;
      if (s[i] == '-') i++;
      if (i >= s.size() || !(s[i] >= '0' && s[i] <= '9')) fail("bad number");
      if (s[i] == '0') i++;
      else
        while (i < s.size() && s[i] >= '0' && s[i] <= '9') i++;
      if (i < s.size() && s[i] == '.') {
        i++;
        if (i >= s.size() || !(s[i] >= '0' && s[i] <= '9')) fail("bad number");
        while (i < s.size() && s[i] >= '0' && s[i] <= '9') i++;
      }
      if (i < s.size() && (s[i] == 'e' || s[i] == 'E')) {
        i++;
        if (i < s.size() && (s[i] == '+' || s[i] == '-')) i++;
        if (i >= s.size() || !(s[i] >= '0' && s[i] <= '9')) fail("bad number");
        while (i < s.size() && s[i] >= '0' && s[i] <= '9') i++;
      }
      j.type = Json::Number;
      j.num = std::strtod(s.substr(st, i - st).c_str(), nullptr);
    } else {
      fail(std::string("unexpected token '") + c + "'");
    }
    depth--;
    return j;
  }
};

}  // namespace

Json parse_json(const std::string &text) {
  Parser p(text);
  Json j = p.value();
  p.ws();
  if (p.i != text.size()) p.fail("unexpected trailing data");
  return j;
}

}  // namespace illumina
