#include "json.hpp"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>

namespace dtj {

namespace {

struct Parser {
  const char* p;
  const char* e;
  [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("json: ") + what); }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(e - p) >= n && memcmp(p, s, n) == 0) { p += n; return true; }
    return false;
  }
  static void put_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) out += (char)cp;
    else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) {
      out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
    } else {
      out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 0x3F));
      out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (e - p < 4) fail("bad \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad hex");
    }
    return v;
  }
  std::string str() {
    if (p >= e || *p != '"') fail("expected string");
    ++p;
    std::string out;
    while (true) {
      if (p >= e) fail("unterminated string");
      char c = *p++;
      if (c == '"') break;
      if (c != '\\') { out += c; continue; }
      if (p >= e) fail("bad escape");
      char x = *p++;
      switch (x) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            uint32_t lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  Value num() {
    const char* s = p;
    bool is_int = true;
    if (p < e && (*p == '-' || *p == '+')) ++p;
    while (p < e && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) {
      if (*p == '.' || *p == 'e' || *p == 'E') is_int = false;
      ++p;
    }
    std::string t(s, p - s);
    if (t.empty()) fail("bad number");
    if (is_int) {
      errno = 0;
      char* end = nullptr;
      long long v = strtoll(t.c_str(), &end, 10);
      if (errno == 0 && end && *end == 0) return Value::integer(v);
      unsigned long long u = strtoull(t.c_str(), &end, 10);
      if (end && *end == 0) return Value::integer((int64_t)u);
    }
    return Value::number(strtod(t.c_str(), nullptr));
  }
  Value val(int depth) {
    if (depth > 256) fail("too deep");
    ws();
    if (p >= e) fail("unexpected end");
    char c = *p;
    if (c == '{') {
      ++p;
      Value v = Value::object();
      ws();
      if (p < e && *p == '}') { ++p; return v; }
      while (true) {
        ws();
        std::string k = str();
        ws();
        if (p >= e || *p != ':') fail("expected :");
        ++p;
        v.o->emplace_back(std::move(k), val(depth + 1));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; break; }
        fail("expected , or }");
      }
      return v;
    }
    if (c == '[') {
      ++p;
      Value v = Value::array();
      ws();
      if (p < e && *p == ']') { ++p; return v; }
      while (true) {
        v.a->push_back(val(depth + 1));
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; break; }
        fail("expected , or ]");
      }
      return v;
    }
    if (c == '"') return Value::string(str());
    if (lit("true")) return Value::boolean(true);
    if (lit("false")) return Value::boolean(false);
    if (lit("null")) return Value::null();
    return num();
  }
};

}  // namespace

Value parse(const char* p, size_t n) {
  Parser ps{p, p + n};
  Value v = ps.val(0);
  ps.ws();
  if (ps.p != ps.e) throw std::runtime_error("json: trailing data");
  return v;
}

void dump_string(const std::string& s, std::string& out) {
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
          snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;
        }
    }
  }
  out += '"';
}

// Shortest representation that round-trips through strtod (17 significant digits worst case),
// printed like serde_json: integral finite values keep a ".0".
void dump_double(double d, std::string& out) {
  if (!std::isfinite(d)) { out += "null"; return; }
  char buf[40];
  for (int prec = 1; prec <= 17; ++prec) {
    snprintf(buf, sizeof buf, "%.*g", prec, d);
    if (strtod(buf, nullptr) == d) break;
  }
  std::string t(buf);
  if (t.find_first_of(".eEn") == std::string::npos) t += ".0";
  out += t;
}

void dump(const Value& v, std::string& out) {
  switch (v.kind) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Int: out += std::to_string(v.i); break;
    case Value::Double: dump_double(v.d, out); break;
    case Value::String: dump_string(v.s, out); break;
    case Value::Arr: {
      out += '[';
      bool first = true;
      for (auto& x : *v.a) {
        if (!first) out += ',';
        first = false;
        dump(x, out);
      }
      out += ']';
      break;
    }
    case Value::Obj: {
      out += '{';
      bool first = true;
      for (auto& kv : *v.o) {
        if (!first) out += ',';
        first = false;
        dump_string(kv.first, out);
        out += ':';
        dump(kv.second, out);
      }
      out += '}';
      break;
    }
  }
}

}  // namespace dtj
