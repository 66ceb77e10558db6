// JSON parser / serializer and msgpack decoder (see json.h).
#include "json.h"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace ib {

const Value* Value::get(const std::string& key) const {
  if (t != Obj || !o) return nullptr;
  for (const auto& kv : *o)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

Value* Value::get_mut(const std::string& key) {
  if (t != Obj || !o) return nullptr;
  for (auto& kv : *o)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

void Value::set(const std::string& key, Value v) {
  if (t != Obj || !o) { t = Obj; o = std::make_shared<Object>(); }
  for (auto& kv : *o)
    if (kv.first == key) { kv.second = std::move(v); return; }
  o->emplace_back(key, std::move(v));
}

bool Value::erase(const std::string& key) {
  if (t != Obj || !o) return false;
  for (auto it = o->begin(); it != o->end(); ++it)
    if (it->first == key) { o->erase(it); return true; }
  return false;
}

// ---------------------------------------------------------------------------
// JSON parser: recursive descent over a bounded buffer, depth-limited.

namespace {

struct JsonParser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) s.push_back(static_cast<char>(cp));
    else if (cp < 0x800) {
      s.push_back(static_cast<char>(0xC0 | (cp >> 6)));
      s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      s.push_back(static_cast<char>(0xE0 | (cp >> 12)));
      s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      s.push_back(static_cast<char>(0xF0 | (cp >> 18)));
      s.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(uint32_t* out) {
    if (end - p < 4) return fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      char c = p[k];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return fail("bad \\u escape");
    }
    p += 4;
    *out = v;
    return true;
  }
  bool string(std::string* s) {
    ++p;  // opening quote
    while (p < end) {
      const char* q = p;
      while (q < end && *q != '"' && *q != '\\') ++q;
      s->append(p, q - p);
      p = q;
      if (p >= end) break;
      if (*p == '"') { ++p; return true; }
      ++p;  // backslash
      if (p >= end) break;
      char c = *p++;
      switch (c) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp <= 0xDBFF && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            uint32_t lo;
            if (!hex4(&lo)) return false;
            if (lo >= 0xDC00 && lo <= 0xDFFF) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            else { put_utf8(*s, cp); cp = lo; }
          }
          put_utf8(*s, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    return fail("unterminated string");
  }
  bool number(Value* v) {
    const char* q = p;
    bool neg = false, frac = false;
    if (q < end && *q == '-') { neg = true; ++q; }
    const char* digits = q;
    while (q < end && *q >= '0' && *q <= '9') ++q;
    if (q == digits) return fail("bad number");
    if (q < end && (*q == '.' || *q == 'e' || *q == 'E')) {
      frac = true;
      if (*q == '.') { ++q; while (q < end && *q >= '0' && *q <= '9') ++q; }
      if (q < end && (*q == 'e' || *q == 'E')) {
        ++q;
        if (q < end && (*q == '+' || *q == '-')) ++q;
        while (q < end && *q >= '0' && *q <= '9') ++q;
      }
    }
    std::string tok(p, q - p);
    p = q;
    if (!frac) {
      errno = 0;
      if (neg) {
        long long x = std::strtoll(tok.c_str(), nullptr, 10);
        if (errno == 0) { *v = Value::integer(x); return true; }
      } else {
        unsigned long long x = std::strtoull(tok.c_str(), nullptr, 10);
        if (errno == 0) { *v = Value::uinteger(x); return true; }
      }
    }
    *v = Value::number(std::strtod(tok.c_str(), nullptr));
    return true;
  }
  bool lit(const char* w, size_t n) {
    if (static_cast<size_t>(end - p) < n || std::memcmp(p, w, n) != 0) return fail("bad literal");
    p += n;
    return true;
  }
  bool value(Value* v) {
    ws();
    if (p >= end) return fail("unexpected end");
    if (++depth > 256) return fail("nesting too deep");
    bool ok = true;
    switch (*p) {
      case '{': {
        ++p;
        *v = Value::object();
        ws();
        if (p < end && *p == '}') { ++p; break; }
        while (true) {
          ws();
          if (p >= end || *p != '"') { ok = fail("expected key"); break; }
          std::string k;
          if (!string(&k)) { ok = false; break; }
          ws();
          if (p >= end || *p != ':') { ok = fail("expected ':'"); break; }
          ++p;
          Value x;
          if (!value(&x)) { ok = false; break; }
          v->o->emplace_back(std::move(k), std::move(x));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          ok = fail("expected ',' or '}'");
          break;
        }
        break;
      }
      case '[': {
        ++p;
        *v = Value::array();
        ws();
        if (p < end && *p == ']') { ++p; break; }
        while (true) {
          Value x;
          if (!value(&x)) { ok = false; break; }
          v->a->push_back(std::move(x));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          ok = fail("expected ',' or ']'");
          break;
        }
        break;
      }
      case '"': {
        std::string s;
        ok = string(&s);
        if (ok) *v = Value::string(std::move(s));
        break;
      }
      case 't': ok = lit("true", 4); if (ok) *v = Value::boolean(true); break;
      case 'f': ok = lit("false", 5); if (ok) *v = Value::boolean(false); break;
      case 'n': ok = lit("null", 4); if (ok) *v = Value(); break;
      default: ok = number(v); break;
    }
    --depth;
    return ok;
  }
};

}  // namespace

bool parse_json(const char* p, size_t n, Value* out, std::string* err) {
  JsonParser jp{p, p + n, {}};
  if (!jp.value(out)) {
    if (err) *err = jp.err;
    return false;
  }
  jp.ws();
  if (jp.p != jp.end) {
    if (err) *err = "trailing characters";
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// JSON writer

void json_escape(const std::string& s, std::string& out) {
  out.push_back('"');
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
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out.push_back(static_cast<char>(c));
        }
    }
  }
  out.push_back('"');
}

void dump_json(const Value& v, std::string& out) {
  char buf[64];
  switch (v.t) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Int: std::snprintf(buf, sizeof(buf), "%lld", static_cast<long long>(v.i)); out += buf; break;
    case Value::UInt: std::snprintf(buf, sizeof(buf), "%llu", static_cast<unsigned long long>(v.u)); out += buf; break;
    case Value::Double:
      if (std::isfinite(v.d)) {
        std::snprintf(buf, sizeof(buf), "%.17g", v.d);
        out += buf;
      } else {
        out += "null";
      }
      break;
    case Value::String: case Value::Bin: json_escape(v.s, out); break;
    case Value::Arr: {
      out.push_back('[');
      bool first = true;
      for (const auto& x : v.arr()) {
        if (!first) out.push_back(',');
        first = false;
        dump_json(x, out);
      }
      out.push_back(']');
      break;
    }
    case Value::Obj: {
      out.push_back('{');
      bool first = true;
      for (const auto& kv : v.obj()) {
        if (!first) out.push_back(',');
        first = false;
        json_escape(kv.first, out);
        out.push_back(':');
        dump_json(kv.second, out);
      }
      out.push_back('}');
      break;
    }
  }
}

std::string dump_json(const Value& v) {
  std::string s;
  dump_json(v, s);
  return s;
}

// ---------------------------------------------------------------------------
// msgpack decoder (spec: github.com/msgpack/msgpack/blob/master/spec.md)

namespace {

struct MpReader {
  const uint8_t* p;
  const uint8_t* end;
  std::string err;
  int depth = 0;

  bool need(size_t n) {
    if (static_cast<size_t>(end - p) < n) { err = "truncated msgpack"; return false; }
    return true;
  }
  uint64_t be(int n) {
    uint64_t v = 0;
    for (int k = 0; k < n; ++k) v = (v << 8) | p[k];
    p += n;
    return v;
  }
  bool raw(size_t n, std::string* s) {
    if (!need(n)) return false;
    s->assign(reinterpret_cast<const char*>(p), n);
    p += n;
    return true;
  }
  bool arr(size_t n, Value* v) {
    *v = Value::array();
    v->a->reserve(n < 1 << 20 ? n : 0);
    for (size_t k = 0; k < n; ++k) {
      Value x;
      if (!value(&x)) return false;
      v->a->push_back(std::move(x));
    }
    return true;
  }
  bool map(size_t n, Value* v) {
    *v = Value::object();
    for (size_t k = 0; k < n; ++k) {
      Value key, x;
      if (!value(&key) || !value(&x)) return false;
      std::string ks;
      if (key.is_str() || key.is_bin()) ks = key.s;
      else ks = dump_json(key);
      v->o->emplace_back(std::move(ks), std::move(x));
    }
    return true;
  }
  bool value(Value* v) {
    if (!need(1)) return false;
    if (++depth > 256) { err = "msgpack nesting too deep"; return false; }
    uint8_t c = *p++;
    bool ok = true;
    if (c <= 0x7f) *v = Value::integer(c);
    else if (c >= 0xe0) *v = Value::integer(static_cast<int8_t>(c));
    else if ((c & 0xf0) == 0x80) ok = map(c & 0x0f, v);
    else if ((c & 0xf0) == 0x90) ok = arr(c & 0x0f, v);
    else if ((c & 0xe0) == 0xa0) { std::string s; ok = raw(c & 0x1f, &s); if (ok) *v = Value::string(std::move(s)); }
    else {
      switch (c) {
        case 0xc0: *v = Value(); break;
        case 0xc2: *v = Value::boolean(false); break;
        case 0xc3: *v = Value::boolean(true); break;
        case 0xc4: case 0xc5: case 0xc6: {
          int w = c == 0xc4 ? 1 : c == 0xc5 ? 2 : 4;
          if (!need(w)) { ok = false; break; }
          std::string s;
          ok = raw(be(w), &s);
          if (ok) *v = Value::bin(std::move(s));
          break;
        }
        case 0xc7: case 0xc8: case 0xc9: {  // ext 8/16/32: skip payload
          int w = c == 0xc7 ? 1 : c == 0xc8 ? 2 : 4;
          if (!need(w + 1)) { ok = false; break; }
          size_t n = be(w);
          ++p;
          if (!need(n)) { ok = false; break; }
          p += n;
          *v = Value();
          break;
        }
        case 0xca: {
          if (!need(4)) { ok = false; break; }
          uint32_t bits = static_cast<uint32_t>(be(4));
          float f;
          std::memcpy(&f, &bits, 4);
          *v = Value::number(f);
          break;
        }
        case 0xcb: {
          if (!need(8)) { ok = false; break; }
          uint64_t bits = be(8);
          double f;
          std::memcpy(&f, &bits, 8);
          *v = Value::number(f);
          break;
        }
        case 0xcc: if (!need(1)) { ok = false; break; } *v = Value::uinteger(be(1)); break;
        case 0xcd: if (!need(2)) { ok = false; break; } *v = Value::uinteger(be(2)); break;
        case 0xce: if (!need(4)) { ok = false; break; } *v = Value::uinteger(be(4)); break;
        case 0xcf: if (!need(8)) { ok = false; break; } *v = Value::uinteger(be(8)); break;
        case 0xd0: if (!need(1)) { ok = false; break; } *v = Value::integer(static_cast<int8_t>(be(1))); break;
        case 0xd1: if (!need(2)) { ok = false; break; } *v = Value::integer(static_cast<int16_t>(be(2))); break;
        case 0xd2: if (!need(4)) { ok = false; break; } *v = Value::integer(static_cast<int32_t>(be(4))); break;
        case 0xd3: if (!need(8)) { ok = false; break; } *v = Value::integer(static_cast<int64_t>(be(8))); break;
        case 0xd4: case 0xd5: case 0xd6: case 0xd7: case 0xd8: {  // fixext: skip
          size_t n = size_t(1) << (c - 0xd4);
          if (!need(n + 1)) { ok = false; break; }
          p += n + 1;
          *v = Value();
          break;
        }
        case 0xd9: case 0xda: case 0xdb: {
          int w = c == 0xd9 ? 1 : c == 0xda ? 2 : 4;
          if (!need(w)) { ok = false; break; }
          std::string s;
          ok = raw(be(w), &s);
          if (ok) *v = Value::string(std::move(s));
          break;
        }
        case 0xdc: if (!need(2)) { ok = false; break; } ok = arr(be(2), v); break;
        case 0xdd: if (!need(4)) { ok = false; break; } ok = arr(be(4), v); break;
        case 0xde: if (!need(2)) { ok = false; break; } ok = map(be(2), v); break;
        case 0xdf: if (!need(4)) { ok = false; break; } ok = map(be(4), v); break;
        default: err = "bad msgpack type byte"; ok = false; break;
      }
    }
    --depth;
    return ok;
  }
};

}  // namespace

bool parse_msgpack(const uint8_t* p, size_t n, Value* out, std::string* err) {
  MpReader r{p, p + n, {}};
  if (!r.value(out)) {
    if (err) *err = r.err;
    return false;
  }
  return true;
}

}  // namespace ib
