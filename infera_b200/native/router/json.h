// JSON / msgpack value model for the native router.
//
// One Value type serves both JSON request bodies and msgpack KV-event
// batches. Objects keep insertion order (request bodies are re-serialised
// with their keys in the client's order). Integers above INT64_MAX (block
// hashes) are kept exactly as unsigned.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace ib {

struct Value;
using Array = std::vector<Value>;
using Object = std::vector<std::pair<std::string, Value>>;

struct Value {
  enum Type : uint8_t { Null, Bool, Int, UInt, Double, String, Bin, Arr, Obj };
  Type t = Null;
  bool b = false;
  int64_t i = 0;
  uint64_t u = 0;
  double d = 0.0;
  std::string s;                 // String or Bin payload
  std::shared_ptr<Array> a;
  std::shared_ptr<Object> o;

  Value() = default;
  static Value null() { return Value(); }
  static Value boolean(bool v) { Value x; x.t = Bool; x.b = v; return x; }
  static Value integer(int64_t v) { Value x; x.t = Int; x.i = v; return x; }
  static Value uinteger(uint64_t v) {
    Value x;
    if (v <= static_cast<uint64_t>(INT64_MAX)) { x.t = Int; x.i = static_cast<int64_t>(v); }
    else { x.t = UInt; x.u = v; }
    return x;
  }
  static Value number(double v) { Value x; x.t = Double; x.d = v; return x; }
  static Value string(std::string v) { Value x; x.t = String; x.s = std::move(v); return x; }
  static Value bin(std::string v) { Value x; x.t = Bin; x.s = std::move(v); return x; }
  static Value array() { Value x; x.t = Arr; x.a = std::make_shared<Array>(); return x; }
  static Value object() { Value x; x.t = Obj; x.o = std::make_shared<Object>(); return x; }

  bool is_null() const { return t == Null; }
  bool is_bool() const { return t == Bool; }
  bool is_int() const { return t == Int || t == UInt; }
  bool is_number() const { return t == Int || t == UInt || t == Double; }
  bool is_str() const { return t == String; }
  bool is_bin() const { return t == Bin; }
  bool is_arr() const { return t == Arr; }
  bool is_obj() const { return t == Obj; }

  int64_t as_int(int64_t dflt = 0) const {
    if (t == Int) return i;
    if (t == UInt) return static_cast<int64_t>(u);
    if (t == Double) return static_cast<int64_t>(d);
    if (t == Bool) return b ? 1 : 0;
    return dflt;
  }
  uint64_t as_u64() const { return t == UInt ? u : static_cast<uint64_t>(as_int()); }
  double as_double(double dflt = 0.0) const {
    if (t == Double) return d;
    if (t == Int) return static_cast<double>(i);
    if (t == UInt) return static_cast<double>(u);
    return dflt;
  }
  bool truthy() const {
    switch (t) {
      case Null: return false;
      case Bool: return b;
      case Int: return i != 0;
      case UInt: return u != 0;
      case Double: return d != 0.0;
      case String: case Bin: return !s.empty();
      case Arr: return a && !a->empty();
      case Obj: return o && !o->empty();
    }
    return false;
  }
  const std::string& str() const { return s; }
  const Array& arr() const { static const Array empty; return a ? *a : empty; }
  const Object& obj() const { static const Object empty; return o ? *o : empty; }

  // object access (nullptr if absent or not an object)
  const Value* get(const std::string& key) const;
  Value* get_mut(const std::string& key);
  void set(const std::string& key, Value v);
  bool erase(const std::string& key);
  void push(Value v) { if (!a) { t = Arr; a = std::make_shared<Array>(); } a->push_back(std::move(v)); }
};

// JSON text -> Value. Returns false (and a message in *err) on malformed input.
bool parse_json(const char* p, size_t n, Value* out, std::string* err);
inline bool parse_json(const std::string& s, Value* out, std::string* err) {
  return parse_json(s.data(), s.size(), out, err);
}
// Value -> compact JSON text (Bin is written as a string of its bytes).
void dump_json(const Value& v, std::string& out);
std::string dump_json(const Value& v);
void json_escape(const std::string& s, std::string& out);

// msgpack bytes -> Value (ext types are skipped as null). Returns false on
// truncated or malformed input.
bool parse_msgpack(const uint8_t* p, size_t n, Value* out, std::string* err);

}  // namespace ib
