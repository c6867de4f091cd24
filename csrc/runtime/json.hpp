// Minimal JSON value + parser + serializer for the runtime library (no external dependency).
// Numbers keep an integer flag so u64 fields (versions, token counts, indices) round-trip exactly.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace dtj {

struct Value;
using Object = std::vector<std::pair<std::string, Value>>;  // insertion-ordered
using Array = std::vector<Value>;

struct Value {
  enum Kind { Null, Bool, Int, Double, String, Arr, Obj } kind = Null;
  bool b = false;
  int64_t i = 0;
  double d = 0;
  std::string s;
  std::shared_ptr<Array> a;
  std::shared_ptr<Object> o;

  Value() = default;
  static Value null() { return Value(); }
  static Value boolean(bool v) { Value x; x.kind = Bool; x.b = v; return x; }
  static Value integer(int64_t v) { Value x; x.kind = Int; x.i = v; x.d = (double)v; return x; }
  static Value number(double v) { Value x; x.kind = Double; x.d = v; return x; }
  static Value string(std::string v) { Value x; x.kind = String; x.s = std::move(v); return x; }
  static Value array() { Value x; x.kind = Arr; x.a = std::make_shared<Array>(); return x; }
  static Value object() { Value x; x.kind = Obj; x.o = std::make_shared<Object>(); return x; }

  bool is_null() const { return kind == Null; }
  bool is_num() const { return kind == Int || kind == Double; }
  double num() const { return kind == Int ? (double)i : d; }
  int64_t as_int() const { return kind == Int ? i : (int64_t)d; }
  const Value* find(const std::string& k) const {
    if (kind != Obj) return nullptr;
    for (auto& kv : *o)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  const Value& at(const std::string& k) const {
    const Value* v = find(k);
    if (!v) throw std::runtime_error("missing key: " + k);
    return *v;
  }
  Value& set(const std::string& k, Value v) {
    for (auto& kv : *o)
      if (kv.first == k) { kv.second = std::move(v); return kv.second; }
    o->emplace_back(k, std::move(v));
    return o->back().second;
  }
  void push(Value v) { a->push_back(std::move(v)); }
};

Value parse(const char* p, size_t n);
inline Value parse(const std::string& s) { return parse(s.data(), s.size()); }
void dump(const Value& v, std::string& out);
inline std::string dump(const Value& v) { std::string s; dump(v, s); return s; }
void dump_string(const std::string& s, std::string& out);
void dump_double(double d, std::string& out);

}  // namespace dtj
