// Minimal JSON DOM: parse (RFC 8259, UTF-8, \u escapes incl. surrogate
// pairs) and serialize. Used for tokenizer.json, model contracts and the
// OpenAI / Anthropic request bodies. Numbers keep their integer value when
// they are integral. Reference counterpart: the C JSON DOM declared in
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_json.h:23-54.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace spc {

class Json {
 public:
  enum class Type { Null, Bool, Number, String, Array, Object };
  Json() = default;
  static Json parse(const std::string& text);  // throws StatusError(ParseError)
  std::string dump() const;

  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::Null; }
  bool is_object() const { return type_ == Type::Object; }
  bool is_array() const { return type_ == Type::Array; }
  bool is_string() const { return type_ == Type::String; }
  bool is_number() const { return type_ == Type::Number; }
  bool is_bool() const { return type_ == Type::Bool; }
  bool is_integer() const { return type_ == Type::Number && is_int_; }  // integral literal

  const std::string& str() const;
  double num() const;
  int64_t int64() const;
  bool boolean() const;
  const std::vector<Json>& arr() const;
  const std::vector<std::pair<std::string, Json>>& obj() const;  // insertion order
  const Json* get(const std::string& key) const;                 // nullptr if absent / not an object
  const Json& at(const std::string& key) const;                  // throws SchemaError if absent
  size_t size() const;

  // construction helpers
  static Json make_null() { return Json(); }
  static Json make_bool(bool b);
  static Json make_number(double v);
  static Json make_int(int64_t v);
  static Json make_string(std::string s);
  static Json make_array(std::vector<Json> a = {});
  static Json make_object();
  void push(Json v);                      // array append
  void set(const std::string& k, Json v);  // object insert / replace

 private:
  Type type_ = Type::Null;
  bool b_ = false;
  double d_ = 0.0;
  int64_t i_ = 0;
  bool is_int_ = false;
  std::string s_;
  std::vector<Json> a_;
  std::vector<std::pair<std::string, Json>> o_;
  friend struct JsonParser;
};

std::string json_escape(const std::string& s);

}  // namespace spc
