// Minimal JSON document model + recursive-descent parser used by the graph and
// weights-manifest readers. Integers without fraction/exponent parse as Int,
// everything else numeric as Number (the distinction drives attribute typing).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace dli::json {

struct Value {
  enum class Type { Null, Bool, Int, Number, String, Array, Object };
  Type type = Type::Null;
  bool b = false;
  std::int64_t i = 0;
  double d = 0.0;
  std::string s;
  std::vector<Value> a;
  std::map<std::string, Value> o;

  const Value* find(const std::string& key) const;
  const Value& at(const std::string& key) const;  // throws std::invalid_argument
};

Value parse(const std::string& text);
std::string escape(const std::string& s);

std::string asString(const Value& v, const std::string& field);
std::int64_t asInt(const Value& v, const std::string& field);
std::vector<std::string> asStringArray(const Value& v, const std::string& field);
std::vector<std::int64_t> asIntArray(const Value& v, const std::string& field);

}  // namespace dli::json
