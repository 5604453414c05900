// Node attributes of a dli.graph.v1 node: a name -> value map whose value type
// set and `require`/`value_or` semantics match the reference runtime
// (include/dli/attributes.h:11-45 of yncxcw/dl-inference), so operator code
// written against it reads the same.
#pragma once

#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <variant>
#include <vector>

namespace dli {

using AttributeValue = std::variant<std::int64_t, double, bool, std::string, std::vector<std::int64_t>,
                                    std::vector<double>, std::vector<std::string>>;

class Attributes {
 public:
  void set(std::string name, AttributeValue value) { values_[std::move(name)] = std::move(value); }
  bool contains(const std::string& name) const { return values_.count(name) != 0; }

  template <typename T>
  const T& require(const std::string& name) const {
    const auto it = values_.find(name);
    if (it == values_.end()) throw std::invalid_argument("missing required attribute: " + name);
    if (!std::holds_alternative<T>(it->second))
      throw std::invalid_argument("attribute has unexpected type: " + name);
    return std::get<T>(it->second);
  }

  template <typename T>
  T value_or(const std::string& name, T fallback) const {
    const auto it = values_.find(name);
    if (it == values_.end()) return fallback;
    if (!std::holds_alternative<T>(it->second))
      throw std::invalid_argument("attribute has unexpected type: " + name);
    return std::get<T>(it->second);
  }

  const std::map<std::string, AttributeValue>& values() const { return values_; }

 private:
  std::map<std::string, AttributeValue> values_;
};

}  // namespace dli
