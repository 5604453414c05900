#include "json.h"

#include <cctype>
#include <cstdlib>
#include <stdexcept>

namespace dli::json {

const Value* Value::find(const std::string& key) const {
  if (type != Type::Object) return nullptr;
  const auto it = o.find(key);
  return it == o.end() ? nullptr : &it->second;
}

const Value& Value::at(const std::string& key) const {
  const Value* v = find(key);
  if (v == nullptr) throw std::invalid_argument("missing JSON field: " + key);
  return *v;
}

namespace {

class Parser {
 public:
  explicit Parser(const std::string& text) : t_(text) {}

  Value document() {
    Value v = value();
    ws();
    if (p_ != t_.size()) error("trailing characters");
    return v;
  }

 private:
  [[noreturn]] void error(const std::string& what) const {
    throw std::invalid_argument("invalid JSON at offset " + std::to_string(p_) + ": " + what);
  }
  void ws() {
    while (p_ < t_.size() && std::isspace(static_cast<unsigned char>(t_[p_]))) ++p_;
  }
  char peek() {
    ws();
    if (p_ >= t_.size()) error("unexpected end");
    return t_[p_];
  }
  void expect(char c) {
    if (peek() != c) error(std::string("expected '") + c + "'");
    ++p_;
  }
  bool literal(const char* word) {
    const std::string w(word);
    if (t_.compare(p_, w.size(), w) == 0) {
      p_ += w.size();
      return true;
    }
    return false;
  }

  Value value() {
    const char c = peek();
    if (c == '{') return object();
    if (c == '[') return array();
    if (c == '"') {
      Value v;
      v.type = Value::Type::String;
      v.s = string();
      return v;
    }
    Value v;
    if (literal("true")) { v.type = Value::Type::Bool; v.b = true; return v; }
    if (literal("false")) { v.type = Value::Type::Bool; v.b = false; return v; }
    if (literal("null")) return v;
    return number();
  }

  Value object() {
    Value v;
    v.type = Value::Type::Object;
    expect('{');
    if (peek() == '}') { ++p_; return v; }
    while (true) {
      if (peek() != '"') error("expected object key");
      std::string key = string();
      expect(':');
      v.o[key] = value();
      const char c = peek();
      ++p_;
      if (c == '}') break;
      if (c != ',') error("expected ',' or '}'");
    }
    return v;
  }

  Value array() {
    Value v;
    v.type = Value::Type::Array;
    expect('[');
    if (peek() == ']') { ++p_; return v; }
    while (true) {
      v.a.push_back(value());
      const char c = peek();
      ++p_;
      if (c == ']') break;
      if (c != ',') error("expected ',' or ']'");
    }
    return v;
  }

  static void utf8(std::string& out, unsigned cp) {
    if (cp < 0x80) {
      out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }

  std::string string() {
    expect('"');
    std::string out;
    while (true) {
      if (p_ >= t_.size()) error("unterminated string");
      const char c = t_[p_++];
      if (c == '"') break;
      if (c != '\\') { out.push_back(c); continue; }
      if (p_ >= t_.size()) error("bad escape");
      const char e = t_[p_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (p_ + 4 > t_.size()) error("bad \\u escape");
          utf8(out, static_cast<unsigned>(std::stoul(t_.substr(p_, 4), nullptr, 16)));
          p_ += 4;
          break;
        }
        default: error("bad escape");
      }
    }
    return out;
  }

  Value number() {
    const std::size_t start = p_;
    bool is_float = false;
    if (p_ < t_.size() && (t_[p_] == '-' || t_[p_] == '+')) ++p_;
    while (p_ < t_.size()) {
      const char c = t_[p_];
      if (std::isdigit(static_cast<unsigned char>(c))) { ++p_; continue; }
      if (c == '.' || c == 'e' || c == 'E' || c == '-' || c == '+') { is_float = true; ++p_; continue; }
      break;
    }
    if (start == p_) error("unexpected character");
    const std::string tok = t_.substr(start, p_ - start);
    Value v;
    try {
      if (is_float) {
        v.type = Value::Type::Number;
        v.d = std::stod(tok);
      } else {
        v.type = Value::Type::Int;
        v.i = std::stoll(tok);
      }
    } catch (const std::exception&) {
      error("bad number '" + tok + "'");
    }
    return v;
  }

  const std::string& t_;
  std::size_t p_ = 0;
};

}  // namespace

Value parse(const std::string& text) { return Parser(text).document(); }

std::string escape(const std::string& s) {
  std::string out;
  out.reserve(s.size());
  for (const char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\t': out += "\\t"; break;
      case '\r': out += "\\r"; break;
      default: out.push_back(c);
    }
  }
  return out;
}

std::string asString(const Value& v, const std::string& field) {
  if (v.type != Value::Type::String) throw std::invalid_argument("JSON field must be a string: " + field);
  return v.s;
}

std::int64_t asInt(const Value& v, const std::string& field) {
  if (v.type != Value::Type::Int) throw std::invalid_argument("JSON field must be an integer: " + field);
  return v.i;
}

std::vector<std::string> asStringArray(const Value& v, const std::string& field) {
  if (v.type != Value::Type::Array) throw std::invalid_argument("JSON field must be a string array: " + field);
  std::vector<std::string> out;
  for (const auto& x : v.a) out.push_back(asString(x, field));
  return out;
}

std::vector<std::int64_t> asIntArray(const Value& v, const std::string& field) {
  if (v.type != Value::Type::Array) throw std::invalid_argument("JSON field must be an integer array: " + field);
  std::vector<std::int64_t> out;
  for (const auto& x : v.a) out.push_back(asInt(x, field));
  return out;
}

}  // namespace dli::json
