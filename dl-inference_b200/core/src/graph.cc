// dli.graph.v1 reader/writer. Attribute typing follows the reference reader
// (src/graph.cc:230-273 of yncxcw/dl-inference): JSON bool/int/float/string map
// to bool/int64/double/string; arrays map to int64, double (any non-integer
// element) or string vectors; an empty array is an int64 vector.
#include "dli/graph.h"

#include <fstream>
#include <sstream>
#include <stdexcept>
#include <type_traits>

#include "json.h"

namespace dli {
namespace {

AttributeValue toAttribute(const json::Value& v) {
  using T = json::Value::Type;
  switch (v.type) {
    case T::Bool: return v.b;
    case T::Int: return v.i;
    case T::Number: return v.d;
    case T::String: return v.s;
    case T::Array: {
      if (v.a.empty()) return std::vector<std::int64_t>{};
      bool strings = true, ints = true, numbers = true;
      for (const auto& x : v.a) {
        strings &= x.type == T::String;
        ints &= x.type == T::Int;
        numbers &= x.type == T::Int || x.type == T::Number;
      }
      if (strings) {
        std::vector<std::string> out;
        for (const auto& x : v.a) out.push_back(x.s);
        return out;
      }
      if (ints) {
        std::vector<std::int64_t> out;
        for (const auto& x : v.a) out.push_back(x.i);
        return out;
      }
      if (numbers) {
        std::vector<double> out;
        for (const auto& x : v.a) out.push_back(x.type == T::Int ? static_cast<double>(x.i) : x.d);
        return out;
      }
      break;
    }
    default: break;
  }
  throw std::invalid_argument("unsupported attribute JSON value");
}

void writeStrings(std::ostringstream& out, const std::vector<std::string>& v) {
  out << '[';
  for (std::size_t i = 0; i < v.size(); ++i) out << (i ? "," : "") << '"' << json::escape(v[i]) << '"';
  out << ']';
}

void writeAttribute(std::ostringstream& out, const AttributeValue& value) {
  std::visit(
      [&](const auto& x) {
        using V = std::decay_t<decltype(x)>;
        if constexpr (std::is_same_v<V, std::string>) {
          out << '"' << json::escape(x) << '"';
        } else if constexpr (std::is_same_v<V, bool>) {
          out << (x ? "true" : "false");
        } else if constexpr (std::is_same_v<V, std::int64_t>) {
          out << x;
        } else if constexpr (std::is_same_v<V, double>) {
          std::ostringstream tmp;
          tmp.precision(17);
          tmp << x;
          std::string s = tmp.str();
          if (s.find_first_of(".eEn") == std::string::npos) s += ".0";  // keep it a float on re-read
          out << s;
        } else if constexpr (std::is_same_v<V, std::vector<std::string>>) {
          writeStrings(out, x);
        } else {
          out << '[';
          for (std::size_t i = 0; i < x.size(); ++i) {
            if (i) out << ',';
            if constexpr (std::is_same_v<typename V::value_type, double>) {
              std::ostringstream tmp;
              tmp.precision(17);
              tmp << x[i];
              std::string s = tmp.str();
              if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
              out << s;
            } else {
              out << x[i];
            }
          }
          out << ']';
        }
      },
      value);
}

}  // namespace

Graph Graph::fromJson(const std::string& text) {
  const json::Value root = json::parse(text);
  if (root.type != json::Value::Type::Object) throw std::invalid_argument("graph JSON root must be an object");
  Graph g;
  if (const auto* f = root.find("format")) g.format = json::asString(*f, "format");
  if (g.format != "dli.graph.v1") throw std::invalid_argument("unsupported graph format: " + g.format);
  if (const auto* f = root.find("model_type")) g.model_type = json::asString(*f, "model_type");
  if (const auto* f = root.find("weights")) g.weights = json::asString(*f, "weights");
  if (const auto* f = root.find("inputs")) g.inputs = json::asStringArray(*f, "inputs");
  if (const auto* f = root.find("outputs")) g.outputs = json::asStringArray(*f, "outputs");
  const json::Value& nodes = root.at("nodes");
  if (nodes.type != json::Value::Type::Array) throw std::invalid_argument("graph nodes must be an array");
  g.nodes.reserve(nodes.a.size());
  for (const auto& nj : nodes.a) {
    if (nj.type != json::Value::Type::Object) throw std::invalid_argument("graph node must be an object");
    Node n;
    n.name = json::asString(nj.at("name"), "name");
    if (const auto* op = nj.find("op")) n.op_type = json::asString(*op, "op");
    else n.op_type = json::asString(nj.at("op_type"), "op_type");
    n.inputs = json::asStringArray(nj.at("inputs"), "inputs");
    n.outputs = json::asStringArray(nj.at("outputs"), "outputs");
    if (const auto* attrs = nj.find("attrs")) {
      if (attrs->type != json::Value::Type::Object) throw std::invalid_argument("node attrs must be an object");
      for (const auto& [k, v] : attrs->o) n.attributes.set(k, toAttribute(v));
    }
    g.nodes.push_back(std::move(n));
  }
  return g;
}

Graph Graph::fromJsonFile(const std::string& path) {
  std::ifstream f(path);
  if (!f) throw std::runtime_error("failed to open graph file: " + path);
  std::ostringstream buf;
  buf << f.rdbuf();
  return fromJson(buf.str());
}

std::string Graph::toJson() const {
  std::ostringstream out;
  out << "{\n  \"format\":\"" << json::escape(format) << "\",\n  \"model_type\":\"" << json::escape(model_type)
      << "\",\n";
  if (!weights.empty()) out << "  \"weights\":\"" << json::escape(weights) << "\",\n";
  out << "  \"inputs\":";
  writeStrings(out, inputs);
  out << ",\n  \"outputs\":";
  writeStrings(out, outputs);
  out << ",\n  \"nodes\":[\n";
  for (std::size_t i = 0; i < nodes.size(); ++i) {
    const Node& n = nodes[i];
    out << "    {\"name\":\"" << json::escape(n.name) << "\",\"op\":\"" << json::escape(n.op_type)
        << "\",\"inputs\":";
    writeStrings(out, n.inputs);
    out << ",\"outputs\":";
    writeStrings(out, n.outputs);
    out << ",\"attrs\":{";
    std::size_t k = 0;
    for (const auto& [name, value] : n.attributes.values()) {
      out << (k++ ? "," : "") << '"' << json::escape(name) << "\":";
      writeAttribute(out, value);
    }
    out << "}}" << (i + 1 != nodes.size() ? "," : "") << "\n";
  }
  out << "  ]\n}\n";
  return out.str();
}

}  // namespace dli
