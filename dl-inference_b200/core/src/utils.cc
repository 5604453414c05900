#include "dli/utils.h"

#include <algorithm>
#include <functional>
#include <numeric>
#include <stdexcept>
#include <type_traits>
#include <variant>

namespace dli {

std::int64_t product(const std::vector<std::int64_t>& shape, std::size_t begin, std::size_t end) {
  end = std::min(end, shape.size());
  if (begin >= end) return 1;
  return std::accumulate(shape.begin() + static_cast<std::ptrdiff_t>(begin),
                         shape.begin() + static_cast<std::ptrdiff_t>(end), std::int64_t{1},
                         std::multiplies<std::int64_t>());
}

std::string formatShape(const std::vector<std::int64_t>& shape) {
  std::string text = "[";
  const char* sep = "";
  for (const std::int64_t d : shape) {
    text += sep;
    text += std::to_string(d);
    sep = ", ";
  }
  return text + "]";
}

void requireCudaInputs(const std::vector<const Tensor*>& inputs, const std::string& op) {
  const bool all_cuda =
      std::all_of(inputs.begin(), inputs.end(), [](const Tensor* t) { return t != nullptr && t->isCuda(); });
  if (!all_cuda) throw std::invalid_argument(op + " expects CUDA tensors");
}

void requireFloat(const Tensor& tensor, const std::string& op) {
  if (isFloating(tensor.dtype())) return;
  throw std::invalid_argument(op + " expects float32, bfloat16 or float16, got " + toString(tensor.dtype()));
}

void requireSameDtype(const Tensor& a, const Tensor& b, const std::string& op) {
  if (a.dtype() == b.dtype()) return;
  throw std::invalid_argument(op + " expects one dtype for its tensors, got " + toString(a.dtype()) + " and " +
                              toString(b.dtype()));
}

double attrDouble(const Attributes& attrs, const std::string& name, double fallback) {
  const auto it = attrs.values().find(name);
  if (it == attrs.values().end()) return fallback;
  return std::visit(
      [&name](const auto& v) -> double {
        using V = std::decay_t<decltype(v)>;
        if constexpr (std::is_same_v<V, double> || std::is_same_v<V, std::int64_t>) {
          return static_cast<double>(v);
        } else {
          throw std::invalid_argument("attribute has unexpected type: " + name);
        }
      },
      it->second);
}

std::vector<std::int64_t> attrInts(const Attributes& attrs, const std::string& name,
                                   std::vector<std::int64_t> fallback) {
  return attrs.contains(name) ? attrs.require<std::vector<std::int64_t>>(name) : std::move(fallback);
}

void* ptr(const Tensor& tensor) { return const_cast<void*>(tensor.deviceData()); }

std::vector<std::int64_t> reshapeShape(const std::vector<std::int64_t>& input,
                                       std::vector<std::int64_t> target) {
  const auto wildcards = std::count(target.begin(), target.end(), std::int64_t{-1});
  if (wildcards > 1) throw std::invalid_argument("reshape has multiple inferred dimensions");
  if (std::any_of(target.begin(), target.end(), [](std::int64_t d) { return d == 0 || d < -1; }))
    throw std::invalid_argument("reshape dimension must be positive or -1");
  const std::int64_t numel = product(input);
  if (wildcards == 1) {
    // the product of the fixed entries is minus the product with the -1 included
    const std::int64_t fixed = -product(target);
    if (numel % fixed != 0) throw std::invalid_argument("reshape inferred dimension is not integral");
    *std::find(target.begin(), target.end(), std::int64_t{-1}) = numel / fixed;
  }
  if (product(target) != numel) throw std::invalid_argument("reshape changes element count");
  return target;
}

}  // namespace dli
